"""ctypes front end for ``liboracle.so`` (the C restatement in ``flashgmm_oracle.c``).

Test infrastructure only.  All arrays are host numpy / CPU torch tensors.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)


def build():
    cc = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
    subprocess.check_call(["make", "-s", "-C", HERE, f"CC={cc}", "liboracle.so"])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        i64, i32 = ctypes.c_int64, ctypes.c_int
        L.oracle_flash_em_fused_f32.argtypes = [_f32p, i64, i32, _f32p, _f32p, _f32p, i32, i32, i32,
                                                _f32p, _f32p, _f32p, _f32p]
        L.oracle_flash_em_fused_f64.argtypes = [_f32p, i64, i32, _f32p, _f32p, _f32p, i32, i32,
                                                _f64p, _f64p, _f64p, _f64p, _f64p, _f64p, _f64p]
        L.oracle_standard_e_step_f32.argtypes = [_f32p, i64, i32, _f32p, _f32p, _f32p, i32, i32, _f32p, _f32p]
        L.oracle_flash_e_step_f32.argtypes = [_f32p, i64, i32, _f32p, _f32p, _f32p, i32, i32, i32, _f32p, _f32p]
        L.oracle_standard_m_step_f32.argtypes = [_f32p, i64, i32, _f32p, i32, i32, _f32p, _f32p, _f32p]
        L.oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _np32(a):
    if hasattr(a, "detach"):
        a = a.detach().cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float32)


def _p32(a):
    return a.ctypes.data_as(_f32p)


def _p64(a):
    return a.ctypes.data_as(_f64p)


def max_threads():
    return lib().oracle_max_threads()


def flash_em_fused(X, mu, var, log_pi, BK=8, nthreads=None):
    """fp32 restatement of ``flash_em_fused_cpu`` -> (new_mu, new_var, new_log_pi, log_norm)."""
    X, mu, var, lp = map(_np32, (X, mu, var, log_pi))
    N, d = X.shape
    K = mu.shape[0]
    nm = np.empty((K, d), np.float32); nv = np.empty((K, d), np.float32)
    nl = np.empty(K, np.float32); ln = np.empty(N, np.float32)
    lib().oracle_flash_em_fused_f32(_p32(X), N, d, _p32(mu), _p32(var), _p32(lp), K, BK,
                                    nthreads or max_threads(), _p32(nm), _p32(nv), _p32(nl), _p32(ln))
    return nm, nv, nl, ln


def flash_em_fused_f64(X, mu, var, log_pi, nthreads=None, with_stats=False):
    """Same algorithm in fp64 -> (new_mu, new_var, new_log_pi, log_norm[, n_k, s_k, sq_k])."""
    X, mu, var, lp = map(_np32, (X, mu, var, log_pi))
    N, d = X.shape
    K = mu.shape[0]
    nm = np.empty((K, d)); nv = np.empty((K, d)); nl = np.empty(K); ln = np.empty(N)
    nk = np.empty(K); sk = np.empty((K, d)); qk = np.empty((K, d))
    lib().oracle_flash_em_fused_f64(_p32(X), N, d, _p32(mu), _p32(var), _p32(lp), K,
                                    nthreads or max_threads(), _p64(nm), _p64(nv), _p64(nl), _p64(ln),
                                    _p64(nk), _p64(sk), _p64(qk))
    if with_stats:
        return nm, nv, nl, ln, nk, sk, qk
    return nm, nv, nl, ln


def standard_e_step(X, mu, var, log_pi, nthreads=None):
    X, mu, var, lp = map(_np32, (X, mu, var, log_pi))
    N, d = X.shape
    K = mu.shape[0]
    g = np.empty((N, K), np.float32); ln = np.empty(N, np.float32)
    lib().oracle_standard_e_step_f32(_p32(X), N, d, _p32(mu), _p32(var), _p32(lp), K,
                                     nthreads or max_threads(), _p32(g), _p32(ln))
    return g, ln


def flash_e_step(X, mu, var, log_pi, BK=4, nthreads=None):
    X, mu, var, lp = map(_np32, (X, mu, var, log_pi))
    N, d = X.shape
    K = mu.shape[0]
    g = np.empty((N, K), np.float32); ln = np.empty(N, np.float32)
    lib().oracle_flash_e_step_f32(_p32(X), N, d, _p32(mu), _p32(var), _p32(lp), K, BK,
                                  nthreads or max_threads(), _p32(g), _p32(ln))
    return g, ln


def standard_m_step(X, gamma, nthreads=None):
    X, g = _np32(X), _np32(gamma)
    N, d = X.shape
    K = g.shape[1]
    nm = np.empty((K, d), np.float32); nv = np.empty((K, d), np.float32); nl = np.empty(K, np.float32)
    lib().oracle_standard_m_step_f32(_p32(X), N, d, _p32(g), K, nthreads or max_threads(),
                                     _p32(nm), _p32(nv), _p32(nl))
    return nm, nv, nl
