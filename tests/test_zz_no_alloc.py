"""fgmm_em_fused_static: the fused EM iteration for callers that cannot allocate.

Code that runs inside another framework's memory pool, or a process whose device
footprint must stay fixed once it has started, cannot call cudaMalloc; this entry point
serves them from a fixed 16 MiB device array compiled into the library.  The test calls
it through the C ABI (ctypes, raw device pointers, no torch on the call path) twice in a
row and compares each result with the regular entry point fgmm_em_fused, run on the same
kernel family with a caller-provided workspace, within the parity tolerances the other
GPU tests use.  It lives in its own file, collected last, and passes alone in a fresh
process as well as after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import load_golden, param_errors

pytestmark = pytest.mark.gpu

TOL = {"mu": 1e-4, "var": 1e-4, "var_abs": 4e-6, "log_pi": 1e-4, "ln": 1e-3}


def _outs(K, d, N, dev):
    return [torch.empty(K, d, device=dev), torch.empty(K, d, device=dev),
            torch.empty(K, device=dev), torch.empty(N, device=dev)]


def _call_static(lib, X, mu, var, lp, outs, stream):
    N, d = X.shape
    K = mu.shape[0]
    return lib.fgmm_em_fused_static(X.data_ptr(), N, d, mu.data_ptr(), var.data_ptr(),
                                    lp.data_ptr(), K, outs[0].data_ptr(), outs[1].data_ptr(),
                                    outs[2].data_ptr(), outs[3].data_ptr(), stream)


def _call_regular(lib, X, mu, var, lp, outs, stream):
    N, d = X.shape
    K = mu.shape[0]
    nbytes = lib.fgmm_em_fused_workspace_bytes(N, d, K)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=X.device)
    return lib.fgmm_em_fused(X.data_ptr(), N, d, mu.data_ptr(), var.data_ptr(), lp.data_ptr(),
                             K, outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(),
                             outs[3].data_ptr(), ws.data_ptr(), nbytes, stream)


@pytest.mark.parametrize("name", ["c2_slice2048", "edge_n257_k129_d33"])
def test_static_scratch_matches_regular_entry_point(name):
    from flashgmm_b200 import _lib
    lib = _lib.load()
    g = load_golden(name)
    dev = torch.device("cuda:0")
    X, mu, var, lp = (torch.from_numpy(np.ascontiguousarray(g[k])).to(dev)
                      for k in ("X", "mu", "var", "log_pi"))
    N, d = X.shape
    K = mu.shape[0]
    stream = torch.cuda.current_stream(dev).cuda_stream
    prev = lib.fgmm_set_family(_lib.FAMILY_SIMT)  # the family the static variant runs
    try:
        want = _outs(K, d, N, dev)
        _lib.check(_call_regular(lib, X, mu, var, lp, want, stream))
        for _ in range(2):  # the array keeps the previous call's contents
            got = _outs(K, d, N, dev)
            _lib.check(_call_static(lib, X, mu, var, lp, got, stream))
            torch.cuda.synchronize(dev)
            w = [t.double().cpu().numpy() for t in want]
            e = param_errors([t.cpu().numpy() for t in got], w)
            assert all(e[k] <= TOL[k] for k in TOL), e
    finally:
        lib.fgmm_set_family(prev)


def test_static_scratch_rejects_oversized_shapes():
    from flashgmm_b200 import _lib
    lib = _lib.load()
    # K=4096, d=256 needs > 16 MiB of scratch: rejected before anything is launched
    rc = lib.fgmm_em_fused_static(ctypes.c_void_p(16), 1 << 20, 256, ctypes.c_void_p(16),
                                  ctypes.c_void_p(16), ctypes.c_void_p(16), 4096,
                                  ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
                                  ctypes.c_void_p(16), None)
    assert rc == _lib.FGMM_ERR_WORKSPACE
    assert b"16777216" in lib.fgmm_last_error()
