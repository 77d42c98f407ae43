"""Generate golden vectors by running the REFERENCE's own CPU path.

Runs ``flash_em_fused`` / ``standard_e_step`` / ``flash_e_step`` /
``standard_m_step`` from the reference's ``flash_gmm/csrc/binding.cpp`` +
``flash_gmm_cpu.cpp``, compiled unmodified by ``oracle/build_ref.py`` into
``oracle/_ref/``, on seeded inputs, and stores inputs and outputs in
``tests/golden/*.npz``.  The reference tree is needed only to regenerate; the
committed fixtures are what the tests read.

Usage:  python tests/golden/make_golden.py   (after ``python oracle/build_ref.py``)
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle.build_ref import load_ref  # noqa: E402
from flashgmm_b200.data import make_mixture, init_params, make_workload  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
NTHREADS = 8  # the reference's per-thread stat buffers make fp32 results thread-count dependent

# name: (N, K, d, seed, mean_scale)
EM_CASES = {
    "c1_iter1": ("c1", None),
    "c2_slice2048": ("c2", 2048),
    "c3_slice4096": ("c3", 4096),
    "c4_slice1024": ("c4", 1024),
    "c5_slice2048": ("c5", 2048),
}
EDGE_CASES = {  # (N, K, d)
    "edge_n1_k1_d1": (1, 1, 1),
    "edge_n7_k3_d7": (7, 3, 7),
    "edge_n130_k17_d1": (130, 17, 1),
    "edge_n257_k129_d33": (257, 129, 33),
    "edge_n100_k5_d256": (100, 5, 256),
    "edge_n300_k40_d100": (300, 40, 100),
}


# 20-iteration trajectories at the headline shapes (name: (workload, N))
FIT20_CASES = {
    "c2_fit20_n16384": ("c2", 16384),
    "c3_fit20_n16384": ("c3", 16384),
    "c4_fit20_n16384": ("c4", 16384),
}
PARAM_KEYS = ("mu", "var", "var_abs", "log_pi")


def x_digest(X):
    """SHA-256 of X's bytes: the fit20 fixtures regenerate X with flashgmm_b200.data and
    check it against this digest instead of storing it."""
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(X.numpy() if hasattr(X, "numpy") else X,
                                               dtype=np.float32).tobytes()).hexdigest()


def fit20_case(R, wl, N, iters=20):
    """The reference op driven 20 times from explicit initial parameters (as
    NativeFlashGMM.fit drives flash_em_fused, flash_gmm/native_wrapper.py:128-146, without
    early stopping), the fp64 restatement driven the same way, and the reference's own
    error against the fp64 trajectory: its largest one-step error (each step started from
    the fp64 trajectory's parameters) and its error after all iterations."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from helpers import param_errors
    from oracle import oracle
    X, mu, var, lp = make_workload(wl, N=N)
    mu0, var0, lp0 = mu.clone(), var.clone(), lp.clone()
    lls = []
    for _ in range(iters):
        mu, var, lp, ln = R.flash_em_fused(X, mu, var, lp, 64, 8)
        lls.append(float(ln.double().mean()))
    zeros = np.zeros(N)
    m64, v64, l64 = mu0.numpy(), var0.numpy(), lp0.numpy()
    one_step = {k: 0.0 for k in PARAM_KEYS}
    ll64 = []
    for _ in range(iters):
        r = oracle.flash_em_fused_f64(X, m64, v64, l64, with_stats=True)
        ll64.append(float(np.mean(r[3])))
        one = R.flash_em_fused(X, torch.from_numpy(np.float32(m64)), torch.from_numpy(np.float32(v64)),
                               torch.from_numpy(np.float32(l64)), 64, 8)
        e = param_errors([a.numpy() for a in one[:3]] + [zeros], [r[0], r[1], r[2], zeros], n_k=r[4], N=N)
        one_step = {k: max(one_step[k], e[k]) for k in PARAM_KEYS}
        m64, v64, l64 = (a.astype(np.float32) for a in r[:3])
    e20 = param_errors([mu.numpy(), var.numpy(), lp.numpy(), zeros], [r[0], r[1], r[2], zeros],
                       n_k=r[4], N=N)
    return dict(x_sha256=x_digest(X), workload=wl, N=N, mu0=mu0, var0=var0, log_pi0=lp0,
                ll=np.array(lls), mu=mu, var=var, log_pi=lp, ll64=np.array(ll64),
                mu64=r[0], var64=r[1], log_pi64=r[2], nk64=r[4],
                one_step=np.array([one_step[k] for k in PARAM_KEYS]),
                err20=np.array([e20[k] for k in PARAM_KEYS]), param_keys=np.array(PARAM_KEYS),
                nthreads=NTHREADS)


def models_cases():
    """Outputs of the reference's pure-Python models and data generator
    (flash_gmm/standard_gmm.py, flash_gmm/flash_gmm.py), imported from the reference tree."""
    from oracle.build_ref import default_reference_root
    ref = os.path.join(default_reference_root(), "flash_gmm")
    sys.path.insert(0, ref)
    import standard_gmm as R_std
    import flash_gmm as R_flash
    out = {}
    for (N, K, d, seed) in ((300, 5, 7, 3), (4096, 8, 32, 0)):
        X, lab, tm, tv, tp = R_std.generate_gmm_data(N, K, d, seed=seed)
        arrs = dict(labels=lab, true_mu=tm, true_var=tv, true_pi=tp, x_sha256=x_digest(X))
        if N <= 1024:
            arrs["X"] = X
        out[f"gen_n{N}_k{K}_d{d}_s{seed}"] = arrs
    X = R_std.generate_gmm_data(4096, 8, 32)[0]
    m = R_flash.FlashGMM(K=8, d=32, BK=4, max_iter=20, tol=0.0)
    h = m.fit(X)
    out["pymodel_flash_c1"] = dict(x_sha256=x_digest(X), ll=np.array([e["log_likelihood"] for e in h]),
                                   io_bytes=np.array([e["io_bytes"] for e in h]), mu=m.mu, var=m.var,
                                   log_pi=m.log_pi)
    s = R_std.StandardGMM(K=8, d=32, max_iter=20, tol=0.0)
    h = s.fit(X)
    out["pymodel_standard_c1"] = dict(x_sha256=x_digest(X), ll=np.array([e["log_likelihood"] for e in h]),
                                      io_bytes=np.array([e["io_bytes"] for e in h]), mu=s.mu, var=s.var,
                                      log_pi=s.log_pi)
    # one e_step / m_step from the reference initialisation
    s = R_std.StandardGMM(K=8, d=32, seed=5)
    s._init_params(X)
    mu0, var0, lp0 = s.mu.clone(), s.var.clone(), s.log_pi.clone()
    gamma, log_ll = s.e_step(X)
    s.m_step(X, gamma)
    out["pymodel_steps_c1"] = dict(x_sha256=x_digest(X), mu0=mu0, var0=var0, log_pi0=lp0, gamma=gamma,
                                   log_ll=log_ll, mu=s.mu, var=s.var, log_pi=s.log_pi)
    return out


def _save(name, **arrs):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **{k: (v.numpy() if hasattr(v, "numpy") else np.asarray(v))
                                 for k, v in arrs.items()})
    print("wrote", path, os.path.getsize(path))


def main(only=None):
    torch.set_num_threads(NTHREADS)
    R = load_ref()
    if only == "models":
        for name, arrs in models_cases().items():
            _save(name, **arrs)
        return
    if only == "fit20":
        for name, (wl, N) in FIT20_CASES.items():
            _save(name, **fit20_case(R, wl, N))
        return
    for name, (wl, N) in EM_CASES.items():
        X, mu, var, lp = make_workload(wl, N=N)
        nm, nv, nl, ln = R.flash_em_fused(X, mu, var, lp, 64, 8)
        _save(name, X=X, mu=mu, var=var, log_pi=lp, new_mu=nm, new_var=nv,
              new_log_pi=nl, log_normalizer=ln, nthreads=NTHREADS, BK=8)
    for name, (N, K, d) in EDGE_CASES.items():
        X, *_ = make_mixture(N, K, d, seed=N + K + d)
        mu, var, lp = init_params(X, K, seed=7) if K <= N else (None, None, None)
        if mu is None:
            g = torch.Generator().manual_seed(7)
            mu = torch.randn(K, d, generator=g) * 3
            var = torch.ones(K, d)
            lp = torch.full((K,), -float(np.log(K)))
        # a non-trivial variance so the log-det term is exercised
        var = var * (0.5 + torch.rand(K, d, generator=torch.Generator().manual_seed(9)))
        nm, nv, nl, ln = R.flash_em_fused(X, mu, var, lp, 64, 8)
        _save(name, X=X, mu=mu, var=var, log_pi=lp, new_mu=nm, new_var=nv,
              new_log_pi=nl, log_normalizer=ln, nthreads=NTHREADS, BK=8)
    for name, arrs in models_cases().items():
        _save(name, **arrs)
    # 20-iteration trajectory on workload c1 through the reference op, as
    # NativeFlashGMM.fit drives it (flash_gmm/native_wrapper.py:128-146) but
    # from explicit initial parameters and without early stopping.
    X, mu, var, lp = make_workload("c1")
    mu0, var0, lp0 = mu.clone(), var.clone(), lp.clone()
    lls = []
    for _ in range(20):
        mu, var, lp, ln = R.flash_em_fused(X, mu, var, lp, 64, 8)
        lls.append(float(ln.mean()))
    _save("c1_fit20", X=X, mu0=mu0, var0=var0, log_pi0=lp0, mu=mu, var=var, log_pi=lp,
          ll=np.array(lls), nthreads=NTHREADS)
    # materialising E-step / M-step ops
    X, mu, var, lp = make_workload("c1", N=1024)
    g, ln = R.standard_e_step(X, mu, var, lp)
    fg, fln = R.flash_e_step(X, mu, var, lp, 4)
    m_mu, m_var, m_lp = R.standard_m_step(X, g)
    _save("estep_c1_1024", X=X, mu=mu, var=var, log_pi=lp, gamma=g, log_normalizer=ln,
          flash_gamma=fg, flash_log_normalizer=fln, m_mu=m_mu, m_var=m_var, m_log_pi=m_lp,
          nthreads=NTHREADS)
    for name, (wl, N) in FIT20_CASES.items():
        _save(name, **fit20_case(R, wl, N))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else None)
