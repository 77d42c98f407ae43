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


def _save(name, **arrs):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **{k: (v.numpy() if hasattr(v, "numpy") else np.asarray(v))
                                 for k, v in arrs.items()})
    print("wrote", path, os.path.getsize(path))


def main():
    torch.set_num_threads(NTHREADS)
    R = load_ref()
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


if __name__ == "__main__":
    main()
