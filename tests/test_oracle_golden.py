"""Pin the CPU oracle (C restatement) against the reference's own outputs.

The golden vectors in tests/golden were produced by the reference's unmodified
C++/OpenMP path (tests/golden/make_golden.py).  With the same thread count the
restatement must reproduce them bit for bit.
"""
import numpy as np
import pytest

from helpers import em_golden_names, load_golden, param_errors
from oracle import oracle

EM = em_golden_names()


@pytest.mark.parametrize("name", EM)
def test_flash_em_fused_bitwise(name):
    g = load_golden(name)
    out = oracle.flash_em_fused(g["X"], g["mu"], g["var"], g["log_pi"], BK=int(g["BK"]),
                                nthreads=int(g["nthreads"]))
    for key, got in zip(["new_mu", "new_var", "new_log_pi", "log_normalizer"], out):
        assert np.array_equal(got, g[key]), f"{name}:{key} differs from the reference"


def test_fit20_trajectory_bitwise():
    g = load_golden("c1_fit20")
    mu, var, lp = g["mu0"], g["var0"], g["log_pi0"]
    lls = []
    for _ in range(20):
        mu, var, lp, ln = oracle.flash_em_fused(g["X"], mu, var, lp, BK=8, nthreads=int(g["nthreads"]))
        lls.append(float(ln.astype(np.float32).mean(dtype=np.float32)))
    assert np.array_equal(mu, g["mu"]) and np.array_equal(var, g["var"]) and np.array_equal(lp, g["log_pi"])
    assert np.allclose(lls, g["ll"], rtol=0, atol=1e-5)


def test_estep_ops_bitwise():
    g = load_golden("estep_c1_1024")
    nt = int(g["nthreads"])
    gam, ln = oracle.standard_e_step(g["X"], g["mu"], g["var"], g["log_pi"], nthreads=nt)
    assert np.array_equal(gam, g["gamma"]) and np.array_equal(ln, g["log_normalizer"])
    fg, fln = oracle.flash_e_step(g["X"], g["mu"], g["var"], g["log_pi"], BK=4, nthreads=nt)
    assert np.array_equal(fg, g["flash_gamma"]) and np.array_equal(fln, g["flash_log_normalizer"])
    m = oracle.standard_m_step(g["X"], g["gamma"], nthreads=nt)
    # reference uses BLAS GEMMs: agreement to fp32 rounding, not bitwise
    assert np.allclose(m[0], g["m_mu"], rtol=1e-5, atol=1e-5)
    assert np.allclose(m[1], g["m_var"], rtol=1e-4, atol=1e-4)
    assert np.allclose(m[2], g["m_log_pi"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", ["c1_iter1", "c2_slice2048", "edge_n257_k129_d33"])
def test_fp64_restatement_close_to_reference(name):
    """The fp64 yardstick and the fp32 reference agree to fp32 noise."""
    g = load_golden(name)
    r64 = oracle.flash_em_fused_f64(g["X"], g["mu"], g["var"], g["log_pi"], with_stats=True)
    N = g["X"].shape[0]
    e = param_errors([g["new_mu"], g["new_var"], g["new_log_pi"], g["log_normalizer"]], r64[:4],
                     n_k=r64[4], N=N)
    assert e["ln"] < 5e-3 and e["log_pi"] < 1e-3 and e["mu"] < 1e-2, e


@pytest.mark.parametrize("name", ["c3_fit20_n16384"])
def test_fit20_fixture_pinned(name):
    """The 20-iteration fixtures store no X: the regenerated workload must match the
    stored digest, and the first step of the bit-exact restatement (and of the fp64
    restatement) must reproduce the stored first log-likelihoods."""
    import hashlib
    from flashgmm_b200.data import make_workload
    g = load_golden(name)
    X, *_ = make_workload(str(g["workload"]), N=int(g["N"]))
    assert hashlib.sha256(X.numpy().tobytes()).hexdigest() == str(g["x_sha256"])
    out = oracle.flash_em_fused(X, g["mu0"], g["var0"], g["log_pi0"], BK=8, nthreads=int(g["nthreads"]))
    assert abs(float(np.mean(out[3].astype(np.float64))) - float(g["ll"][0])) < 1e-9
    r = oracle.flash_em_fused_f64(X, g["mu0"], g["var0"], g["log_pi0"])
    assert abs(float(np.mean(r[3])) - float(g["ll64"][0])) < 1e-9
