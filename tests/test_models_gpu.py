"""The Python model layer on the GPU against the reference's own Python models.

Fixtures (``tests/golden/pymodel_*.npz``, made by ``make_golden.py models``) hold the
reference's ``FlashGMM`` (``flash_gmm/flash_gmm.py``) and ``StandardGMM``
(``flash_gmm/standard_gmm.py``) run on the CPU: 20-iteration histories (mean
log-likelihood and simulated IO bytes per iteration), final parameters, and one
``e_step`` / ``m_step`` pair from the reference initialisation.  The data is the
reference generator's (N=4,096, K=8, d=32, seed 0), regenerated here by
``generate_gmm_data`` and checked against a digest.
"""
import numpy as np
import pytest
import torch

from helpers import load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _data(g):
    import hashlib
    from flashgmm_b200.standard_gmm import generate_gmm_data
    X = generate_gmm_data(4096, 8, 32)[0]
    assert hashlib.sha256(X.numpy().tobytes()).hexdigest() == str(g["x_sha256"])
    return X.to(DEV)


def _close_params(model, g, tol_mu=1e-4, tol_var=1e-3, tol_lp=1e-4):
    mu, var, lp = (t.double().cpu().numpy() for t in (model.mu, model.var, model.log_pi))
    scale = np.maximum(np.abs(g["mu"]), np.sqrt(g["var"]))
    assert np.max(np.abs(mu - g["mu"]) / scale) < tol_mu
    assert np.max(np.abs(var - g["var"]) / g["var"]) < tol_var
    assert np.max(np.abs(lp - g["log_pi"])) < tol_lp


def test_flash_gmm_fit_matches_reference_model():
    from flashgmm_b200.flash_gmm import FlashGMM
    g = load_golden("pymodel_flash_c1")
    X = _data(g)
    m = FlashGMM(K=8, d=32, BK=4, max_iter=20, tol=0.0)
    h = m.fit(X)
    assert len(h) == 20
    assert [e["io_bytes"] for e in h] == [int(v) for v in g["io_bytes"]]
    assert np.max(np.abs(np.array([e["log_likelihood"] for e in h]) - g["ll"])) < 1e-3
    _close_params(m, g)
    lab = m.predict(X)
    gamma = m.predict_proba(X)
    assert gamma.shape == (4096, 8)
    assert torch.allclose(gamma.sum(1), torch.ones(4096, device=DEV), atol=1e-5)
    assert torch.equal(lab, gamma.argmax(1))


def test_standard_gmm_fit_matches_reference_model():
    from flashgmm_b200.standard_gmm import StandardGMM
    g = load_golden("pymodel_standard_c1")
    X = _data(g)
    m = StandardGMM(K=8, d=32, max_iter=20, tol=0.0)
    h = m.fit(X)
    assert len(h) == 20
    assert [e["io_bytes"] for e in h] == [int(v) for v in g["io_bytes"]]
    assert np.max(np.abs(np.array([e["log_likelihood"] for e in h]) - g["ll"])) < 1e-3
    _close_params(m, g)


def test_e_step_m_step_methods_match_reference():
    from flashgmm_b200.standard_gmm import StandardGMM
    g = load_golden("pymodel_steps_c1")
    X = _data(g)
    m = StandardGMM(K=8, d=32, seed=5)
    m._init_params(X)
    # the reference initialisation: the same points, the same variance up to the
    # device's summation order
    assert np.array_equal(m.mu.cpu().numpy(), g["mu0"])
    assert np.allclose(m.var.cpu().numpy(), g["var0"], rtol=1e-5)
    assert np.array_equal(m.log_pi.cpu().numpy(), g["log_pi0"])
    m.mu, m.var, m.log_pi = (torch.from_numpy(g[k]).to(DEV) for k in ("mu0", "var0", "log_pi0"))
    gamma, log_ll = m.e_step(X)
    assert np.max(np.abs(gamma.cpu().numpy() - g["gamma"])) < 1e-4
    assert np.max(np.abs(log_ll.cpu().numpy() - g["log_ll"])) < 1e-3
    m.m_step(X, torch.from_numpy(g["gamma"]).to(DEV))
    _close_params(m, g)


def test_top_level_module_runs_the_cuda_op():
    """``import flash_gmm_native as _C`` (the reference wrapper's import) gets the CUDA op."""
    import flash_gmm_native as _C
    g = load_golden("c1_iter1")
    t = [torch.from_numpy(g[k]).to(DEV) for k in ("X", "mu", "var", "log_pi")]
    out = _C.flash_em_fused(*t, 64, 8)
    assert len(out) == 4 and all(o.is_cuda for o in out)
    ln = out[3].cpu().numpy()
    assert np.max(np.abs(ln - g["log_normalizer"])) < 1e-3


def test_compiled_op_module_matches_the_c_abi_path():
    """The compiled extension's ops (what ``import flash_gmm_native`` exports) give the same
    bits as the ctypes binding of the same C ABI."""
    import flash_gmm_native as top
    from flashgmm_b200 import flash_gmm_native as C
    g = load_golden("c2_slice2048")
    t = [torch.from_numpy(g[k]).to(DEV) for k in ("X", "mu", "var", "log_pi")]
    for a, b in zip(top.flash_em_fused(*t), C.flash_em_fused(*t)):
        assert torch.equal(a, b)
    ga, la = top.standard_e_step(*t)
    gb, lb = C.standard_e_step(*t)
    assert torch.equal(ga, gb) and torch.equal(la, lb)
    fa = top.flash_e_step(*t, BK=4)
    assert torch.equal(fa[0], gb)
    for a, b in zip(top.standard_m_step(t[0], ga), C.standard_m_step(t[0], gb)):
        assert torch.equal(a, b)
    with pytest.raises(RuntimeError):
        top.flash_em_fused(t[0].double(), *t[1:])
