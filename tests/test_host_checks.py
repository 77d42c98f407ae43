"""Argument checking in the drop-in op module (raises before any compute; no GPU needed)."""
import pytest
import torch

from flashgmm_b200 import flash_gmm_native as C


def _params(N=16, K=4, d=8, dtype=torch.float32):
    return (torch.randn(N, d, dtype=dtype), torch.randn(K, d, dtype=dtype),
            torch.ones(K, d, dtype=dtype), torch.zeros(K, dtype=dtype))


def test_rejects_non_float32():
    with pytest.raises(RuntimeError, match="float32"):
        C.flash_em_fused(*_params(dtype=torch.float64))


def test_rejects_non_2d():
    X, mu, var, lp = _params()
    with pytest.raises(RuntimeError, match="2D"):
        C.flash_em_fused(X.reshape(-1), mu, var, lp)


def test_rejects_cpu_tensors_no_fallback():
    with pytest.raises(RuntimeError, match="CUDA"):
        C.flash_em_fused(*_params())


def test_defaults_match_reference_signature():
    import inspect
    sig = inspect.signature(C.flash_em_fused)
    assert list(sig.parameters) == ["X", "mu", "var", "log_pi", "BN", "BK"]
    assert sig.parameters["BN"].default == 64 and sig.parameters["BK"].default == 8
