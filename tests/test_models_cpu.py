"""Host-side parts of the Python model layer, checked against outputs of the
reference's own Python code (fixtures made by ``tests/golden/make_golden.py models``):
the data generator, the IO counter and the op module's top-level name."""
import hashlib

import numpy as np
import torch

from helpers import load_golden


def _digest(X):
    return hashlib.sha256(np.ascontiguousarray(X.numpy(), dtype=np.float32).tobytes()).hexdigest()


def test_generate_gmm_data_matches_reference():
    from flashgmm_b200.standard_gmm import generate_gmm_data
    for name, args in (("gen_n300_k5_d7_s3", (300, 5, 7, 3)), ("gen_n4096_k8_d32_s0", (4096, 8, 32, 0))):
        g = load_golden(name)
        X, lab, tm, tv, tp = generate_gmm_data(*args[:3], seed=args[3])
        assert _digest(X) == str(g["x_sha256"])
        if "X" in g:
            assert np.array_equal(X.numpy(), g["X"])
        assert np.array_equal(lab.numpy(), g["labels"])
        for a, k in ((tm, "true_mu"), (tv, "true_var"), (tp, "true_pi")):
            assert np.array_equal(a.numpy(), g[k])


def test_io_counter_semantics():
    from flashgmm_b200.standard_gmm import IOCounter
    io = IOCounter()
    io.record("X", torch.zeros(10, 4), "read")
    io.record("X", torch.zeros(10, 4), "read")
    io.record("g", torch.zeros(3, dtype=torch.float64), "write")
    assert (io.reads, io.writes, io.total()) == (320, 24, 344)
    assert io.details == {"read:X": 320, "write:g": 24}
    assert io.summary().startswith("Total IO: 0.00 MB")
    io.reset()
    assert io.total() == 0 and io.details == {}


def test_top_level_op_module_names():
    import flash_gmm_native as _C
    for name in ("flash_em_fused", "standard_e_step", "flash_e_step", "standard_m_step"):
        assert callable(getattr(_C, name))
    # CUDA only: a CPU tensor is refused with a RuntimeError, as the reference's TORCH_CHECKs do
    X = torch.zeros(4, 2)
    try:
        _C.flash_em_fused(X, torch.zeros(1, 2), torch.ones(1, 2), torch.zeros(1))
    except RuntimeError as e:
        assert "CUDA" in str(e) or "cuda" in str(e)
    else:
        raise AssertionError("CPU tensors must be refused")
