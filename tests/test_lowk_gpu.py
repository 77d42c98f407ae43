"""GPU parity of the fused low-K family (K <= 16, d <= 128; one statistics launch).

Shapes cover its code paths: several 128-point tiles per block and many blocks, one and
two components per phase-2 thread, d not a multiple of 4 (scalar staging), ragged tile
tails.  Each case is compared with the reference's fp32 algorithm (the C restatement)
and the fp64 restatement under the same rule and tolerances as the golden cases
(test_parity_gpu.check, slack 1.5 as for the other fp32 CUDA-core family).
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from test_parity_gpu import SLACK_BY_FAMILY, check

pytestmark = pytest.mark.gpu

SHAPES = [(300000, 8, 32),   # ~2,300 tiles: several per block
          (5000, 16, 128),   # two components per phase-2 thread
          (3001, 9, 116),    # two per thread, five component groups, ragged tail
          (2000, 12, 33),    # d % 4 != 0: scalar staging, padded dimensions
          (129, 1, 4),       # one component, one full tile and one point
          (4096, 8, 32)]     # configuration 1's shape


@pytest.fixture
def lowk():
    from flashgmm_b200 import flash_gmm_native as C, _lib
    prev = C.set_family(_lib.FAMILY_LOWK)
    yield C
    C.set_family(prev)


@pytest.mark.parametrize("N,K,d", SHAPES)
def test_lowk_matches_reference(lowk, N, K, d):
    from flashgmm_b200.data import make_mixture, init_params
    C = lowk
    assert C.family_for(N, d, K) == 3
    dev = torch.device("cuda:0")
    X, *_ = make_mixture(N, K, d, seed=N + 13 * K + d)
    mu, var, lp = init_params(X, K, seed=2)
    var = var * (0.5 + torch.rand(K, d, generator=torch.Generator().manual_seed(7)))
    got = [o.cpu().numpy() for o in C.flash_em_fused(X.to(dev), mu.to(dev), var.to(dev), lp.to(dev))]
    for a in got:
        assert np.all(np.isfinite(a))
    g = {"X": X.numpy(), "mu": mu.numpy(), "var": var.numpy(), "log_pi": lp.numpy()}
    ref = oracle.flash_em_fused(X, mu, var, lp, BK=8, nthreads=8)
    g.update(new_mu=ref[0], new_var=ref[1], new_log_pi=ref[2], log_normalizer=ref[3])
    check(f"lowk N={N} K={K} d={d}", got, g, SLACK_BY_FAMILY["lowk"])


def test_lowk_step_split_and_shards(lowk):
    """em_step == em_stats + em_update, and the statistics of two halves add up to the
    whole's (the all-reduce invariant of a sharded fit)."""
    from flashgmm_b200.data import make_mixture, init_params
    C = lowk
    dev = torch.device("cuda:0")
    X, *_ = make_mixture(20000, 8, 32, seed=5)
    mu, var, lp = (t.to(dev) for t in init_params(X, 8, seed=1))
    X = X.to(dev)
    stats, ln = C.em_stats(X, mu, var, lp)
    stats, ln = stats.clone(), ln.clone()
    upd = C.em_update(stats, X.shape[0], 8, 32)
    nm, nv, nl, st2, ln2 = C.em_step(X, mu, var, lp)
    for a, b in zip((nm, nv, nl), upd):
        assert torch.equal(a, b)
    assert torch.equal(st2, stats) and torch.equal(ln2, ln)
    h = X.shape[0] // 2
    a = C.em_stats(X[:h], mu, var, lp)[0].clone()
    b = C.em_stats(X[h:], mu, var, lp)[0].clone()
    rel = ((a + b) - stats).abs() / stats.abs().clamp_min(1e-3)
    assert rel.max().item() < 1e-4
