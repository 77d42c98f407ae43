"""Device-resident iteration loop: ``NativeFlashGMM.fit(graph_iters=G)`` replays a CUDA
graph of G iterations and applies the stopping rule afterwards; it must reproduce the
one-iteration-at-a-time loop (which follows ``flash_gmm/native_wrapper.py:123-148``)
exactly: same history, same parameters, same log-normalizer."""
import numpy as np
import pytest
import torch

from helpers import load_golden

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("max_iter,tol", [(23, 0.0), (40, 1e-3)])
def test_graph_loop_equals_eager_loop(max_iter, tol):
    from flashgmm_b200.native_wrapper import NativeFlashGMM
    g = load_golden("c2_slice2048")
    dev = torch.device("cuda:0")
    X = torch.from_numpy(g["X"]).to(dev)
    init = [torch.from_numpy(g[k]).to(dev) for k in ("mu", "var", "log_pi")]
    K, d = init[0].shape
    a = NativeFlashGMM(K, d, max_iter=max_iter, tol=tol)
    ha = a.fit(X, init=init, graph_iters=0)
    b = NativeFlashGMM(K, d, max_iter=max_iter, tol=tol)
    hb = b.fit(X, init=init, graph_iters=10)
    assert len(ha) == len(hb)
    if tol > 0:
        assert len(ha) < max_iter, "the tolerance should stop the fit early"
    assert [h["log_likelihood"] for h in ha] == [h["log_likelihood"] for h in hb]
    for x, y in ((a.mu, b.mu), (a.var, b.var), (a.log_pi, b.log_pi)):
        assert torch.equal(x, y)
    assert torch.equal(a.log_normalizer, b.log_normalizer)
