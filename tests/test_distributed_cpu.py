"""Sharded-fit host logic on CPU `gloo` ranks (world size 2).

The statistics backend is swapped for an fp64 CPU restatement (oracle), so these tests
exercise the row split, the single all_reduce of the packed statistics, the replicated
M-step and the failure paths -- everything but the CUDA kernels -- without a GPU.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashgmm_b200.distributed import DistributedFlashGMM, ShardedFitError, split_rows


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def cpu_stats(X, mu, var, log_pi, state):
    from oracle import oracle
    r = oracle.flash_em_fused_f64(X, mu, var, log_pi, nthreads=2, with_stats=True)
    ln = r[3]
    stats = np.concatenate([r[4], r[5].ravel(), r[6].ravel(), [ln.sum()]])
    return torch.from_numpy(stats), torch.from_numpy(ln)


def cpu_update(stats, n_total, K, d):
    s = stats.double()
    n = s[:K]
    sk = s[K:K + K * d].reshape(K, d)
    qk = s[K + K * d:K + 2 * K * d].reshape(K, d)
    inv = 1.0 / n.clamp_min(1e-8)
    mu = sk * inv[:, None]
    var = (qk * inv[:, None] - mu * mu).clamp_min(1e-6)
    lp = (n / n_total).clamp_min(1e-8).log()
    return mu.float(), var.float(), lp.float()


def _data():
    from flashgmm_b200.data import make_mixture, init_params
    X, *_ = make_mixture(600, 4, 6, seed=11)
    mu, var, lp = init_params(X, 4, seed=2)
    return X, (mu, var, lp)


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        X, init = _data()
        a, b = split_rows(X.shape[0], world, rank)
        if mode == "bad_init" and rank == 1:
            init = (init[0] + 1.0, init[1], init[2])
        m = DistributedFlashGMM(4, 6, max_iter=5, tol=0.0, stats_fn=cpu_stats, update_fn=cpu_update)
        if mode == "die" and rank == 1:
            q.put((rank, "died"))
            q.close()
            q.join_thread()  # flush before the abrupt exit
            os._exit(0)  # leaves between steps, before the first collective of the fit
        try:
            m.fit(X[a:b], init)
            q.put((rank, "ok", m.mu.numpy(), m.var.numpy(), m.log_pi.numpy()))
        except ShardedFitError as e:
            q.put((rank, "error", str(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(world):
        item = q.get(timeout=120)
        out[item[0]] = item[1:]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_split_rows_covers_everything():
    for n in [1, 7, 600, 65536]:
        for w in [1, 2, 3, 8]:
            r = [split_rows(n, w, k) for k in range(w)]
            assert r[0][0] == 0 and r[-1][1] == n
            assert all(r[k][1] == r[k + 1][0] for k in range(w - 1))


def test_sharded_fit_equals_single_process():
    out = _run("ok")
    X, init = _data()
    mu, var, lp = init
    n_total = float(X.shape[0])
    for _ in range(5):
        stats, _ = cpu_stats(X, mu, var, lp, {})
        mu, var, lp = cpu_update(stats, n_total, 4, 6)
    for r in (0, 1):
        assert out[r][0] == "ok"
        np.testing.assert_allclose(out[r][1], mu.numpy(), rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(out[r][2], var.numpy(), rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(out[r][3], lp.numpy(), rtol=1e-6, atol=1e-6)
    # replicated parameters are bitwise identical across ranks
    assert all(np.array_equal(out[0][i], out[1][i]) for i in (1, 2, 3))


def test_dead_rank_surfaces_as_error_on_peer():
    out = _run("die")
    assert out[1][0] == "died"
    assert out[0][0] == "error" and "all_reduce failed" in out[0][1]


def test_mismatched_initial_parameters_rejected():
    out = _run("bad_init")
    assert out[0][0] == "error" and out[1][0] == "error"
    assert "differ" in out[0][1]
