"""Sharded EM over several GPUs of one node (one process per GPU).

The reference has no multi-GPU code.  The points are independent given the
parameters, so N is split across ranks: every rank runs Pass 1 + Pass 2 on its own
rows (:func:`flash_gmm_native.em_stats`), the packed fp64 statistics
``[n_k | s_k | sq_k | sum ln]`` (K(2d+1)+1 values, ~0.5 MB at K=256, d=128) are
summed with one ``all_reduce`` (NCCL over NVLink), and every rank applies the same
M-step (:func:`flash_gmm_native.em_update`) to the global sums, so the parameters
stay replicated with no broadcast.  The log-normalizers stay sharded.

Failure handling: every collective runs under the process group's timeout; a rank
that dies or stops participating makes the others' next ``all_reduce`` raise, and
``fit`` re-raises it as :class:`ShardedFitError` naming the iteration.  Nothing here
waits on the GPU without that bound.
"""
import time

import torch
import torch.distributed as dist


class ShardedFitError(RuntimeError):
    """A collective of the sharded fit failed (peer gone, timeout, or backend error)."""


def split_rows(n_total, world, rank):
    """Contiguous row range ``[start, stop)`` of rank ``rank`` (first ranks get the remainder)."""
    base, rem = divmod(n_total, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def _gpu_stats(X, mu, var, log_pi, state):
    from . import flash_gmm_native as C
    if "points" not in state:
        state["points"] = C.prepare_points(X, mu.shape[0])
        state["ws"] = C.StatsWorkspace(X.shape[0], X.shape[1], mu.shape[0], X.device)
        state["tc"] = C.family_for(X.shape[0], X.shape[1], mu.shape[0]) == 2
    stats, ln = C.em_stats(X, mu, var, log_pi, points=state["points"], workspace=state["ws"],
                           prepared=state.get("prepared", False))
    return stats, ln


def _gpu_update(stats, n_total, K, d, state=None):
    """The M-step after the all-reduce.  On the tensor-core family the same launch writes
    the next step's parameter operands into this rank's workspace (one launch instead of
    an update plus a preparation)."""
    from . import flash_gmm_native as C
    if state is not None and state.get("tc"):
        out = C.em_update_prepared(stats, n_total, state["points"], state["ws"])
        state["prepared"] = True
        return out
    return C.em_update(stats, n_total, K, d)


class DistributedFlashGMM:
    """EM over a row-sharded data set.  Drop-in counterpart of ``NativeFlashGMM`` whose
    ``fit`` takes this rank's rows; all ranks must call ``fit`` together.

    ``stats_fn(X, mu, var, log_pi, state) -> (stats fp64 [K(2d+1)+1], log_norm)`` and
    ``update_fn(stats, n_total, K, d) -> (mu, var, log_pi)`` default to the CUDA ops;
    tests substitute CPU versions to exercise the sharding and collective logic on
    ``gloo`` ranks.
    """

    def __init__(self, K, d, max_iter=100, tol=1e-4, group=None, stats_fn=None, update_fn=None):
        self.K = K
        self.d = d
        self.max_iter = max_iter
        self.tol = tol
        self.group = group
        self.stats_fn = stats_fn or _gpu_stats
        self.update_fn = update_fn or _gpu_update
        self.mu = self.var = self.log_pi = None
        self.log_normalizer = None

    def _allreduce(self, t, it):
        try:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        except Exception as e:  # peer failure, timeout, backend error
            raise ShardedFitError(f"all_reduce failed at iteration {it}: {e}") from e
        return t

    def fit(self, X_local, init, verbose=False):
        """Run EM.  ``init = (mu, var, log_pi)`` must be identical on every rank (e.g.
        drawn from a shared seed); it is checked with one collective."""
        mu, var, log_pi = (t.to(X_local.device).contiguous() for t in init)
        n_local = torch.tensor([float(X_local.shape[0])], dtype=torch.float64, device=X_local.device)
        n_total = self._allreduce(n_local.clone(), -1).item()
        chk = torch.stack([mu.double().sum(), var.double().sum(), log_pi.double().sum()])
        mine = chk.clone()
        self._allreduce(chk, -1)
        world = dist.get_world_size(self.group)
        if not torch.allclose(chk, mine * world, rtol=1e-12, atol=0.0):
            raise ShardedFitError("initial parameters differ between ranks")
        state = {}
        prev_ll = -float("inf")
        history = []
        for it in range(self.max_iter):
            t0 = time.time()
            stats, ln = self.stats_fn(X_local, mu, var, log_pi, state)
            stats = self._allreduce(stats.clone(), it)
            if self.update_fn is _gpu_update:
                mu, var, log_pi = self.update_fn(stats, n_total, self.K, self.d, state=state)
            else:
                mu, var, log_pi = self.update_fn(stats, n_total, self.K, self.d)
            avg_ll = stats[-1].item() / n_total
            if X_local.is_cuda and self.stats_fn is _gpu_stats:
                from . import _lib
                _lib.check_device_error()
            self.log_normalizer = ln
            history.append({"iter": it, "log_likelihood": avg_ll,
                            "time_ms": (time.time() - t0) * 1000})
            if verbose and dist.get_rank(self.group) == 0 and (it % 10 == 0 or it < 5):
                print(f"  iter {it:3d}: LL={avg_ll:.4f}")
            if abs(avg_ll - prev_ll) < self.tol:
                break
            prev_ll = avg_ll
        self.mu, self.var, self.log_pi = mu, var, log_pi
        return history
