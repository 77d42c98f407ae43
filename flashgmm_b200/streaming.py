"""EM over a data set kept in host memory, for N x d beyond what the GPU holds.

The reference's precedent is its N-chunk streaming experiment
(``flash_gmm/flash_gmm_v9.py:145-261``: chunks of X copied host-to-device on a second
stream while the previous chunk computes).  Here every iteration streams X through two
device chunk buffers: the copy of chunk i + 1 (pinned host memory, a copy stream) runs
while ``em_stats`` processes chunk i on the compute stream; the packed fp64 statistics
of the chunks are summed on the device and one ``em_update`` per iteration applies
them.  Statistics are sums over points, so the result equals the in-memory fit up to the
order of the fp64 additions.
"""
import time

import torch

from . import _lib
from . import flash_gmm_native as _C


class StreamingFlashGMM:
    """``NativeFlashGMM`` for ``X`` in host memory.  ``fit(X_host)`` accepts a CPU tensor
    (pinned on entry if it is not) and keeps at most two chunks of ``chunk_points`` rows,
    plus their operand buffers, on the GPU."""

    def __init__(self, K: int, d: int, max_iter: int = 100, tol: float = 1e-4, seed: int = 42,
                 chunk_points: int = 1 << 20, device=None):
        self.K = K
        self.d = d
        self.max_iter = max_iter
        self.tol = tol
        self.seed = seed
        self.chunk_points = int(chunk_points)
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.mu = None
        self.var = None
        self.log_pi = None

    def _init_params(self, X):
        """The reference's initialisation (``flash_gmm/native_wrapper.py:115-121``) with the
        random point indices drawn on the host (X is not on the GPU)."""
        N = X.shape[0]
        gen = torch.Generator().manual_seed(self.seed)
        idx = torch.randperm(N, generator=gen)[:self.K]
        mu = X[idx].clone()
        v = 0.0
        for c0 in range(0, N, self.chunk_points):  # per-dimension variance, chunked, in fp64
            v += X[c0:c0 + self.chunk_points].double().pow(2).sum(0)
        mean = X.double().sum(0) / N
        gvar = (v / N - mean * mean) * N / max(N - 1, 1)
        var = torch.ones(self.K, self.d) * float(gvar.mean())
        lp = torch.full((self.K,), -float(torch.log(torch.tensor(float(self.K)))))
        return mu.to(self.device), var.to(self.device), lp.to(self.device)

    def fit(self, X: torch.Tensor, verbose: bool = False, init=None):
        if X.is_cuda:
            raise RuntimeError("StreamingFlashGMM.fit takes X in host memory")
        X = X.contiguous()
        if not X.is_pinned():
            X = X.pin_memory()
        N, d = X.shape
        if d != self.d:
            raise RuntimeError(f"X has d={d}, model has d={self.d}")
        dev = self.device
        if init is not None:
            self.mu, self.var, self.log_pi = (t.to(dev).contiguous().clone() for t in init)
        else:
            self.mu, self.var, self.log_pi = self._init_params(X)
        C = min(self.chunk_points, N)
        bounds = [(c0, min(c0 + C, N)) for c0 in range(0, N, C)]
        with torch.cuda.device(dev):
            bufs = [torch.empty(C, d, dtype=torch.float32, device=dev) for _ in range(2)]
            copy = torch.cuda.Stream(dev)
            comp = torch.cuda.current_stream(dev)
            landed = [torch.cuda.Event() for _ in range(2)]
            freed = [torch.cuda.Event() for _ in range(2)]
            workspaces = {}
            acc = torch.zeros(_C.stats_len(self.K, d), dtype=torch.float64, device=dev)

            def issue_copy(i):
                b = i % 2
                c0, c1 = bounds[i]
                with torch.cuda.stream(copy):
                    copy.wait_event(freed[b])
                    bufs[b][:c1 - c0].copy_(X[c0:c1], non_blocking=True)
                    landed[b].record(copy)

            prev_ll = -float("inf")
            history = []
            for it in range(self.max_iter):
                t0 = time.time()
                acc.zero_()
                issue_copy(0)
                for i, (c0, c1) in enumerate(bounds):
                    if i + 1 < len(bounds):
                        issue_copy(i + 1)
                    b = i % 2
                    comp.wait_event(landed[b])
                    n = c1 - c0
                    ws = workspaces.get(n)
                    if ws is None:
                        ws = workspaces[n] = _C.StatsWorkspace(n, d, self.K, dev)
                    Xc = bufs[b][:n]
                    stats, _ = _C.em_stats(Xc, self.mu, self.var, self.log_pi, workspace=ws)
                    acc.add_(stats)
                    freed[b].record(comp)
                self.mu, self.var, self.log_pi = _C.em_update(acc, N, self.K, d)
                avg_ll = acc[-1].item() / N
                _lib.check_device_error()
                elapsed = time.time() - t0
                history.append({"iter": it, "log_likelihood": avg_ll, "time_ms": elapsed * 1000})
                if verbose and (it % 10 == 0 or it < 5):
                    print(f"  iter {it:3d}: LL={avg_ll:.4f}  time={elapsed*1000:.1f}ms")
                if abs(avg_ll - prev_ll) < self.tol:
                    if verbose:
                        print(f"  Converged at iter {it}")
                    break
                prev_ll = avg_ll
        return history
