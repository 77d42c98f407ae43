"""Drop-in for the reference's ``flash_gmm/native_wrapper.py`` model classes
(``NativeFlashGMM`` and ``NativeStandardGMM``).

``NativeFlashGMM(K, d, BN=64, BK=8, max_iter=100, tol=1e-4, seed=42).fit(X)``
keeps the reference's constructor, attributes (``mu``, ``var``, ``log_pi``),
initialisation (``_init_params``, ``native_wrapper.py:115-121``), per-iteration
history entries and stopping rule (``|ΔLL| < tol``, ``native_wrapper.py:123-148``).

What changes underneath: X's tensor-core operand rows are prepared once per fit
(X does not change between iterations) and scratch is allocated once, so each
iteration is the fused statistics launch sequence plus the M-step, all on the
current stream.  The reference's per-iteration ``log_norm.mean().item()`` host
sync is kept because the stopping rule needs it; ``fit`` also accepts a CPU
tensor and copies it to the GPU first.
"""
import time

import torch

from . import _lib
from . import flash_gmm_native as _C


class _EMModel:
    """What both model classes share: the reference's initialisation
    (``flash_gmm/native_wrapper.py:64-70, 115-121``), moving X to the GPU, and
    ``predict_proba`` / ``predict`` (``flash_gmm/flash_gmm.py:185-193``)."""

    def _init_params(self, X: torch.Tensor):
        N = X.shape[0]
        gen = torch.Generator(device=X.device).manual_seed(self.seed)
        idx = torch.randperm(N, generator=gen, device=X.device)[:self.K]
        self.mu = X[idx].clone()
        self.var = torch.ones(self.K, self.d, device=X.device) * X.var(dim=0, keepdim=True).mean()
        self.log_pi = torch.full((self.K,), -torch.log(torch.tensor(float(self.K))).item(),
                                 device=X.device)

    def _to_device(self, X):
        if X.is_cuda:
            return X
        dev = torch.device(self.device) if self.device is not None else torch.device("cuda")
        if X.is_pinned():
            return X.to(dev, non_blocking=True)
        return X.to(dev)

    def predict_proba(self, X: torch.Tensor) -> torch.Tensor:
        """Responsibilities gamma[N, K] under the fitted parameters (the E-step op)."""
        X = self._to_device(X).contiguous()
        gamma, _ = _C.flash_e_step(X, self.mu, self.var, self.log_pi)
        return gamma

    def predict(self, X: torch.Tensor) -> torch.Tensor:
        return self.predict_proba(X).argmax(dim=1)


class NativeStandardGMM(_EMModel):
    """Standard EM (materialised L and gamma) on this package's CUDA kernels.

    Drop-in for ``NativeStandardGMM`` (``flash_gmm/native_wrapper.py:48-96``): same
    constructor, initialisation, history and stopping rule; each iteration is
    ``standard_e_step`` then ``standard_m_step``.
    """

    def __init__(self, K: int, d: int, max_iter: int = 100, tol: float = 1e-4, seed: int = 42,
                 device=None):
        self.K = K
        self.d = d
        self.max_iter = max_iter
        self.tol = tol
        self.seed = seed
        self.device = device
        self.mu = None
        self.var = None
        self.log_pi = None

    def fit(self, X: torch.Tensor, verbose: bool = False, init=None):
        """Run EM; ``init=(mu, var, log_pi)`` overrides the random initialisation."""
        X = self._to_device(X).contiguous()
        if init is not None:
            self.mu, self.var, self.log_pi = (t.to(X.device).contiguous() for t in init)
        else:
            self._init_params(X)
        prev_ll = -float("inf")
        history = []
        for it in range(self.max_iter):
            t0 = time.time()
            gamma, log_norm = _C.standard_e_step(X, self.mu, self.var, self.log_pi)
            avg_ll = log_norm.mean().item()
            _lib.check_device_error()
            self.mu, self.var, self.log_pi = _C.standard_m_step(X, gamma)
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


class NativeFlashGMM(_EMModel):
    """Flash-GMM EM on B200 kernels: each iteration is the fused statistics launch
    sequence plus the M-step; the N x K responsibilities are never returned or kept."""

    def __init__(self, K: int, d: int, BN: int = 64, BK: int = 8,
                 max_iter: int = 100, tol: float = 1e-4, seed: int = 42, device=None):
        self.K = K
        self.d = d
        self.BN = BN
        self.BK = BK
        self.max_iter = max_iter
        self.tol = tol
        self.seed = seed
        self.device = device
        self.mu = None
        self.var = None
        self.log_pi = None

    def fit(self, X: torch.Tensor, verbose: bool = False, init=None, graph_iters: int = 10):
        """Run EM; ``init=(mu, var, log_pi)`` overrides the random initialisation.

        ``graph_iters > 1`` runs the iterations as replays of one CUDA graph holding that
        many iterations (statistics + in-place update, and a copy of each iteration's
        log-likelihood and parameters into device history buffers), so the host
        synchronises once per replay instead of once per iteration.  The stopping rule is
        then applied to the replayed iterations in order and the parameters are restored to
        those of the stopping iteration: results equal the one-iteration-at-a-time loop
        (``graph_iters <= 1``), which follows the reference exactly.
        """
        X = self._to_device(X).contiguous()
        if init is not None:
            self.mu, self.var, self.log_pi = (t.to(X.device).contiguous().clone() for t in init)
        else:
            self._init_params(X)
        N = X.shape[0]
        points = _C.prepare_points(X, self.K)
        ws = _C.StatsWorkspace(N, self.d, self.K, X.device)
        # the tensor-core family reuses the operands each step leaves for the next one
        self._reuse = _C.family_for(N, self.d, self.K) == 2
        if graph_iters and graph_iters > 1 and self.max_iter > 1:
            return self._fit_graph(X, N, points, ws, verbose, int(graph_iters))
        prev_ll = -float("inf")
        history = []
        for it in range(self.max_iter):
            t0 = time.time()
            # from the second iteration on, the parameters are the previous step's outputs,
            # whose tensor-core operands that step already left in the workspace
            self.mu, self.var, self.log_pi, stats, log_norm = _C.em_step(
                X, self.mu, self.var, self.log_pi, points=points, workspace=ws,
                prepared=self._reuse and it > 0)
            avg_ll = stats[-1].item() / N
            _lib.check_device_error()
            self.log_normalizer = log_norm
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

    def _fit_graph(self, X, N, points, ws, verbose, G):
        dev = X.device
        K, d = self.K, self.d
        mu, var, lp = self.mu.clone(), self.var.clone(), self.log_pi.clone()
        h_ll = torch.empty(G, dtype=torch.float64, device=dev)
        h_mu = torch.empty(G, K, d, dtype=torch.float32, device=dev)
        h_var = torch.empty(G, K, d, dtype=torch.float32, device=dev)
        h_lp = torch.empty(G, K, dtype=torch.float32, device=dev)
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            # one-time setup inside the library (kernel attributes) happens outside capture
            _C.em_stats(X, mu, var, lp, points=points, workspace=ws)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(G):
                    _, _, _, stats, log_norm = _C.em_step(X, mu, var, lp, points=points,
                                                          workspace=ws, out=(mu, var, lp),
                                                          prepared=self._reuse and i > 0)
                    h_ll[i].copy_(stats[-1])
                    h_mu[i].copy_(mu)
                    h_var[i].copy_(var)
                    h_lp[i].copy_(lp)
        torch.cuda.current_stream(dev).wait_stream(stream)
        prev_ll = -float("inf")
        history = []
        done = False
        it = 0
        last = 0
        start = (mu.clone(), var.clone(), lp.clone())
        while it < self.max_iter and not done:
            start = (mu.clone(), var.clone(), lp.clone())  # parameters entering this replay
            t0 = time.time()
            graph.replay()
            lls = (h_ll / N).tolist()  # one synchronisation per replay
            _lib.check_device_error()
            elapsed = (time.time() - t0) * 1000 / G
            for i in range(G):
                if it >= self.max_iter:
                    break
                history.append({"iter": it, "log_likelihood": lls[i], "time_ms": elapsed})
                if verbose and (it % 10 == 0 or it < 5):
                    print(f"  iter {it:3d}: LL={lls[i]:.4f}  time={elapsed:.1f}ms")
                last = i
                it += 1
                if abs(lls[i] - prev_ll) < self.tol:
                    if verbose:
                        print(f"  Converged at iter {it - 1}")
                    done = True
                    break
                prev_ll = lls[i]
        # a replay may have run past the stopping iteration: take its parameters, and its
        # log-normalizer (computed from the parameters it started from)
        self.mu, self.var, self.log_pi = h_mu[last].clone(), h_var[last].clone(), h_lp[last].clone()
        before = (h_mu[last - 1], h_var[last - 1], h_lp[last - 1]) if last > 0 else start
        _, ln = _C.em_stats(X, *before, points=points, workspace=ws)
        self.log_normalizer = ln.clone()
        return history
