"""Drop-in for the reference's pure-Python fused model ``flash_gmm/flash_gmm.py``
(``FlashGMM``): E and M fused, no N x K matrix materialised by the model.

``FlashGMM(K, d, BK=4, max_iter=100, tol=1e-4, seed=42)`` keeps the reference's
constructor, attributes (``mu``, ``var``, ``log_pi``, ``io_counter``), initialisation,
history entries (with ``io_bytes``) and stopping rule.  Each ``_fused_em_step`` is
this package's CUDA statistics pass (Pass 1 log-normalizer + Pass 2 statistics,
``em_stats``) followed by the reference model's own update (``flash_gmm.py:162-169``:
mu = s/n, var = clamp(sq/n - mu^2, 1e-6), log_pi = log(n/N), no floor on n), applied by
``em_update(..., floors=False)``.  ``BK`` (the reference's component tile) is accepted
and only shapes the simulated IO records, as it does there; the kernels' tiles are
fixed.  ``predict_proba`` / ``predict`` use the GPU ``flash_e_step`` op.
"""
import time

import torch

from . import _lib
from . import flash_gmm_native as _C
from .standard_gmm import IOCounter, init_params_like_reference


class FlashGMM:
    """Flash-GMM with diagonal covariance on this package's CUDA kernels."""

    def __init__(self, K: int, d: int, BK: int = 4, max_iter: int = 100, tol: float = 1e-4,
                 seed: int = 42, device=None):
        self.K = K
        self.d = d
        self.BK = BK
        self.max_iter = max_iter
        self.tol = tol
        self.seed = seed
        self.device = device
        self.mu = None
        self.var = None
        self.log_pi = None
        self.io_counter = IOCounter()
        self._cache = None  # (X pointer, shape) -> prepared operands and scratch

    def _to_device(self, X):
        if X.is_cuda:
            return X.contiguous()
        dev = torch.device(self.device) if self.device is not None else torch.device("cuda")
        return X.to(dev).contiguous()

    def _init_params(self, X: torch.Tensor):
        self.mu, self.var, self.log_pi = init_params_like_reference(X, self.K, self.d, self.seed)

    def _operands(self, X):
        key = (X.data_ptr(), tuple(X.shape), X.device)
        if self._cache is None or self._cache[0] != key:
            N, d = X.shape
            self._cache = (key, _C.prepare_points(X, self.K), _C.StatsWorkspace(N, d, self.K, X.device))
        return self._cache[1], self._cache[2]

    def _record_io(self, X):
        """The reference model's simulated IO for one fused step (``flash_gmm.py:78-158``)."""
        io = self.io_counter
        tiles = (self.K + self.BK - 1) // self.BK
        for p in (1, 2):
            io.record(f"X_pass{p}", X, "read")
            for t in range(tiles):
                k0, k1 = t * self.BK, min((t + 1) * self.BK, self.K)
                for tens in (self.mu[k0:k1], self.var[k0:k1], self.log_pi[k0:k1]):
                    io.record(f"params_p{p}_{t}", tens, "read")

    def _fused_em_step(self, X: torch.Tensor) -> torch.Tensor:
        """One fused E+M step; updates the parameters and returns the log-normalizer[N]."""
        X = self._to_device(X)
        N = X.shape[0]
        points, ws = self._operands(X)
        self._record_io(X)
        stats, ln = _C.em_stats(X, self.mu, self.var, self.log_pi, points=points, workspace=ws)
        self.mu, self.var, self.log_pi = _C.em_update(stats, N, self.K, self.d, floors=False)
        io = self.io_counter
        io.record("mu_new", self.mu, "write")
        io.record("var_new", self.var, "write")
        io.record("log_pi_new", self.log_pi, "write")
        return ln.clone()

    def fit(self, X: torch.Tensor, verbose: bool = False):
        """EM until ``|ΔLL| < tol`` or ``max_iter`` (``flash_gmm.py:171-205``)."""
        X = self._to_device(X)
        self._init_params(X)
        prev_ll = -float("inf")
        history = []
        for it in range(self.max_iter):
            self.io_counter.reset()
            t0 = time.time()
            log_normalizer = self._fused_em_step(X)
            avg_ll = log_normalizer.mean().item()
            _lib.check_device_error()
            elapsed = time.time() - t0
            history.append({"iter": it, "log_likelihood": avg_ll, "time_ms": elapsed * 1000,
                            "io_bytes": self.io_counter.total()})
            if verbose and (it % 10 == 0 or it < 5):
                print(f"  iter {it:3d}: LL={avg_ll:.4f}  time={elapsed*1000:.1f}ms  "
                      f"IO={self.io_counter.total()/1e6:.1f}MB")
            if abs(avg_ll - prev_ll) < self.tol:
                if verbose:
                    print(f"  Converged at iter {it}")
                break
            prev_ll = avg_ll
        return history

    def predict_proba(self, X: torch.Tensor) -> torch.Tensor:
        """Responsibilities gamma[N, K] (materialised: the caller asked for them)."""
        gamma, _ = _C.flash_e_step(self._to_device(X), self.mu, self.var, self.log_pi, BK=self.BK)
        return gamma

    def predict(self, X: torch.Tensor) -> torch.Tensor:
        return self.predict_proba(X).argmax(dim=1)
