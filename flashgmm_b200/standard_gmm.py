"""Drop-in for the reference's ``flash_gmm/standard_gmm.py``: the materialising EM model
``StandardGMM`` (with its ``e_step`` / ``m_step`` methods), the simulated-IO counter
``IOCounter`` and the data generator ``generate_gmm_data``.

``StandardGMM`` keeps the reference's constructor, attributes, initialisation, history
entries and stopping rule (``standard_gmm.py:55-205``).  Its E-step and M-step run on
this package's CUDA ops (``standard_e_step`` / ``standard_m_step``), which materialise
the N x K log-likelihood and responsibilities exactly as the reference model describes
(L written, read back for the log-sum-exp, gamma written); the IO counter records the
same simulated traffic as the reference's, tensor by tensor.
"""
import time
from dataclasses import dataclass, field

import torch

from . import _lib
from . import flash_gmm_native as _C


@dataclass
class IOCounter:
    """Simulated HBM read/write bytes per EM iteration (``standard_gmm.py:15-45``)."""
    reads: int = 0
    writes: int = 0
    details: dict = field(default_factory=dict)

    def record(self, name: str, tensor: torch.Tensor, op: str):
        nbytes = tensor.numel() * tensor.element_size()
        if op == "read":
            self.reads += nbytes
        else:
            self.writes += nbytes
        key = f"{op}:{name}"
        self.details[key] = self.details.get(key, 0) + nbytes

    def total(self):
        return self.reads + self.writes

    def summary(self):
        head = (f"Total IO: {self.total() / 1e6:.2f} MB  (R: {self.reads / 1e6:.2f} MB, "
                f"W: {self.writes / 1e6:.2f} MB)")
        return "\n".join([head] + [f"  {k}: {v / 1e6:.2f} MB" for k, v in sorted(self.details.items())])

    def reset(self):
        self.reads = 0
        self.writes = 0
        self.details.clear()


def init_params_like_reference(X, K, d, seed):
    """The reference models' initialisation (``standard_gmm.py:72-79``,
    ``flash_gmm.py:37-43``): K random points drawn with a CPU generator seeded ``seed``,
    every variance the mean per-dimension variance of X, uniform weights.  X may be on
    the GPU: the permutation is drawn on the host so the same seed picks the same points
    as the reference does."""
    N = X.shape[0]
    gen = torch.Generator().manual_seed(seed)
    idx = torch.randperm(N, generator=gen)[:K].to(X.device)
    mu = X[idx].clone()
    var = torch.ones(K, d, device=X.device) * X.var(dim=0, keepdim=True).mean()
    log_pi = torch.full((K,), -float(torch.log(torch.tensor(float(K)))), device=X.device)
    return mu.contiguous(), var.contiguous(), log_pi


class StandardGMM:
    """Standard EM with materialised L and gamma on this package's CUDA kernels.

    ``StandardGMM(K, d, max_iter=100, tol=1e-4, seed=42)`` as in ``standard_gmm.py:48-70``;
    ``device`` (default ``cuda``) is where a CPU ``X`` passed to ``fit`` is moved.
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
        self.io_counter = IOCounter()

    def _to_device(self, X):
        if X.is_cuda:
            return X.contiguous()
        dev = torch.device(self.device) if self.device is not None else torch.device("cuda")
        return X.to(dev).contiguous()

    def _init_params(self, X: torch.Tensor):
        self.mu, self.var, self.log_pi = init_params_like_reference(X, self.K, self.d, self.seed)

    def e_step(self, X: torch.Tensor):
        """Responsibilities and per-point log-likelihood -> ``(gamma[N, K], log_ll[N])``
        (``standard_gmm.py:81-132``)."""
        X = self._to_device(X)
        io = self.io_counter
        for name, t in (("X", X), ("mu", self.mu), ("var", self.var), ("log_pi", self.log_pi)):
            io.record(name, t, "read")
        gamma, log_ll = _C.standard_e_step(X, self.mu, self.var, self.log_pi)
        io.record("L_matrix", gamma, "write")  # the kernel writes L into the gamma buffer,
        io.record("L_matrix", gamma, "read")   # reads it back and normalises it in place
        io.record("gamma", gamma, "write")
        return gamma, log_ll

    def m_step(self, X: torch.Tensor, gamma: torch.Tensor):
        """Update ``mu``, ``var``, ``log_pi`` from responsibilities (``standard_gmm.py:134-160``):
        mu = gamma^T X / n_k, var = clamp(gamma^T (X - mu)^2 / n_k, 1e-6), log_pi = log(n_k / N).
        The variance is evaluated as gamma^T X^2 / n_k - mu^2 from fp64 sums, which equals
        the reference's two-pass form up to rounding."""
        X = self._to_device(X)
        io = self.io_counter
        io.record("gamma", gamma, "read")
        io.record("X", X, "read")
        self.mu, self.var, self.log_pi = _C.standard_m_step(X, gamma)
        io.record("mu_new", self.mu, "write")
        io.record("var_new", self.var, "write")
        io.record("log_pi_new", self.log_pi, "write")

    def fit(self, X: torch.Tensor, verbose: bool = False):
        """EM until ``|ΔLL| < tol`` or ``max_iter`` (``standard_gmm.py:162-195``)."""
        X = self._to_device(X)
        self._init_params(X)
        prev_ll = -float("inf")
        history = []
        for it in range(self.max_iter):
            self.io_counter.reset()
            t0 = time.time()
            gamma, log_ll = self.e_step(X)
            avg_ll = log_ll.mean().item()
            _lib.check_device_error()
            self.m_step(X, gamma)
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
        self.io_counter.reset()
        gamma, _ = self.e_step(X)
        return gamma

    def predict(self, X: torch.Tensor) -> torch.Tensor:
        return self.predict_proba(X).argmax(dim=1)


def generate_gmm_data(N: int, K: int, d: int, seed: int = 0):
    """Synthetic data from a known diagonal GMM -> ``(X, labels, true_mu, true_var, true_pi)``,
    all CPU tensors, the same values as the reference's generator
    (``standard_gmm.py:207-237``) for the same arguments: means ~N(0, 5^2), variances
    ~U[0.5, 1.0], uniform weights; labels drawn by ``multinomial``, points generated
    component by component and then shuffled.  The draws are taken from one CPU
    generator in the same order as the reference takes them, which is what makes the
    outputs equal."""
    g = torch.Generator().manual_seed(seed)
    true_mu = torch.randn(K, d, generator=g) * 5.0
    true_var = torch.rand(K, d, generator=g) * 0.5 + 0.5
    true_pi = torch.ones(K) / K
    z = torch.multinomial(true_pi, N, replacement=True, generator=g)
    blocks, labels = [], []
    for k in range(K):
        count = int((z == k).sum())
        if count:
            blocks.append(true_mu[k] + torch.randn(count, d, generator=g) * true_var[k].sqrt())
            labels.append(torch.full((count,), k, dtype=torch.int64))
    X = torch.cat(blocks, dim=0)
    lab = torch.cat(labels)
    order = torch.randperm(N, generator=g)
    return X[order], lab[order], true_mu, true_var, true_pi
