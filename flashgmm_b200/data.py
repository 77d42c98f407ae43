"""Seeded synthetic workloads for the fused diagonal-covariance EM iteration.

The reference measures on synthetic mixtures only (``flash_gmm/standard_gmm.py:207-237``
``generate_gmm_data``; ``flash_gmm/benchmark_gpu.py:91`` uses ``torch.randn``).  The
five workloads below follow the configuration list this build is measured on:

* ``c1``  N=4,096   K=8     d=32   means ~N(0,5^2 I), var ~U[0.5,2], uniform weights
* ``c2``  N=65,536  K=256   d=128  means ~N(0,5^2 I), var ~U[0.5,2], Dirichlet(1) weights
* ``c3``  N=262,144 K=128   d=64   means ~N(0,3^2 I), var ~U[0.5,2], Dirichlet(1) weights
* ``c4``  N=65,536  K=1,024 d=64   means ~N(0,5^2 I), var ~U[0.5,2], uniform weights
* ``c5``  N=2^24    K=1,024 d=128  unit directions u_k, x = normalize(u_z + 0.05 eps)

Initial parameters (identical for every implementation under test): ``mu`` = K
distinct data points, ``var`` = 1, ``log_pi`` = -log K.  The reference's own
``_init_params`` (``flash_gmm/native_wrapper.py:115-121``) draws its random
permutation on the data's device, so CPU and CUDA runs would start from different
points; every comparison here therefore passes explicit initial parameters.

All draws use a CPU ``torch.Generator`` so the same seed gives the same bytes on
any machine with this torch build.
"""
from dataclasses import dataclass
import math

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    N: int
    K: int
    d: int
    iters: int
    mean_scale: float = 5.0
    weights: str = "uniform"        # "uniform" | "dirichlet"
    kind: str = "mixture"           # "mixture" | "directions"


WORKLOADS = {
    "c1": Workload("c1", 4096, 8, 32, 20, 5.0, "uniform"),
    "c2": Workload("c2", 65536, 256, 128, 20, 5.0, "dirichlet"),
    "c3": Workload("c3", 262144, 128, 64, 20, 3.0, "dirichlet"),
    "c4": Workload("c4", 65536, 1024, 64, 20, 5.0, "uniform"),
    "c5": Workload("c5", 1 << 24, 1024, 128, 10, 0.0, "uniform", "directions"),
}


CHUNK = 1 << 16


def _components(Kt, d, seed, mean_scale, weights, kind):
    g = torch.Generator().manual_seed(int(seed))
    if kind == "directions":
        u = torch.randn(Kt, d, generator=g, dtype=torch.float64)
        return u / u.norm(dim=1, keepdim=True), None, torch.full((Kt,), 1.0 / Kt, dtype=torch.float64)
    mu = torch.randn(Kt, d, generator=g, dtype=torch.float64) * mean_scale
    var = torch.rand(Kt, d, generator=g, dtype=torch.float64) * 1.5 + 0.5
    if weights == "dirichlet":
        e = -torch.log(torch.rand(Kt, generator=g, dtype=torch.float64))
        pi = e / e.sum()
    else:
        pi = torch.full((Kt,), 1.0 / Kt, dtype=torch.float64)
    return mu, var, pi


def _chunk(c, n, d, seed, mu, var, pi, kind):
    """Points [c*CHUNK, c*CHUNK + n) -- each chunk has its own generator, so any
    row range can be produced without generating the rows before it."""
    g = torch.Generator().manual_seed(int(seed) * 1000003 + 17 + c)
    z = torch.multinomial(pi, n, replacement=True, generator=g)
    if kind == "directions":
        v = mu[z].float() + 0.05 * torch.randn(n, d, generator=g)
        return v / v.norm(dim=1, keepdim=True), z
    eps = torch.randn(n, d, generator=g, dtype=torch.float64)
    return (mu[z] + var[z].sqrt() * eps).float(), z


def make_mixture(N, K, d, seed=0, mean_scale=5.0, weights="uniform", kind="mixture",
                 n_true=None, rows=None):
    """Sample ``X`` (fp32, CPU) from a diagonal Gaussian mixture (or, for
    ``kind="directions"``, noisy unit directions).

    ``rows=(start, stop)`` returns only that slice of the N-point data set (used by
    sharded multi-GPU runs); the values are identical to the same rows of the
    full set.  Returns ``(X, labels, true_mu, true_var, true_pi)``.
    """
    Kt = n_true or K
    mu, var, pi = _components(Kt, d, seed, mean_scale, weights, kind)
    r0, r1 = rows if rows is not None else (0, N)
    r0, r1 = max(0, r0), min(N, r1)
    X = torch.empty(max(0, r1 - r0), d, dtype=torch.float32)
    z = torch.empty(max(0, r1 - r0), dtype=torch.int64)
    c = r0 // CHUNK
    while c * CHUNK < r1:
        lo, hi = c * CHUNK, min(N, (c + 1) * CHUNK)
        xc, zc = _chunk(c, hi - lo, d, seed, mu, var, pi, kind)
        a, b = max(lo, r0), min(hi, r1)
        X[a - r0:b - r0] = xc[a - lo:b - lo]
        z[a - r0:b - r0] = zc[a - lo:b - lo]
        c += 1
    return X, z, mu.float(), None if var is None else var.float(), pi.float()


def init_params(X, K, seed=1):
    """Initial ``(mu, var, log_pi)``: K distinct random points, unit variance, uniform pi."""
    g = torch.Generator().manual_seed(int(seed))
    N, d = X.shape
    idx = torch.randperm(N, generator=g)[:K]
    mu = X[idx].clone().contiguous()
    var = torch.ones(K, d, dtype=torch.float32)
    log_pi = torch.full((K,), -math.log(K), dtype=torch.float32)
    return mu, var, log_pi


def make_workload(name_or_wl, seed=0, N=None, rows=None):
    """Data + initial parameters for a named workload.

    ``N`` shrinks the data set (a prefix-independent sample of the same mixture);
    ``rows`` returns only a slice of X.  The initial means are always drawn from the
    first min(N, 65536) points so every shard / rank starts from the same parameters.
    """
    wl = WORKLOADS[name_or_wl] if isinstance(name_or_wl, str) else name_or_wl
    n = N or wl.N
    kw = dict(seed=seed, mean_scale=wl.mean_scale, weights=wl.weights, kind=wl.kind)
    X, *_ = make_mixture(n, wl.K, wl.d, rows=rows, **kw)
    m = min(n, CHUNK)
    if rows is None or rows[0] == 0 and rows[1] >= m:
        X0 = X[:m]
    else:
        X0 = make_mixture(n, wl.K, wl.d, rows=(0, m), **kw)[0]
    mu, var, log_pi = init_params(X0, wl.K, seed=seed + 1)
    return X, mu, var, log_pi
