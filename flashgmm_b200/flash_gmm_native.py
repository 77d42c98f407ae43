"""Drop-in for the reference's compiled op module ``flash_gmm_native``.

The reference exposes its ops through pybind (``flash_gmm/csrc/binding.cpp:94-108``)
and its Python models import them as ``import flash_gmm_native as _C``
(``flash_gmm/native_wrapper.py:17-18``).  This module keeps those names, argument
names, defaults and return shapes, and routes every call through the C ABI of
``libflashgmm_b200.so`` on the tensors' CUDA device and the current torch stream.

Differences from the reference, all deliberate:

* CUDA tensors only.  The reference dispatches CPU tensors to its OpenMP path
  (``binding.cpp:68-75``); this package has no CPU implementation and raises.
* Stricter checks: besides the reference's "X must be float32" / "X must be 2D"
  (``binding.cpp:38-39,66``), shapes, dtypes, devices and contiguity of every
  argument are checked and reported as ``RuntimeError``.
* ``BN`` / ``BK`` are accepted and ignored: the reference's CUDA launcher also
  ignores ``BK`` (``flash_gmm/csrc/flash_gmm_cuda.cu:430-447``); here the tile
  shapes are fixed by the kernels.
"""
import torch

from . import _lib

__all__ = ["flash_em_fused", "standard_e_step", "flash_e_step", "standard_m_step", "em_stats", "em_step",
           "StatsWorkspace",
           "em_update", "em_update_prepared", "prepare_points", "stats_len", "family_for", "set_family"]


def _stream_ptr(device):
    return torch.cuda.current_stream(device).cuda_stream


def _check_f32_cuda(name, t, dim, device=None):
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a torch.Tensor")
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32")
    if t.dim() != dim:
        raise RuntimeError(f"{name} must be {dim}D")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (flashgmm_b200 has no CPU path)")
    if device is not None and t.device != device:
        raise RuntimeError(f"{name} is on {t.device}, expected {device}")


def _check_params(X, mu, var, log_pi):
    _check_f32_cuda("X", X, 2)
    dev = X.device
    _check_f32_cuda("mu", mu, 2, dev)
    _check_f32_cuda("var", var, 2, dev)
    _check_f32_cuda("log_pi", log_pi, 1, dev)
    N, d = X.shape
    K = mu.shape[0]
    if mu.shape != (K, d) or var.shape != (K, d) or log_pi.shape != (K,):
        raise RuntimeError(f"shape mismatch: X{tuple(X.shape)} mu{tuple(mu.shape)} "
                           f"var{tuple(var.shape)} log_pi{tuple(log_pi.shape)}")
    return X.contiguous(), mu.contiguous(), var.contiguous(), log_pi.contiguous(), N, d, K


def stats_len(K, d):
    return int(_lib.load().fgmm_stats_len(K, d))


def family_for(N, d, K):
    return int(_lib.load().fgmm_family_for(N, d, K))


def set_family(family):
    """Select the kernel family (``_lib.FAMILY_AUTO/SIMT/TC``); returns the previous one."""
    return int(_lib.load().fgmm_set_family(int(family)))


def _workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def flash_em_fused(X, mu, var, log_pi, BN=64, BK=8):
    """One fused EM iteration; returns ``[new_mu, new_var, new_log_pi, log_normalizer]``.

    Same contract as the reference op (``flash_gmm/csrc/binding.cpp:62-76``).
    """
    X, mu, var, log_pi, N, d, K = _check_params(X, mu, var, log_pi)
    lib = _lib.load()
    dev = X.device
    with torch.cuda.device(dev):
        ws_bytes = lib.fgmm_em_fused_workspace_bytes(N, d, K)
        if ws_bytes == 0:
            raise RuntimeError(f"flash_em_fused: unsupported shape N={N} K={K} d={d}")
        ws = _workspace(ws_bytes, dev)
        new_mu = torch.empty(K, d, dtype=torch.float32, device=dev)
        new_var = torch.empty(K, d, dtype=torch.float32, device=dev)
        new_lp = torch.empty(K, dtype=torch.float32, device=dev)
        ln = torch.empty(N, dtype=torch.float32, device=dev)
        _lib.check(lib.fgmm_em_fused(X.data_ptr(), N, d, mu.data_ptr(), var.data_ptr(),
                                     log_pi.data_ptr(), K, new_mu.data_ptr(), new_var.data_ptr(),
                                     new_lp.data_ptr(), ln.data_ptr(), ws.data_ptr(), ws.numel(),
                                     _stream_ptr(dev)))
    return [new_mu, new_var, new_lp, ln]


def standard_e_step(X, mu, var, log_pi):
    """E-step with materialised responsibilities -> ``[gamma[N, K], log_normalizer[N]]``.

    Same contract as the reference op (``flash_gmm/csrc/binding.cpp:35-49``, CUDA kernels
    ``flash_gmm/csrc/flash_gmm_cuda.cu:328-400``).
    """
    X, mu, var, log_pi, N, d, K = _check_params(X, mu, var, log_pi)
    lib = _lib.load()
    dev = X.device
    with torch.cuda.device(dev):
        nb = lib.fgmm_e_step_workspace_bytes(N, d, K)
        if nb == 0:
            raise RuntimeError(f"standard_e_step: unsupported shape N={N} K={K} d={d}")
        ws = _workspace(nb, dev)
        gamma = torch.empty(N, K, dtype=torch.float32, device=dev)
        ln = torch.empty(N, dtype=torch.float32, device=dev)
        _lib.check(lib.fgmm_e_step(X.data_ptr(), N, d, mu.data_ptr(), var.data_ptr(),
                                   log_pi.data_ptr(), K, gamma.data_ptr(), ln.data_ptr(),
                                   ws.data_ptr(), ws.numel(), _stream_ptr(dev)))
    return [gamma, ln]


def flash_e_step(X, mu, var, log_pi, BK=4):
    """Same outputs as :func:`standard_e_step` (``flash_gmm/csrc/binding.cpp:51-60``).

    The reference runs this op on the CPU only and refuses CUDA tensors; here it runs on
    the GPU.  ``BK`` (the reference's component tile of its online log-sum-exp) is
    accepted and ignored: the result does not depend on it.
    """
    return standard_e_step(X, mu, var, log_pi)


def standard_m_step(X, gamma):
    """M-step from responsibilities -> ``[new_mu, new_var, new_log_pi]``.

    Same contract and formulas as the reference op (``flash_gmm/csrc/binding.cpp:78-92``):
    no floor on ``n_k``, variance clamped at 1e-6, ``log_pi = log(n_k / N)``; the sums are
    accumulated in fp64.
    """
    _check_f32_cuda("X", X, 2)
    dev = X.device
    _check_f32_cuda("gamma", gamma, 2, dev)
    X = X.contiguous()
    gamma = gamma.contiguous()
    N, d = X.shape
    if gamma.shape[0] != N:
        raise RuntimeError(f"shape mismatch: X{tuple(X.shape)} gamma{tuple(gamma.shape)}")
    K = gamma.shape[1]
    lib = _lib.load()
    with torch.cuda.device(dev):
        nb = lib.fgmm_m_step_workspace_bytes(N, d, K)
        if nb == 0:
            raise RuntimeError(f"standard_m_step: unsupported shape N={N} K={K} d={d}")
        ws = _workspace(nb, dev)
        out = [torch.empty(K, d, dtype=torch.float32, device=dev),
               torch.empty(K, d, dtype=torch.float32, device=dev),
               torch.empty(K, dtype=torch.float32, device=dev)]
        _lib.check(lib.fgmm_m_step(X.data_ptr(), N, d, gamma.data_ptr(), K, out[0].data_ptr(),
                                   out[1].data_ptr(), out[2].data_ptr(), ws.data_ptr(),
                                   ws.numel(), _stream_ptr(dev)))
    return out


def prepare_points(X, K):
    """Tensor-core operand rows for X (constant over a fit), or ``None`` if the shape
    runs on the SIMT family.  Pass the result to :func:`em_stats`."""
    _check_f32_cuda("X", X, 2)
    X = X.contiguous()
    N, d = X.shape
    lib = _lib.load()
    with torch.cuda.device(X.device):
        nb = lib.fgmm_points_bytes(N, d, K)
        if nb == 0:
            return None
        pts = _workspace(nb, X.device)
        _lib.check(lib.fgmm_prepare_points(X.data_ptr(), N, d, K, pts.data_ptr(), pts.numel(),
                                           _stream_ptr(X.device)))
    return pts


class StatsWorkspace:
    """Reusable scratch for :func:`em_stats` (avoids an allocation per iteration)."""

    def __init__(self, N, d, K, device):
        lib = _lib.load()
        self.key = (N, d, K, device)
        self.ws = _workspace(lib.fgmm_em_stats_workspace_bytes(N, d, K), device)
        self.stats = torch.empty(stats_len(K, d), dtype=torch.float64, device=device)
        self.ln = torch.empty(N, dtype=torch.float32, device=device)


def em_stats(X, mu, var, log_pi, points=None, workspace=None, prepared=False):
    """Pass 1 + Pass 2 over local points -> ``(stats fp64 [K(2d+1)+1], log_normalizer[N])``.

    ``stats`` packs ``[n_k | s_k | sq_k | sum log_normalizer]``; sum it across ranks
    before :func:`em_update` for a sharded fit.  ``prepared=True`` asserts that
    :func:`em_update_prepared` produced ``mu, var, log_pi`` with this ``workspace`` and
    ``points``, so their tensor-core operands are reused.
    """
    X, mu, var, log_pi, N, d, K = _check_params(X, mu, var, log_pi)
    lib = _lib.load()
    dev = X.device
    with torch.cuda.device(dev):
        if workspace is None or workspace.key != (N, d, K, dev):
            workspace = StatsWorkspace(N, d, K, dev)
        if points is None and lib.fgmm_points_bytes(N, d, K) > 0:
            points = prepare_points(X, K)
        _lib.check(lib.fgmm_em_stats_ex(X.data_ptr(), points.data_ptr() if points is not None else None,
                                        N, d, mu.data_ptr(), var.data_ptr(), log_pi.data_ptr(), K,
                                        workspace.stats.data_ptr(), workspace.ln.data_ptr(),
                                        workspace.ws.data_ptr(), workspace.ws.numel(),
                                        STEP_PREPARED if prepared else 0, _stream_ptr(dev)))
    return workspace.stats, workspace.ln


STEP_PREPARED = 1


def em_step(X, mu, var, log_pi, points=None, workspace=None, out=None, prepared=False):
    """One EM iteration over prepared points: :func:`em_stats` and :func:`em_update` in
    one call (the update runs inside the statistics reduction's launch).  Returns
    ``(new_mu, new_var, new_log_pi, stats, log_normalizer)``; ``out`` may be the input
    parameter tensors themselves (in-place update).  ``prepared=True`` asserts that
    ``mu, var, log_pi`` are exactly the outputs of the previous ``em_step`` with this
    ``workspace`` (and ``points``), so their tensor-core operands, which that call left
    in the workspace, are reused instead of rebuilt."""
    X, mu, var, log_pi, N, d, K = _check_params(X, mu, var, log_pi)
    lib = _lib.load()
    dev = X.device
    with torch.cuda.device(dev):
        if workspace is None or workspace.key != (N, d, K, dev):
            workspace = StatsWorkspace(N, d, K, dev)
        if points is None and lib.fgmm_points_bytes(N, d, K) > 0:
            points = prepare_points(X, K)
        if out is None:
            out = (torch.empty(K, d, dtype=torch.float32, device=dev),
                   torch.empty(K, d, dtype=torch.float32, device=dev),
                   torch.empty(K, dtype=torch.float32, device=dev))
        _lib.check(lib.fgmm_em_step(X.data_ptr(), points.data_ptr() if points is not None else None,
                                    N, d, mu.data_ptr(), var.data_ptr(), log_pi.data_ptr(), K,
                                    out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(),
                                    workspace.stats.data_ptr(), workspace.ln.data_ptr(),
                                    workspace.ws.data_ptr(), workspace.ws.numel(),
                                    STEP_PREPARED if prepared else 0, _stream_ptr(dev)))
    return out[0], out[1], out[2], workspace.stats, workspace.ln


def em_update_prepared(stats, n_total, points, workspace, out=None):
    """The update step of a sharded fit: :func:`em_update` (floored) in one launch that also
    writes the tensor-core operands of the new parameters into ``workspace``, so the next
    ``em_stats(..., prepared=True)`` skips preparing them.  Tensor-core family only."""
    N, d, K, dev = workspace.key
    lib = _lib.load()
    with torch.cuda.device(dev):
        if out is None:
            out = (torch.empty(K, d, dtype=torch.float32, device=dev),
                   torch.empty(K, d, dtype=torch.float32, device=dev),
                   torch.empty(K, dtype=torch.float32, device=dev))
        _lib.check(lib.fgmm_em_update_prepared(stats.data_ptr(), float(n_total), points.data_ptr(),
                                               N, d, K, out[0].data_ptr(), out[1].data_ptr(),
                                               out[2].data_ptr(), workspace.ws.data_ptr(),
                                               workspace.ws.numel(), _stream_ptr(dev)))
    return out


def em_update(stats, n_total, K, d, out=None, floors=True):
    """M-step from (summed) stats -> ``(new_mu, new_var, new_log_pi)``.

    ``floors=True`` is the fused op's update (n_k and the weight floored at 1e-8,
    ``flash_gmm/csrc/flash_gmm_cpu.cpp:270-284``); ``floors=False`` the pure-Python
    model's (``flash_gmm/flash_gmm.py:162-169``): no floor, only the variance clamped."""
    if stats.dtype != torch.float64 or not stats.is_cuda or stats.numel() != stats_len(K, d):
        raise RuntimeError("stats must be a CUDA float64 tensor of length K(2d+1)+1")
    dev = stats.device
    lib = _lib.load()
    with torch.cuda.device(dev):
        if out is None:
            out = (torch.empty(K, d, dtype=torch.float32, device=dev),
                   torch.empty(K, d, dtype=torch.float32, device=dev),
                   torch.empty(K, dtype=torch.float32, device=dev))
        _lib.check(lib.fgmm_em_update_ex(stats.data_ptr(), float(n_total), K, d,
                                         0 if floors else _lib.UPDATE_NO_FLOORS, out[0].data_ptr(),
                                         out[1].data_ptr(), out[2].data_ptr(), _stream_ptr(dev)))
    return out
