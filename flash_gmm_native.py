"""Top-level name of the drop-in op module.

The reference's Python models import their compiled ops as ``import flash_gmm_native as
_C`` (``flash_gmm/native_wrapper.py:17-18``).  With this repository on ``sys.path`` that
import resolves here.  The reference's four ops (``flash_em_fused``, ``standard_e_step``,
``flash_e_step``, ``standard_m_step``; ``flash_gmm/csrc/binding.cpp:94-108``) come from
the compiled PyTorch extension ``flashgmm_b200/_fgmm_torch.so`` (pybind11 over this
package's C ABI). The statistics / update building blocks of sharded and out-of-core fits
come from :mod:`flashgmm_b200.flash_gmm_native`.  The reference's wrapper therefore runs
unmodified on the CUDA kernels.
"""
from flashgmm_b200._ext import load as _load_ext
from flashgmm_b200.flash_gmm_native import (  # noqa: F401
    StatsWorkspace, em_stats, em_step, em_update, em_update_prepared, family_for,
    prepare_points, set_family, stats_len)

_C = _load_ext()
flash_em_fused = _C.flash_em_fused
standard_e_step = _C.standard_e_step
flash_e_step = _C.flash_e_step
standard_m_step = _C.standard_m_step

__all__ = ["flash_em_fused", "standard_e_step", "flash_e_step", "standard_m_step", "em_stats",
           "em_step", "em_update", "em_update_prepared", "prepare_points", "stats_len",
           "family_for", "set_family", "StatsWorkspace"]
