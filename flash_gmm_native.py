"""Top-level name of the drop-in op module.

The reference's Python models import their compiled ops as ``import flash_gmm_native
as _C`` (``flash_gmm/native_wrapper.py:17-18``).  With this repository on ``sys.path``
that import resolves here and gets this package's CUDA ops
(:mod:`flashgmm_b200.flash_gmm_native`), so the reference's wrapper runs unmodified.
"""
from flashgmm_b200.flash_gmm_native import *  # noqa: F401,F403
from flashgmm_b200.flash_gmm_native import __all__  # noqa: F401
