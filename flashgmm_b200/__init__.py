"""flashgmm_b200: B200-native (sm_100a) fused diagonal-covariance GMM EM iteration.

Public surface (mirrors the reference's ``flash_gmm_native`` op module and its
``NativeFlashGMM`` model class):

* :mod:`flashgmm_b200.flash_gmm_native` -- ``flash_em_fused`` plus the split
  ``em_stats`` / ``em_update`` used by sharded multi-GPU fits.
* :class:`flashgmm_b200.native_wrapper.NativeFlashGMM`.
"""
__version__ = "0.1.0"
