"""ctypes binding of the C ABI in ``include/flashgmm_b200.h``.

The shared library ``flashgmm_b200/libflashgmm_b200.so`` is built in-tree by
``flashgmm_b200/build.py`` (``make -C flashgmm_b200/csrc``).  There is no CPU
implementation behind this module: if the library is missing, every entry point
raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FLASHGMM_LIB") or os.path.join(HERE, "libflashgmm_b200.so")

FGMM_OK = 0
FGMM_ERR_INVALID = 1
FGMM_ERR_UNSUPPORTED = 2
FGMM_ERR_WORKSPACE = 3
FGMM_ERR_CUDA = 4
FAMILY_AUTO, FAMILY_SIMT, FAMILY_TC, FAMILY_LOWK = 0, 1, 2, 3
UPDATE_NO_FLOORS = 1

# (name, restype, argtypes) for every symbol the header declares.
_vp, _i64, _i32, _sz, _d = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_size_t, ctypes.c_double
SIGNATURES = {
    "fgmm_last_error": (ctypes.c_char_p, []),
    "fgmm_version": (ctypes.c_int, []),
    "fgmm_set_family": (ctypes.c_int, [ctypes.c_int]),
    "fgmm_family_for": (ctypes.c_int, [_i64, _i32, _i32]),
    "fgmm_stats_len": (_i64, [_i32, _i32]),
    "fgmm_points_bytes": (_sz, [_i64, _i32, _i32]),
    "fgmm_prepare_points": (ctypes.c_int, [_vp, _i64, _i32, _i32, _vp, _sz, _vp]),
    "fgmm_em_stats_workspace_bytes": (_sz, [_i64, _i32, _i32]),
    "fgmm_em_stats": (ctypes.c_int, [_vp, _vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _sz, _vp]),
    "fgmm_em_update": (ctypes.c_int, [_vp, _d, _i32, _i32, _vp, _vp, _vp, _vp]),
    "fgmm_em_stats_ex": (ctypes.c_int, [_vp, _vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _sz, _i32, _vp]),
    "fgmm_em_update_prepared": (ctypes.c_int, [_vp, _d, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "fgmm_em_update_ex": (ctypes.c_int, [_vp, _d, _i32, _i32, _i32, _vp, _vp, _vp, _vp]),
    "fgmm_em_step": (ctypes.c_int, [_vp, _vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp,
                                    _vp, _sz, _i32, _vp]),
    "fgmm_device_error": (ctypes.c_int, [ctypes.c_int]),
    "fgmm_em_stats_launches": (ctypes.c_int, [_i64, _i32, _i32]),
    "fgmm_em_stats_profiled": (ctypes.c_int, [_vp, _vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _sz, _vp,
                                              ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_char_p), _i32]),
    "fgmm_em_fused_workspace_bytes": (_sz, [_i64, _i32, _i32]),
    "fgmm_em_fused_static": (ctypes.c_int, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp]),
    "fgmm_em_fused": (ctypes.c_int, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "fgmm_e_step_workspace_bytes": (ctypes.c_size_t, [_i64, _i32, _i32]),
    "fgmm_e_step": (ctypes.c_int, [_vp, _i64, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _sz, _vp]),
    "fgmm_m_step_workspace_bytes": (ctypes.c_size_t, [_i64, _i32, _i32]),
    "fgmm_m_step": (ctypes.c_int, [_vp, _i64, _i32, _vp, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
}

_lib = None


class FlashGMMError(RuntimeError):
    """Raised when a C-ABI call returns a non-zero status (mirrors TORCH_CHECK's RuntimeError)."""

    def __init__(self, code, msg):
        super().__init__(f"flashgmm_b200 error {code}: {msg}")
        self.code = code


def load():
    """Load the in-tree CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"flashgmm_b200 CUDA library not built: {LIB_PATH} "
                          "(run `python -m flashgmm_b200.build`)")
    try:  # share torch's CUDA runtime when torch is present
        import torch  # noqa: F401
    except ImportError:
        pass
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc):
    if rc != FGMM_OK:
        msg = load().fgmm_last_error()
        raise FlashGMMError(rc, msg.decode() if msg else "")
    return rc


class DeviceWaitError(RuntimeError):
    """A tensor-core kernel gave up a bounded wait: the results of that launch (and of
    every launch since) are incomplete."""


def check_device_error():
    """Raise :class:`DeviceWaitError` if a tensor-core kernel recorded a wait timeout on
    the current device since the last check (the code is cleared).  Synchronises the
    device: call it where the host already waits for results."""
    code = load().fgmm_device_error(1)
    if code < 0:
        raise DeviceWaitError("fgmm_device_error: CUDA error while reading the device error word")
    if code:
        raise DeviceWaitError(f"a tensor-core kernel gave up a bounded wait (code {code}); "
                              "the results of this iteration are incomplete")
