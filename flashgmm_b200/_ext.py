"""Loader of the compiled PyTorch op module ``flashgmm_b200/_fgmm_torch.so`` (pybind11
bindings over the C ABI, built by ``flashgmm_b200/build.py`` from ``csrc/fgmm_torch.cpp``).
Raises if it has not been built: there is no fallback."""
import importlib.util
import os

HERE = os.path.dirname(os.path.abspath(__file__))
EXT_PATH = os.path.join(HERE, "_fgmm_torch.so")
_mod = None


def load():
    global _mod
    if _mod is None:
        import torch  # noqa: F401  (libtorch first)
        from . import _lib
        _lib.load()  # the CUDA library the extension links against
        if not os.path.exists(EXT_PATH):
            raise ImportError(f"flashgmm_b200 PyTorch extension not built: {EXT_PATH} "
                              "(run `python -m flashgmm_b200.build`)")
        spec = importlib.util.spec_from_file_location("_fgmm_torch", EXT_PATH)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _mod = mod
    return _mod
