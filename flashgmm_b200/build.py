"""Build the in-tree CUDA library (sm_100a) with ``make -C flashgmm_b200/csrc`` and the
PyTorch op module ``flashgmm_b200/_fgmm_torch.so`` (pybind11 bindings over the library's
C ABI, ``csrc/fgmm_torch.cpp``)."""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
EXT_NAME = "_fgmm_torch"
EXT_PATH = os.path.join(HERE, EXT_NAME + ".so")


def build_torch_ext(verbose=False):
    """Compile csrc/fgmm_torch.cpp against torch and libflashgmm_b200.so (found next to
    the extension at run time through its rpath)."""
    if os.path.exists("/usr/bin/g++"):
        os.environ.setdefault("CXX", "/usr/bin/g++")
    from torch.utils.cpp_extension import CUDA_HOME, load
    bdir = os.path.join(HERE, "csrc", "_build", "torch_ext")
    os.makedirs(bdir, exist_ok=True)
    load(name=EXT_NAME, sources=[os.path.join(HERE, "csrc", "fgmm_torch.cpp")],
         extra_cflags=["-O2", "-std=c++17"],
         extra_include_paths=[os.path.join(CUDA_HOME or "/usr/local/cuda", "include")],
         extra_ldflags=[f"-L{HERE}", "-lflashgmm_b200", r"-Wl,-rpath,\$$ORIGIN:\$$ORIGIN/../../.."],
         build_directory=bdir, verbose=verbose, with_cuda=True, is_python_module=True)
    shutil.copyfile(os.path.join(bdir, EXT_NAME + ".so"), EXT_PATH)
    return EXT_PATH


def build(verbose=False, jobs=8):
    cmd = ["make", "-C", os.path.join(HERE, "csrc"), f"-j{jobs}"]
    out = None if verbose else subprocess.DEVNULL
    subprocess.check_call(cmd, stdout=out)
    build_torch_ext(verbose)
    return os.path.join(HERE, "libflashgmm_b200.so")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
