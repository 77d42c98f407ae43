"""Build the reference's own CPU EM path (test infrastructure, never shipped).

Compiles ``flash_gmm/csrc/binding.cpp`` and ``flash_gmm/csrc/flash_gmm_cpu.cpp``
straight from the read-only reference tree into ``oracle/_ref/`` as a Python
extension named ``flash_gmm_ref`` (the reference calls it ``flash_gmm_native``;
the name is changed only so it cannot shadow the drop-in module).  The flags
follow the reference's ``flash_gmm/setup.py:28-29`` (``-O3 -std=c++17
-fopenmp``).  ``WITH_CUDA`` is left undefined so only the CPU dispatch in
``binding.cpp:62-76`` is compiled.

The built ``.so`` is the ``kind: "reference"`` CPU baseline and the checker the
C restatement in ``flashgmm_oracle.c`` is pinned against.  It is only imported by
``tests/``, ``bench.py --impl reference`` / its ``cpu_baseline`` leg, and the
golden-vector generator.

Usage:  python oracle/build_ref.py [REFERENCE_ROOT]
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "flash_gmm_ref"


def default_reference_root():
    """The reference checkout: ``$FLASHGMM_REFERENCE``, else a ``reference`` directory
    beside this repository, else None."""
    env = os.environ.get("FLASHGMM_REFERENCE")
    if env:
        return env
    sib = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return sib if os.path.isdir(os.path.join(sib, "flash_gmm", "csrc")) else None


def build(ref_root=None, verbose=False):
    ref_root = ref_root or default_reference_root()
    if not ref_root:
        raise FileNotFoundError("no reference checkout: set FLASHGMM_REFERENCE")
    csrc = os.path.join(ref_root, "flash_gmm", "csrc")
    srcs = [os.path.join(csrc, "binding.cpp"), os.path.join(csrc, "flash_gmm_cpu.cpp")]
    for s in srcs:
        if not os.path.exists(s):
            raise FileNotFoundError(s)
    os.makedirs(OUT, exist_ok=True)
    # The /opt/gcc wrapper cannot find libgomp.spec; the system g++ links OpenMP fine.
    if os.path.exists("/usr/bin/g++"):
        os.environ["CXX"] = "/usr/bin/g++"
        os.environ["CC"] = "/usr/bin/gcc"
    from torch.utils.cpp_extension import load
    mod = load(name=NAME, sources=srcs,
               extra_cflags=["-O3", "-std=c++17", "-fopenmp"],
               extra_ldflags=["-fopenmp"],
               build_directory=OUT, verbose=verbose, with_cuda=False)
    return mod


def load_ref():
    """Import the prebuilt reference extension from ``oracle/_ref`` (no rebuild)."""
    import importlib.util
    import torch  # noqa: F401  (libtorch must be loaded first)
    path = os.path.join(OUT, NAME + ".so")
    if not os.path.exists(path):
        raise ImportError(f"reference CPU extension not built: {path}")
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    m = build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True)
    print("built", m.__file__)
