"""Build the in-tree CUDA library (sm_100a) with ``make -C flashgmm_b200/csrc``."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(verbose=False, jobs=8):
    cmd = ["make", "-C", os.path.join(HERE, "csrc"), f"-j{jobs}"]
    out = None if verbose else subprocess.DEVNULL
    subprocess.check_call(cmd, stdout=out)
    return os.path.join(HERE, "libflashgmm_b200.so")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
