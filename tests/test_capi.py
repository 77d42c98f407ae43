"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU needed)."""
import glob
import os
import re
import subprocess

import pytest

from flashgmm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(fgmm_\w+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    syms = declared_symbols()
    for must in ["fgmm_em_fused", "fgmm_em_stats", "fgmm_em_update", "fgmm_prepare_points"]:
        assert must in syms


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(fgmm_\w+)", out))
    for s in declared_symbols():
        assert s in exported, f"{s} declared but not exported"
        assert hasattr(lib, s)
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"


def test_size_queries_without_gpu():
    lib = _lib.load()
    assert lib.fgmm_stats_len(256, 128) == 256 * 257 + 1
    assert lib.fgmm_em_fused_workspace_bytes(65536, 128, 256) > 0
    assert lib.fgmm_em_fused_workspace_bytes(10, 300, 4) == 0      # d > 256 unsupported
    assert lib.fgmm_family_for(10, 300, 4) == -1
    assert lib.fgmm_family_for(0, 8, 4) == -1


def test_family_selection_without_gpu():
    """FGMM_FAMILY_AUTO: low-K for K <= 16, d <= 128 and K d <= 512; tcgen05 for other
    d <= 128; SIMT above.  A forced family the shape is outside of reports -1."""
    lib = _lib.load()
    assert lib.fgmm_family_for(4096, 32, 8) == _lib.FAMILY_LOWK
    assert lib.fgmm_family_for(1000, 32, 16) == _lib.FAMILY_LOWK    # K d = 512
    assert lib.fgmm_family_for(1000, 64, 16) == _lib.FAMILY_TC      # K d = 1024
    assert lib.fgmm_family_for(1000, 2, 17) == _lib.FAMILY_TC       # K > 16
    assert lib.fgmm_family_for(1000, 160, 2) == _lib.FAMILY_SIMT    # d > 128
    prev = lib.fgmm_set_family(_lib.FAMILY_LOWK)
    try:
        assert lib.fgmm_family_for(1000, 128, 16) == _lib.FAMILY_LOWK
        assert lib.fgmm_family_for(1000, 128, 17) == -1
        assert lib.fgmm_family_for(1000, 129, 2) == -1
        assert lib.fgmm_em_stats_launches(1000, 128, 16) == 2
        assert lib.fgmm_em_stats_workspace_bytes(1000, 128, 16) > 0
    finally:
        lib.fgmm_set_family(prev)


def test_invalid_arguments_report_errors():
    lib = _lib.load()
    rc = lib.fgmm_em_fused(None, 0, 8, None, None, None, 4, None, None, None, None, None, 0, None)
    assert rc == _lib.FGMM_ERR_INVALID
    assert b"N, K and d" in lib.fgmm_last_error()
    rc = lib.fgmm_em_stats(None, None, 10, 300, None, None, None, 4, None, None, None, 0, None)
    assert rc == _lib.FGMM_ERR_UNSUPPORTED
    rc = lib.fgmm_em_update(None, 10.0, 4, 8, None, None, None, None)
    assert rc == _lib.FGMM_ERR_INVALID
    with pytest.raises(_lib.FlashGMMError):
        _lib.check(_lib.FGMM_ERR_INVALID)
