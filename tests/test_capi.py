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
