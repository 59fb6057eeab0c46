"""The C ABI: the library loads without a GPU, exports every entry point the
public header declares, and rejects invalid arguments before launching."""
import ctypes as C
import os
import re

import pytest

from fastgs_core_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for f in os.listdir(os.path.join(ROOT, "include")):
        if f.endswith(".h"):
            src = open(os.path.join(ROOT, "include", f)).read()
            names |= set(re.findall(r"FGS_API\s+[\w\s\*]+?\b(fgs_\w+)\s*\(", src))
    return names


def test_library_loads_and_exports_header_symbols():
    L = _lib.lib()
    declared = _declared()
    assert declared, "no FGS_API declarations found"
    for name in sorted(declared):
        assert hasattr(L, name), name
    # the Python binding declares a signature for every entry point
    assert declared <= set(_lib.exported_symbols()), sorted(declared - set(_lib.exported_symbols()))
    assert L.fgs_version() == 0x000100


def test_invalid_arguments_rejected_without_launch():
    L = _lib.lib()
    assert L.fgs_preprocess_forward(None, *([None] * 22)) == _lib.FGS_ERR_INVALID
    assert b"params" in L.fgs_last_error()
    bad = _lib.PreprocessParams(10, 3, 16, 1.0, 1.0, 1.0, 1.0, 64, 64, 0, 0)
    assert L.fgs_preprocess_forward(C.byref(bad), *([None] * 22)) == _lib.FGS_ERR_INVALID
    rp = _lib.RasterParams(64, 64, 5, 0, 0, 0)  # wrong tile count
    assert L.fgs_rasterize_forward(C.byref(rp), *([None] * 18)) == _lib.FGS_ERR_INVALID
    assert L.fgs_sort_pairs(10, 0, None, None, None, None, None, 0, None) == _lib.FGS_ERR_INVALID
    assert L.fgs_sort_pairs(1 << 31, 45, None, None, None, None, None, 0, None) == _lib.FGS_ERR_CAPACITY
    with pytest.raises(ValueError):
        _lib.check(_lib.FGS_ERR_INVALID, "x")
    # sizes do not need a device
    assert L.fgs_sort_workspace_bytes(1000, 45) > 1000 * 12
    assert L.fgs_scan_scratch_bytes(1 << 20) >= 8
