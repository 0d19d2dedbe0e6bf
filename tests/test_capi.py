"""CPU: the C-ABI library builds, loads and exports every symbol include/exl3_b200.h declares, and its
host-side validation rejects bad arguments before any device work."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "exl3_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"EXL3_API\s+[\w\s\*]+?\b(exl3_\w+)\s*\(", text)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for s in ("exl3_decode_wt", "exl3_gemv", "exl3_gemv_workspace", "exl3_rot", "exl3_norm_rot",
              "exl3_swiglu_rot", "exl3_strerror", "exl3_version"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    from omlx_exl3_b200 import _lib
    L = _lib.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib._build.LIB)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(exl3_\w+)", out))
    for s in declared_symbols():
        assert s in exported, s
        assert hasattr(L, s)
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"


def test_strerror_and_version():
    from omlx_exl3_b200 import _lib
    L = _lib.lib()
    assert L.exl3_strerror(0) == b"ok"
    assert b"bits" in L.exl3_strerror(-2)
    assert L.exl3_version() >> 16 == 1


def _desc(**kw):
    from omlx_exl3_b200._lib import GemvDesc
    d = GemvDesc()
    d.k, d.n_members = kw.get("k", 4096), kw.get("nm", 1)
    ns = kw.get("n", [4096])
    for i in range(3):
        d.n[i] = ns[i] if i < len(ns) else 0
    d.bits, d.codebook, d.rows = kw.get("bits", 4), kw.get("cb", 0), kw.get("rows", 1)
    d.out_dtype, d.grid = kw.get("out", 0), kw.get("grid", 148)
    return d


def test_gemv_workspace_sizes():
    from omlx_exl3_b200 import _lib
    L = _lib.lib()
    pb, cb = ctypes.c_size_t(), ctypes.c_size_t()
    assert L.exl3_gemv_workspace(ctypes.byref(_desc()), ctypes.byref(pb), ctypes.byref(cb)) == 0
    # 32 blocks x 256 k-slices over 148 CTAs: 56 units per CTA -> at most 2 segments each
    assert cb.value == 32 * 4              # one arrival counter per 128-column block
    assert pb.value == 148 * 2 * 8 * 128 * 4


@pytest.mark.parametrize("kw,status", [
    (dict(k=4095), -1), (dict(n=[4000]), -1), (dict(rows=9), -1), (dict(rows=0), -1), (dict(nm=4), -1),
    (dict(bits=9), -2), (dict(bits=0), -2), (dict(cb=3), -3), (dict(out=2), -4),
])
def test_gemv_rejects_bad_descriptors(kw, status):
    from omlx_exl3_b200 import _lib
    L = _lib.lib()
    pb, cb = ctypes.c_size_t(), ctypes.c_size_t()
    assert L.exl3_gemv_workspace(ctypes.byref(_desc(**kw)), ctypes.byref(pb), ctypes.byref(cb)) == status


def test_null_and_shape_checks_come_first():
    from omlx_exl3_b200 import _lib
    L = _lib.lib()
    assert L.exl3_decode_wt(None, 16, 16, 4, 0, 0, -1, None, None) == -6
    assert L.exl3_decode_wt(8, 15, 16, 4, 0, 0, -1, 8, None) == -1
    assert L.exl3_decode_wt(8, 16, 16, 9, 0, 0, -1, 8, None) == -2
    assert L.exl3_decode_wt(8, 16, 16, 4, 5, 0, -1, 8, None) == -3
    assert L.exl3_rot(8, 0, 1, 100, 8, 1, 8, None) == -1
    assert L.exl3_swiglu_rot(8, 0, 1, 100, 8, 8, None) == -1
    assert L.exl3_norm_rot(8, 8, 0, 1, 128, 1e-6, 8, 4, 8, 8, None) == -1


def test_python_check_raises():
    from omlx_exl3_b200 import _lib
    with pytest.raises(ValueError):
        _lib.check(-1, "x")
    with pytest.raises(RuntimeError):
        _lib.check(-7, "x")
