"""The C-ABI library loads on a CPU-only host and exports every function
include/beatlm_b200.h declares (no compute calls: there is no GPU here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = []
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            text = open(os.path.join(ROOT, "include", h)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(bl_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared()
    assert "bl_attention" in names and "bl_status" in names and "bl_last_error" in names


def test_library_exports_every_declared_symbol():
    from beatlm_b200 import build
    so = build.build()
    L = ctypes.CDLL(so)
    missing = [n for n in declared() if not hasattr(L, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    from beatlm_b200 import _native
    assert set(declared()) <= set(_native.SIGNATURES), set(declared()) - set(_native.SIGNATURES)


def test_version_and_argument_errors_need_no_gpu():
    from beatlm_b200 import _native as N
    assert N.lib().bl_version().startswith(b"beatlm-b200")
    a = N.AttentionArgs(batch=1, tokens=8, heads=1, head_dim=32, head_begin=0, head_end=1,
                        row_begin=0, row_end=8, scale=0.125, qk_dtype=N.BL_F16,
                        v_dtype=N.BL_F16, out_dtype=N.BL_F32)
    with pytest.raises(N.BackendError, match="head_dim"):
        N.check(N.lib().bl_attention(ctypes.byref(a), None))
    a.head_dim = 64
    a.row_end = 9
    with pytest.raises(N.BackendError, match="rows"):
        N.check(N.lib().bl_attention(ctypes.byref(a), None))
