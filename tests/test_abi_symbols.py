"""The C-ABI library builds for sm_100a, loads, and exports every function include/*.h declares (no CUDA
calls are made here, so this runs without a GPU)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(REPO, "include", h) for h in sorted(os.listdir(os.path.join(REPO, "include"))) if h.endswith(".h")]


def declared():
    names = []
    for h in HEADERS:
        txt = open(h).read()
        names += re.findall(r"^LK_API\s+[\w\s\*]+?\b((?:lkfl|lk|fl)_\w+)\s*\(", txt, re.M)
    return names


def test_headers_declare_entry_points():
    names = declared()
    assert "fl_moe" in names and "fl_wide_moe" in names and "lk_moe_forward" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol(native):
    L = ctypes.CDLL(native.LIB_PATH)
    missing = [n for n in declared() if not hasattr(L, n)]
    assert not missing, missing


def test_binding_signatures_cover_headers(native):
    assert set(declared()) == set(native.SIGNATURES)


def test_build_targets_sm100a_only():
    from loki_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
