"""The C-ABI library loads and exports every function include/navi_b200.h declares,
and the Python binding's prototype table covers exactly that set (CPU only: no
compute call is made without a GPU)."""
import ctypes
import os
import re

from navi_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if not h.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(navi_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_function():
    L = capi.lib()
    missing = [n for n in sorted(declared_functions()) if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert {n for n, _, _ in capi.SIGNATURES} == declared_functions()


def test_version_and_error_without_gpu():
    L = capi.lib()
    assert b"sm_100a" in L.navi_version()
    n = ctypes.c_int(-1)
    st = L.navi_device_count(ctypes.byref(n))
    assert st in (capi.NAVI_OK, capi.NAVI_E_CUDA)
