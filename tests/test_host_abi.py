"""CPU-side checks of the C-ABI boundary: the library loads and exports every
entry point declared in include/usaf_b200.h, with the Python binding covering
the same set.  No compute calls (no GPU here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "include", "usaf_b200.h")


def declared():
    src = open(HDR).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(usaf_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    assert "usaf_dispatch" in names and "usaf_sparse_adam" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    from usaf_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    from usaf_b200 import _lib
    assert sorted(_lib.EXPORTED) == declared()


def test_version_string():
    from usaf_b200 import _lib
    assert b"sm_100a" in _lib.LIB.usaf_version()


def test_cpu_tensor_rejected():
    import torch
    from usaf_b200 import _lib
    with pytest.raises(TypeError):
        _lib.ptr(torch.zeros(3))
