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


def _prototypes():
    src = open(HDR).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(usaf_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", src):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def test_binding_arity_matches_header():
    """Every ctypes signature takes as many arguments as the C prototype."""
    from usaf_b200 import _lib
    protos = _prototypes()
    bad = {n: (protos[n], len(_lib._SIGS[n][1])) for n in protos
           if n in _lib._SIGS and protos[n] != len(_lib._SIGS[n][1])}
    assert not bad, bad


def _struct_fields(name):
    src = open(HDR).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    end = re.search(r"\}\s*" + name + r"\s*;", src).start()
    body = src[src.rindex("typedef struct {", 0, end) + len("typedef struct {"):end]
    n = 0
    for decl in body.split(";"):
        decl = decl.strip()
        if decl:
            n += decl.count(",") + 1     # "int32_t T, E, P_cap" declares three
    return n


def test_struct_layouts_match_header():
    from usaf_b200 import _lib
    assert len(_lib.QWeight._fields_) == _struct_fields("usaf_qweight")
    assert len(_lib.RoutePlan._fields_) == _struct_fields("usaf_route_plan")
