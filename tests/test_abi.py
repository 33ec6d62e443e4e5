"""The C ABI: libb200k.so loads on a machine without a GPU and exports every
entry point that include/b200k.h declares, with the ctypes table matching
the header (no compute is launched here)."""
import os
import re

import b200k
from b200k import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "b200k.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(b2k_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "b2k_norm" in names and "b2k_cross_entropy" in names
    assert len(names) >= 15


def test_every_declared_symbol_is_exported():
    exported = _lib.exported_symbols()
    for name in declared_functions():
        assert name in exported, f"{name} missing from the ctypes table"
        assert exported[name], f"{name} not exported by libb200k.so"


def test_ctypes_table_matches_header_arity():
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    for name, (_res, args) in _lib.SIGNATURES.items():
        m = re.search(r"\b" + name + r"\s*\(([^)]*)\)", src)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), f"{name}: header {len(params)} args, ctypes {len(args)}"


def test_library_basics_without_gpu():
    assert _lib.lib.b2k_version() >= 100
    assert isinstance(_lib.last_error(), str)
    assert os.path.exists(_lib.LIB_PATH)


def test_invalid_arguments_are_rejected_before_any_launch():
    # bad epilogue id: status EINVAL and a message, no CUDA call needed
    st = _lib.lib.b2k_norm(None, 0, None, 0, None, None, None, 0, None, 0, 4, 4, _lib.BF16,
                           _lib.NORM_LN, _lib.AFF_WB, 99, 1e-5, None)
    assert st == _lib.EINVAL and "act" in _lib.last_error()
    st = _lib.lib.b2k_norm(None, 0, None, 0, None, None, None, 0, None, 0, 4, 4, _lib.BF16,
                           _lib.NORM_L2, _lib.AFF_WB, 0, 1e-5, None)
    assert st != _lib.OK
    st = _lib.lib.b2k_rope(None, 0, None, 0, None, 0, None, 0, 4, 7, _lib.F16, 0, None)
    assert st == _lib.EINVAL and "even" in _lib.last_error()
    # empty inputs are a no-op
    assert _lib.lib.b2k_softmax(None, 0, None, 0, 0, 16, _lib.F32, 0, None, 0, None) == _lib.OK
