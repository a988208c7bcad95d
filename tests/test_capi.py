"""The C-ABI library loads without a GPU and exports every entry point include/compactlogic_b200.h declares."""
import ctypes
import os
import re

from compactlogic_b200 import _lib

from conftest import ROOT


def _declared():
    with open(os.path.join(ROOT, "include", "compactlogic_b200.h")) as f:
        src = f.read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(clb_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    declared = _declared()
    assert len(declared) >= 29
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert sorted(_lib.symbols()) == _declared()


def test_errors_are_reported_not_fatal():
    L = _lib.lib()
    assert L.clb_abi_version() == 1
    # invalid arguments are rejected before any CUDA call (works without a GPU)
    st = L.clb_logic_forward(7, None, 0, 0, 0, None, 0, 1, 1, 0, None, None, None, 0, None, 0, None, 0, 0, 0, None)
    assert st == _lib.CLB_ERR_DTYPE
    assert b"dtype" in L.clb_last_error()
    st = L.clb_groupbitsum(None, 10, 1, 64, 0, 3, None, None)
    assert st == _lib.CLB_ERR_DIVISIBILITY
    st = L.clb_tensor_packbits(None, 1, 1, 12, None, None, None)
    assert st == _lib.CLB_ERR_INVALID
