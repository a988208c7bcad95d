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


def test_gather_backward_index_sizes_and_argument_checks():
    """Occurrence-index sizing and the gather backward's argument validation (no CUDA call is made)."""
    L = _lib.lib()
    r256 = lambda v: (v + 255) // 256 * 256
    n_out, K, inf = 64000, 16, 64000
    assert L.clb_logic_index_bytes(n_out, K, inf) == (r256(4 * (inf + 1)) + 2 * r256(8 * 2 * n_out * K) + r256(4 * inf) +
                                                    r256(32 * 2 * n_out * K))  # + the per-step baked records
    assert L.clb_logic_index_bytes(1 << 20, 16, 10) > 0                  # 2^24 slots: at the limit
    assert L.clb_logic_index_bytes((1 << 20) + 1, 16, 10) == -1          # slot id field overflow
    assert L.clb_logic_index_bytes(10, 0, 10) == -1
    assert L.clb_logic_index_bytes(10, 4, 0) == -1
    st = L.clb_logic_index_build(None, 10, 4, 3, None, 8, None, 0, None)  # n_out not a multiple of group
    assert st == _lib.CLB_ERR_INVALID and b"group" in L.clb_last_error()
    st = L.clb_logic_index_build(None, 10, 4, 1, None, 8, None, 16, None)  # buffer too small
    assert st == _lib.CLB_ERR_WORKSPACE
    args = [0, None, 8, 8, 8, 10, 4, 1, 0, None, None, None, 8, None, 0, 0, 0, 1.0, None, 8, None, None, 0, None]
    a = list(args)
    a[0] = 9
    assert L.clb_logic_backward_gather(*a) == _lib.CLB_ERR_DTYPE
    a = list(args)
    a[8] = 2  # select mode has no gradient
    assert L.clb_logic_backward_gather(*a) == _lib.CLB_ERR_INVALID
    assert L.clb_logic_backward_gather(*args) == _lib.CLB_ERR_INVALID  # null pointers
    a = list(args)
    a[3] = 0  # no columns: nothing to do
    assert L.clb_logic_backward_gather(*a) == _lib.CLB_OK
    # fp32: 128 columns per chunk when everything is 16-byte aligned, 32 (scalar) otherwise
    assert L.clb_logic_backward_gather_chunks(0, 256, 1024, 1000, 512, 1024, None, 0, 1024, 1024) == 8
    assert L.clb_logic_backward_gather_chunks(0, 256, 1023, 1000, 512, 1023, None, 0, 1024, 1024) == 32


def test_forward_stage_sizes_and_checks():
    """The baked forward stage's size query and argument checks (no CUDA call is made)."""
    L = _lib.lib()
    n = L.clb_logic_forward_stage_bytes(_lib.CLB_F32, 64000, 16)
    assert n >= 64000 * 16 * (16 + 8) and n % 256 == 0
    assert L.clb_logic_forward_stage_bytes(_lib.CLB_F32, 0, 16) == 0
    assert L.clb_logic_forward_stage_bytes(9, 10, 4) == 0
    st = L.clb_logic_forward_staged(7, None, 0, 0, 0, None, 0, 1, 1, 0, None, None, None, 0, None, 0, None, 0, 0, 0,
                                    None, 0, None)
    assert st == _lib.CLB_ERR_DTYPE
