"""ctypes binding of the in-tree C-ABI library (include/compactlogic_b200.h).

The library is required: importing a layer that needs it without the built ``.so`` raises, and every
call checks the returned status and raises (``ValueError`` for the reference's ValueError cases,
``RuntimeError`` otherwise).  There is no CPU fallback.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libcompactlogic_b200.so")

CLB_OK, CLB_ERR_INVALID, CLB_ERR_DTYPE, CLB_ERR_INDEX, CLB_ERR_CUDA, CLB_ERR_WORKSPACE, CLB_ERR_DIVISIBILITY = range(7)
CLB_F32, CLB_F64, CLB_BF16, CLB_F16 = 0, 1, 2, 3
W_LOGITS, W_PROBS, W_SELECT = 0, 1, 2

_DTYPES = {torch.float32: CLB_F32, torch.float64: CLB_F64, torch.bfloat16: CLB_BF16, torch.float16: CLB_F16}

_i64, _int, _p, _sz, _dbl = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_double

# name -> (restype, argtypes)
_SIGS = {
    "clb_last_error": (ctypes.c_char_p, []),
    "clb_abi_version": (_int, []),
    "clb_launch_count": (ctypes.c_longlong, []),
    "clb_difflogic_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _int]),
    "clb_difflogic_forward": (_int, [_int, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _p, _p, _sz, _p]),
    "clb_difflogic_backward_w": (_int, [_int, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _p, _p, _sz, _p]),
    "clb_difflogic_backward_w_noalloc": (_int, [_int, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _p, _p]),
    "clb_difflogic_backward_x": (_int, [_int, _p, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _p, _p,
                                        _sz, _p]),
    "clb_difflogic_backward_x_atomic": (_int, [_int, _p, _i64, _i64, _p, _p, _p, _p, _p, _i64, _i64, _p, _p, _sz,
                                               _p]),
    "clb_difflogic_eval": (_int, [_int, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _p, _p, _sz, _p]),
    "clb_tensor_packbits": (_int, [_p, _i64, _i64, _int, _p, ctypes.POINTER(ctypes.c_int64), _p]),
    "clb_groupbitsum": (_int, [_p, _i64, _i64, _int, _i64, _i64, _p, _p]),
    "clb_convlogic_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int]),
    "clb_convlogic_forward": (_int, [_int, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, _i64, _int, _int,
                                     _int, _p, _p, _sz, _p]),
    "clb_convlogic_backward_x": (_int, [_int, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                        _i64, _int, _int, _p, _p, _sz, _p]),
    "clb_convlogic_backward_w": (_int, [_int, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                        _int, _p, _p, _sz, _p]),
    "clb_convlogic_eval": (_int, [_int, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, _i64, _int, _int, _int,
                                  _p, _p, _sz, _p]),
    "clb_slots_dense": (_int, [_p, _p, _i64, _i64, _i64, _p, _p, _p]),
    "clb_slots_conv": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p, _p, _p]),
    "clb_logic_forward": (_int, [_int, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _int, _p, _p, _p, _int, _p, _i64, _p,
                                 _i64, _i64, _i64, _p]),
    "clb_logic_forward_stage_bytes": (_sz, [_int, _i64, _i64]),
    "clb_logic_forward_staged": (_int, [_int, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _int, _p, _p, _p, _int, _p,
                                        _i64, _p, _i64, _i64, _i64, _p, _sz, _p]),
    "clb_logic_backward_chunks": (_i64, [_int, _p, _i64, _i64, _i64, _p, _i64, _p, _i64, _p, _i64]),
    "clb_logic_backward": (_int, [_int, _p, _i64, _i64, _p, _i64, _i64, _i64, _int, _p, _p, _int, _p, _i64, _p, _i64,
                                  _i64, _i64, _dbl, _p, _i64, _int, _i64, _p, _i64, _p]),
    "clb_logic_grad_finalize": (_int, [_int, _p, _i64, _i64, _i64, _i64, _int, _p, _p, _p]),
    "clb_conv_plane_parts": (_i64, [_i64, _i64, _int, _int, _i64]),
    "clb_conv_plane_forward": (_int, [_int, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _int,
                                      _i64, _p, _p, _p, _p, _i64, _int, _p, _p, _p, _p, _i64, _p, _p]),
    "clb_conv_plane_backward": (_int, [_int, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _int,
                                       _i64, _p, _p, _p, _p, _i64, _int, _p, _p, _p, _i64, _p, _i64, _int, _p, _i64,
                                       _p, _p]),
    "clb_l2_probe": (_int, [_int, _p, _p, _i64, _int, _int, _p, _p]),
    "clb_logic_index_bytes": (_i64, [_i64, _i64, _i64]),
    "clb_logic_index_build": (_int, [_p, _i64, _i64, _i64, _p, _i64, _p, _i64, _p]),
    "clb_logic_backward_gather_chunks": (_i64, [_int, _p, _i64, _i64, _p, _i64, _p, _i64, _p, _i64]),
    "clb_logic_backward_gather": (_int, [_int, _p, _i64, _i64, _i64, _i64, _i64, _i64, _int, _p, _p, _p, _i64, _p,
                                         _i64, _i64, _i64, _dbl, _p, _i64, _p, _p, _i64, _p]),
    "clb_logic_forward_peers": (_int, [_int, _p, _i64, _i64, _i64, _p, _i64, _i64, _int, _p, _p, _int, _p, _int, _i64,
                                       _p]),
    "clb_logic_backward_peers": (_int, [_int, _p, _i64, _i64, _p, _i64, _i64, _int, _p, _p, _int, _p, _int, _i64, _p,
                                        _i64, _int, _i64, _p, _i64, _p]),
    "clb_peer_alloc": (_int, [_sz, ctypes.POINTER(_p)]),
    "clb_peer_free": (_int, [_p]),
    "clb_ipc_export": (_int, [_p, _p]),
    "clb_ipc_import": (_int, [_p, ctypes.POINTER(_p)]),
    "clb_ipc_close": (_int, [_p]),
    "clb_transpose": (_int, [_int, _p, _i64, _i64, _i64, _p, _i64, _p]),
    "clb_cast": (_int, [_int, _p, _int, _p, _i64, _p]),
    "clb_pack_inputs": (_int, [_int, _p, _i64, _i64, _i64, _p, _i64, _p]),
    "clb_entropy_monitor": (_int, [_p, _i64, _i64, ctypes.c_float, ctypes.c_float, _int, _int, _p, _p, _p, _p, _p]),
    "clb_resample_rows": (_int, [_p, _p, _p, _p, _i64, _i64, _p, ctypes.c_float, ctypes.c_float, _int, _int, _p, _p,
                                 _p, _p, _p, _p, _p, _p, _p]),
    "clb_pack_thresholds": (_int, [_int, _p, _i64, _i64, _i64, _int, _p, _i64, _p]),
    "clb_packed_select": (_int, [_p, _p, _p, _i64, _i64, _i64, _p, _p, _p]),
    "clb_packed_layer": (_int, [_p, _i64, _i64, _p, _p, _i64, _p, _i64, _p]),
    "clb_packed_count_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "clb_packed_layer_count": (_int, [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _i64, _p, _sz, _p]),
    "clb_packed_count": (_int, [_p, _i64, _i64, _i64, _i64, _p, _i64, _i64, _p]),
}

_lib = None


def lib():
    """The loaded C-ABI library (raises ImportError when it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"compactlogic_b200: native library {LIB_PATH} is missing; build it with "
                "`python -m compactlogic_b200.build` (needs nvcc). There is no CPU fallback.")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def symbols():
    """Names of every entry point this binding declares."""
    return list(_SIGS)


def check(status: int, what: str = "") -> None:
    if status == CLB_OK:
        return
    msg = lib().clb_last_error().decode(errors="replace")
    if status == CLB_ERR_DIVISIBILITY:
        raise ValueError(msg)
    raise RuntimeError(f"compactlogic_b200 {what} failed (status {status}): {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def launches() -> int:
    """Kernels launched by the library so far (host-side counter)."""
    return int(lib().clb_launch_count())


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise RuntimeError(f"compactlogic_b200: unsupported dtype {dt} (float32, float64, bfloat16, float16)") from None


def acc_dtype(dt: torch.dtype) -> torch.dtype:
    """Arithmetic dtype of gradients / logits for activations of dtype dt."""
    return torch.float64 if dt == torch.float64 else torch.float32


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("compactlogic_b200 kernels need CUDA tensors (there is no CPU fallback)")
