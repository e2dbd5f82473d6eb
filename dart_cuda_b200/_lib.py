"""ctypes binding of ``lib/libmat_mul.so``.

The library is the product: there is no CPU or PyTorch fallback.  If the
shared library is missing this module raises instead of degrading.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_bool, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("DART_CUDA_B200_LIB", PKG / "lib" / "libmat_mul.so"))

DC_OK = 0
DC_ERR_INVALID = 1
DC_F32 = 0
DC_BF16 = 1
DC_AFT_CAUSAL = 0x1
DC_AFT_ACCUMULATE = 0x2
DC_AFT_WS_VALID = 0x4
DC_AFT_SIMT = 0x8
DC_AFT_COMPUTE_BF16 = 0x10
DC_AFT_SAVE_STATS = 0x20
DC_AFT_BWD_NO_DKDV = 0x40
DC_AFT_BWD_DKDV = 0x80
DC_AFT_DW_PACKED = 0x100


def DC_AFT_SPARE_SMS(n):
    return (n & 0xFF) << 16


DC_GEMM_TRANS_A = 0x1
DC_GEMM_TRANS_B = 0x2
DC_GEMM_BIAS = 0x4
DC_GEMM_GELU = 0x8
DC_GEMM_GELU_BWD = 0x10
DC_GEMM_ACCUMULATE = 0x20

_lib = None


class DcError(RuntimeError):
    pass


# name -> (restype, argtypes); the C declarations are in include/dart_cuda_b200.h
_VP, _FP, _IP = c_void_p, POINTER(c_float), POINTER(c_int32)
SIGNATURES = {
    # dc_ entry points
    "dc_last_error": (ctypes.c_char_p, []),
    "dc_version": (ctypes.c_char_p, []),
    "dc_device_status": (c_int, [_VP, POINTER(c_int)]),
    "dc_aft_dw_packed_size": (c_int, [c_int, c_int, POINTER(c_size_t)]),
    "dc_aft_prep_mode": (c_int, [c_int]),
    "dc_aft_dw_unpack": (c_int, [_VP, _VP, c_int, c_int, c_int, _VP]),
    "dc_profile_enable": (c_int, [c_int]),
    "dc_profile_read": (c_int, [ctypes.c_char_p, _FP, POINTER(c_int), c_int]),
    "dc_aft_trace": (c_int, [_VP, c_size_t, c_int]),
    "dc_aft_workspace_size": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, POINTER(c_size_t)]),
    "dc_aft_fwd": (c_int, [_VP, _VP, _VP, _VP, c_int, _VP, c_int, c_int, c_int, c_int, c_int, c_int,
                           _VP, c_size_t, _VP]),
    "dc_aft_bwd": (c_int, [_VP, _VP, _VP, _VP, c_int, _VP, _VP, _VP, _VP, _VP, c_int, c_int, c_int,
                           c_int, c_int, c_int, _VP, c_size_t, _VP]),
    "dc_layernorm_fwd": (c_int, [_VP, _VP, _VP, _VP, c_int, c_int, c_float, _VP]),
    "dc_layernorm_bwd": (c_int, [_VP, _VP, _VP, _VP, _VP, _VP, c_int, c_int, c_float, c_int, _VP]),
    "dc_bias_fwd": (c_int, [_VP, _VP, _VP, c_int, c_int, _VP]),
    "dc_bias_bwd": (c_int, [_VP, _VP, _VP, c_int, c_int, c_int, _VP]),
    "dc_ce_fwd": (c_int, [_VP, _VP, _VP, _VP, c_int, c_int, c_float, _VP]),
    "dc_ce_bwd": (c_int, [_VP, _VP, _VP, _VP, c_int, c_int, c_float, _VP]),
    "dc_adam_step": (c_int, [_VP, _VP, _VP, _VP, c_int64, c_int, c_float, c_float, c_float, c_float,
                             c_float, _VP]),
    "dc_gemm": (c_int, [_VP, c_int, _VP, c_int, _VP, c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                        _VP, _VP, c_int, _VP, c_int, _VP]),
    "dc_gemm_gate": (c_int, [_VP, c_int, _VP, c_int, _VP, c_int, c_int, c_int, c_int, c_int, c_int,
                             c_float, _VP, _VP, c_int, _VP, _VP]),
    "dc_aft_fwd_strided": (c_int, [_VP, _VP, _VP, _VP, c_int, _VP, c_int, c_int, c_int, c_int, c_int,
                                   c_int, c_int, c_int, _VP, c_size_t, _VP]),
    "dc_aft_bwd_strided": (c_int, [_VP, _VP, _VP, _VP, c_int, _VP, _VP, _VP, _VP, _VP, c_int, c_int,
                                   c_int, c_int, c_int, c_int, c_int, c_int, _VP, c_size_t, _VP]),
    "dc_embedding_fwd": (c_int, [_VP, _VP, _VP, _VP, c_int, c_int, c_int, c_int, _VP]),
    "dc_embedding_bwd": (c_int, [_VP, _VP, _VP, _VP, c_int, c_int, c_int, c_int, _VP]),
    "dc_gate_fwd": (c_int, [_VP, c_int, _VP, _VP, c_int, c_int, c_int, _VP]),
    "dc_gate_bwd": (c_int, [_VP, c_int, _VP, _VP, c_int, _VP, c_int, _VP, c_int, c_int, _VP]),
    "dc_greedy_embed": (c_int, [_VP, c_int, c_int, c_int, _VP, _VP, _VP, c_int, _VP, c_int, _VP, _VP]),
    "dc_aft_decode_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "dc_aft_decode": (c_int, [_VP, c_int, _VP, c_int, ctypes.c_longlong, _VP, c_int, c_int, c_int, _VP,
                              c_int, _VP, c_int, _VP, c_size_t, _VP]),
    "dc_kv_cache_fill": (c_int, [_VP, c_int, c_int, c_int, c_int, _VP, _VP]),
    "dc_copy2d": (c_int, [_VP, c_size_t, _VP, c_size_t, c_size_t, c_size_t, _VP]),
    # the reference's handle ABI
    "create_tensor": (_VP, [c_int32, c_int32, _FP]),
    "destroy_tensor": (None, [_VP]),
    "get_tensor_data": (None, [_VP, _FP]),
    "get_tensor_grad": (None, [_VP, _FP]),
    "tensor_to_host": (None, [_VP, _FP]),
    "set_tensor_data": (None, [_VP, _FP]),
    "zero_grad": (None, [_VP]),
    "tensor_step": (None, [_VP, c_float]),
    "backward": (None, [_VP]),
    "aft_forward": (_VP, [_VP, _VP, _VP, _VP, c_bool]),
    "aft_cross_forward": (_VP, [_VP, _VP, _VP, _VP]),
    "layernorm_forward": (_VP, [_VP, _VP, _VP, c_float]),
    "add_tensor_row_broadcast": (_VP, [_VP, _VP]),
    "cross_entropy_loss": (_VP, [_VP, _IP, c_int32, c_int32]),
    "adam_step": (None, [_VP, _VP, _VP, c_int32, c_float, c_float, c_float, c_float]),
    "add_tensors": (_VP, [_VP, _VP]),
    "mul_tensors": (_VP, [_VP, _VP]),
    "sum_tensor": (_VP, [_VP]),
    "mean_tensor": (_VP, [_VP]),
    "matmul_tensors": (_VP, [_VP, _VP]),
    "gelu_tensor": (_VP, [_VP]),
    "embedding_forward": (_VP, [_IP, _VP, _VP, c_int32, c_int32]),
}


def lib():
    """Load and bind the library (once)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise DcError(
                f"{LIB_PATH} is missing; build it with `python -m dart_cuda_b200.build` "
                "(there is no fallback path)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str = "") -> None:
    if status != DC_OK:
        msg = lib().dc_last_error().decode(errors="replace")
        raise DcError(f"{what} failed with status {status}: {msg}")
