"""PyTorch-facing calls of the batched C ABI (``dc_*`` entry points).

PyTorch supplies device memory and the current CUDA stream only; every
computation runs in ``libmat_mul.so``.  All tensors must be CUDA tensors.

AFT-full operator (reference: native/src/kernels/attention.cuh:6-40 forward,
native/src/engine.cu:522-590 backward), batched over B sequences that share
the pairwise bias ``w``:

    Z = aft_fwd(Q, K, V, w, causal=True)
    dQ, dK, dV, dW = aft_bwd(Q, K, V, w, dZ, causal=True)
"""
from __future__ import annotations

from ctypes import byref, c_int, c_size_t

import torch

from ._lib import (DC_AFT_ACCUMULATE, DC_AFT_BWD_DKDV, DC_AFT_BWD_NO_DKDV, DC_AFT_CAUSAL, DC_AFT_DW_PACKED,
                   DC_AFT_COMPUTE_BF16, DC_AFT_SAVE_STATS, DC_AFT_SIMT, DC_AFT_SPARE_SMS,
                   DC_AFT_WS_VALID, DC_BF16, DC_F32, DC_GEMM_ACCUMULATE, DC_GEMM_BIAS, DC_GEMM_GELU,
                   DC_GEMM_GELU_BWD, DC_GEMM_TRANS_A, DC_GEMM_TRANS_B, DcError, check, lib)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return DC_F32
    if t.dtype == torch.bfloat16:
        return DC_BF16
    raise DcError(f"unsupported dtype {t.dtype}")


def _ptr(t):
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, name: str, rows_strided=False):
    if not t.is_cuda:
        raise DcError(f"{name} must be a CUDA tensor")
    if rows_strided:
        if t.dim() != 2 or t.stride(1) != 1:
            raise DcError(f"{name} must be 2-D with unit column stride")
    elif not t.is_contiguous():
        raise DcError(f"{name} must be contiguous")


def _as3d(t: torch.Tensor) -> torch.Tensor:
    return t.unsqueeze(0) if t.dim() == 2 else t


class AftWorkspace:
    """Device scratch for one AFT shape: the operand panels (A', E'V, E'),
    the row/column maxima and the backward's g/n panels.  A workspace filled
    by ``aft_fwd`` can be handed to ``aft_bwd`` with ``ws_valid=True`` so the
    backward skips recomputing the panels.  With ``save_stats=True`` the
    forward also keeps r and 1/den there and such a backward skips the second
    pass of the forward contraction as well."""

    def __init__(self, B, Tq, Tk, D, dtype: torch.dtype, flags: int = 0, device=None,
                 save_stats=False):
        n = c_size_t(0)
        self.save_stats = bool(save_stats or flags & DC_AFT_SAVE_STATS)
        if self.save_stats:
            flags |= DC_AFT_SAVE_STATS
        code = DC_F32 if dtype == torch.float32 else DC_BF16
        check(lib().dc_aft_workspace_size(B, Tq, Tk, D, code, flags, byref(n)), "dc_aft_workspace_size")
        self.nbytes = int(n.value)
        self._buf = torch.empty(self.nbytes + 1024, dtype=torch.uint8, device=device or "cuda")
        base = self._buf.data_ptr()
        self.ptr = (base + 1023) // 1024 * 1024


def _flags(causal, accumulate=False, ws_valid=False, simt=False, compute_bf16=False):
    f = 0
    if causal:
        f |= DC_AFT_CAUSAL
    if accumulate:
        f |= DC_AFT_ACCUMULATE
    if ws_valid:
        f |= DC_AFT_WS_VALID
    if simt:
        f |= DC_AFT_SIMT
    if compute_bf16:
        f |= DC_AFT_COMPUTE_BF16
    return f


def aft_fwd(Q, K, V, w, causal=True, out=None, workspace: AftWorkspace | None = None,
            ws_valid=False, simt=False, compute_bf16=False):
    Q3, K3, V3 = _as3d(Q), _as3d(K), _as3d(V)
    for t, n in ((Q3, "Q"), (K3, "K"), (V3, "V")):
        _need(t, n)
    _need(w, "w", rows_strided=True)
    B, Tq, D = Q3.shape
    Tk = K3.shape[1]
    if w.dtype != torch.float32 or w.dim() != 2:
        raise DcError("w must be a 2-D float32 tensor")
    Z = torch.empty_like(Q) if out is None else out
    ws = workspace.ptr if workspace is not None else None
    nb = workspace.nbytes if workspace is not None else 0
    flags = _flags(causal, ws_valid=ws_valid, simt=simt, compute_bf16=compute_bf16)
    if workspace is not None and workspace.save_stats:
        flags |= DC_AFT_SAVE_STATS
    check(lib().dc_aft_fwd(Q3.data_ptr(), K3.data_ptr(), V3.data_ptr(), w.data_ptr(), w.stride(0),
                           Z.data_ptr(), B, Tq, Tk, D, _dtype_code(Q3), flags, ws, nb, _stream()),
          "dc_aft_fwd")
    return Z


def aft_dw_packed_size(Tq: int, Tk: int) -> int:
    """Floats of a block-packed causal dW (dw_packed=True in aft_bwd)."""
    n = c_size_t(0)
    check(lib().dc_aft_dw_packed_size(int(Tq), int(Tk), byref(n)), "dc_aft_dw_packed_size")
    return int(n.value)


def aft_dw_unpack(packed: torch.Tensor, dW: torch.Tensor) -> torch.Tensor:
    """Expand a block-packed causal dW into dW [Tq, Tk] (row stride dW.stride(0))."""
    if dW.dtype != torch.float32 or dW.dim() != 2 or dW.stride(1) != 1:
        raise DcError("dW must be a 2-D float32 tensor with unit column stride")
    Tq, Tk = dW.shape
    if packed.numel() < aft_dw_packed_size(Tq, Tk):
        raise DcError("packed dW is too small")
    check(lib().dc_aft_dw_unpack(packed.data_ptr(), dW.data_ptr(), dW.stride(0), Tq, Tk, _stream()),
          "dc_aft_dw_unpack")
    return dW


def aft_bwd(Q, K, V, w, dZ, causal=True, grads=None, accumulate=False,
            workspace: AftWorkspace | None = None, ws_valid=False, simt=False, compute_bf16=False,
            part=None, spare_sms=0, dw_packed=False):
    """dQ, dK, dV, dW of the AFT-full op.

    part=None computes all four.  part="dw" computes dQ and dW only and leaves
    g, n in `workspace`; part="dkdv" then computes dK and dV from them (same
    workspace, ws_valid=True), so a data-parallel caller can all-reduce dW
    while dK and dV run.  spare_sms leaves that many SMs free for such a
    collective.  Entries of `grads` a part does not write may be None.
    dw_packed=True (causal only): dW is a 1-D float32 buffer of
    aft_dw_packed_size(Tq, Tk) floats in the block-packed layout."""
    Q3, K3, V3, G3 = _as3d(Q), _as3d(K), _as3d(V), _as3d(dZ)
    for t, n in ((Q3, "Q"), (K3, "K"), (V3, "V"), (G3, "dZ")):
        _need(t, n)
    _need(w, "w", rows_strided=True)
    B, Tq, D = Q3.shape
    Tk = K3.shape[1]
    if part not in (None, "dw", "dkdv"):
        raise DcError(f"part must be None, 'dw' or 'dkdv' (got {part!r})")
    if grads is None:
        dW0 = (torch.empty(aft_dw_packed_size(Tq, Tk), device=w.device) if dw_packed else
               torch.empty(w.shape[0], w.stride(0), device=w.device)[:, : w.shape[1]])
        grads = (torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V), dW0)
    dQ, dK, dV, dW = grads
    if dw_packed:
        if dW is not None and (dW.dtype != torch.float32 or not dW.is_contiguous()
                               or dW.numel() < aft_dw_packed_size(Tq, Tk)):
            raise DcError("packed dW must be a contiguous float32 buffer of aft_dw_packed_size floats")
    elif dW is not None and (dW.dtype != torch.float32 or dW.stride(0) != w.stride(0) or dW.stride(1) != 1):
        raise DcError("dW must be float32 with the row stride of w")
    ws = workspace.ptr if workspace is not None else None
    nb = workspace.nbytes if workspace is not None else 0
    flags = _flags(causal, accumulate, ws_valid, simt, compute_bf16) | DC_AFT_SPARE_SMS(spare_sms)
    if workspace is not None and workspace.save_stats:
        flags |= DC_AFT_SAVE_STATS
    if dw_packed:
        flags |= DC_AFT_DW_PACKED
    if part == "dw":
        flags |= DC_AFT_BWD_NO_DKDV
    elif part == "dkdv":
        flags |= DC_AFT_BWD_DKDV
    check(lib().dc_aft_bwd(Q3.data_ptr(), K3.data_ptr(), V3.data_ptr(), w.data_ptr(), w.stride(0),
                           G3.data_ptr(), _ptr(dQ), _ptr(dK), _ptr(dV), _ptr(dW),
                           B, Tq, Tk, D, _dtype_code(Q3), flags, ws, nb, _stream()),
          "dc_aft_bwd")
    return dQ, dK, dV, dW


DC_STATUS_AFT_RANGE = 0x80  # an AFT-full input outside the factorised range


def device_status(sync_stream=True) -> int:
    """Synchronise and return the device status bits (0 = no kernel reported
    anything); raises DcError when bits are set."""
    bits = c_int(0)
    check(lib().dc_device_status(_stream(), byref(bits)), "dc_device_status")
    return bits.value


def read_status() -> int:
    """Synchronise, read and clear the device status bits without raising:
    0x1-0x10 a bounded wait gave up, 0x20 token id out of range, 0x40 decode
    past capacity, 0x80 (DC_STATUS_AFT_RANGE) an AFT-full input outside the
    range of the factorised stabilisation."""
    bits = c_int(0)
    rc = lib().dc_device_status(_stream(), byref(bits))
    if rc not in (0, 5):  # DC_OK, DC_ERR_DEVICE
        check(rc, "dc_device_status")
    return bits.value


# ---------------------------------------------------------------- row ops
def layernorm_fwd(x, gamma, beta, eps=1e-5, out=None):
    R, C = x.shape
    y = torch.empty_like(x) if out is None else out
    check(lib().dc_layernorm_fwd(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), y.data_ptr(), R, C,
                                 eps, _stream()), "dc_layernorm_fwd")
    return y


def layernorm_bwd(x, gamma, dy, eps=1e-5, grads=None, accumulate=False):
    R, C = x.shape
    if grads is None:
        grads = (torch.empty_like(x), torch.empty(C, device=x.device), torch.empty(C, device=x.device))
    dx, dg, db = grads
    check(lib().dc_layernorm_bwd(x.data_ptr(), gamma.data_ptr(), dy.data_ptr(), dx.data_ptr(),
                                 dg.data_ptr(), db.data_ptr(), R, C, eps, int(accumulate), _stream()),
          "dc_layernorm_bwd")
    return dx, dg, db


def bias_fwd(a, b, out=None):
    M, N = a.shape
    y = torch.empty_like(a) if out is None else out
    check(lib().dc_bias_fwd(a.data_ptr(), b.data_ptr(), y.data_ptr(), M, N, _stream()), "dc_bias_fwd")
    return y


def bias_bwd(dy, grads=None, accumulate=False):
    M, N = dy.shape
    if grads is None:
        grads = (torch.empty_like(dy), torch.empty(N, device=dy.device))
    da, db = grads
    check(lib().dc_bias_bwd(dy.data_ptr(), _ptr(da), db.data_ptr(), M, N, int(accumulate), _stream()),
          "dc_bias_bwd")
    return da, db


def ce_fwd(logits, targets, eps=0.1, row_loss=None, out=None):
    T, V = logits.shape
    loss = torch.empty(1, device=logits.device) if out is None else out
    check(lib().dc_ce_fwd(logits.data_ptr(), targets.data_ptr(), loss.data_ptr(), _ptr(row_loss), T, V,
                          eps, _stream()), "dc_ce_fwd")
    return loss


def ce_bwd(logits, targets, grad_scale=None, eps=0.1, out=None):
    T, V = logits.shape
    g = torch.empty_like(logits) if out is None else out
    check(lib().dc_ce_bwd(logits.data_ptr(), targets.data_ptr(), _ptr(grad_scale), g.data_ptr(), T, V,
                          eps, _stream()), "dc_ce_bwd")
    return g


def adam_step(p, g, m, v, t, lr, b1=0.9, b2=0.999, eps=1e-8, weight_decay=0.001):
    check(lib().dc_adam_step(p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(), int(t),
                             lr, b1, b2, eps, weight_decay, _stream()), "dc_adam_step")


# ---------------------------------------------------------------- dense layers
def _ld(t: torch.Tensor, name: str) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise DcError(f"{name} must be 2-D with unit column stride")
    return t.stride(0)


def gemm(A, B, out=None, trans_a=False, trans_b=False, bias=None, residual=None, accumulate=False,
         gelu=False, gelu_aux=None, gelu_bwd_aux=None, alpha=1.0, gate=None):
    """C = epilogue(alpha * op(A) @ op(B)) through ``dc_gemm``: A and B fp32
    (tf32 tensor-core operands) or bf16, C fp32.  ``residual`` (or C itself
    with ``accumulate``) is added after the bias; ``gelu`` applies the tanh
    GELU and stores the pre-activation in ``gelu_aux`` when given;
    ``gelu_bwd_aux`` multiplies by the GELU derivative at that
    pre-activation.  ``gate`` ([N]) ends the epilogue with
    sigmoid(value) * gate (``dc_gemm_gate``)."""
    if A.dtype != B.dtype:
        raise DcError("A and B must share a dtype")
    M = A.shape[1] if trans_a else A.shape[0]
    K = A.shape[0] if trans_a else A.shape[1]
    N = B.shape[0] if trans_b else B.shape[1]
    if (B.shape[1] if trans_b else B.shape[0]) != K:
        raise DcError(f"inner dimensions differ: op(A) [{M},{K}], B {tuple(B.shape)}")
    C = torch.empty(M, N, device=A.device) if out is None else out
    flags = ((DC_GEMM_TRANS_A if trans_a else 0) | (DC_GEMM_TRANS_B if trans_b else 0) |
             (DC_GEMM_BIAS if bias is not None else 0) | (DC_GEMM_ACCUMULATE if accumulate else 0))
    aux, ldx = None, 0
    if gelu:
        flags |= DC_GEMM_GELU
        if gelu_aux is not None:
            aux, ldx = gelu_aux.data_ptr(), _ld(gelu_aux, "gelu_aux")
    if gelu_bwd_aux is not None:
        flags |= DC_GEMM_GELU_BWD
        aux, ldx = gelu_bwd_aux.data_ptr(), _ld(gelu_bwd_aux, "gelu_bwd_aux")
    R, ldr = (None, 0) if residual is None else (residual.data_ptr(), _ld(residual, "residual"))
    if gate is None:
        check(lib().dc_gemm(A.data_ptr(), _ld(A, "A"), B.data_ptr(), _ld(B, "B"), C.data_ptr(), _ld(C, "C"),
                            M, N, K, _dtype_code(A), flags, float(alpha), _ptr(bias), R, ldr, aux, ldx,
                            _stream()), "dc_gemm")
        return C
    if aux is not None:
        raise DcError("the gate excludes GELU and GELU_BWD")
    check(lib().dc_gemm_gate(A.data_ptr(), _ld(A, "A"), B.data_ptr(), _ld(B, "B"), C.data_ptr(), _ld(C, "C"),
                             M, N, K, _dtype_code(A), flags, float(alpha), _ptr(bias), R, ldr, gate.data_ptr(),
                             _stream()), "dc_gemm_gate")
    return C


# ---------------------------------------------------------------- timing
def profile_enable(on: bool = True) -> None:
    """Bracket every library kernel launch with CUDA events (drops old records)."""
    check(lib().dc_profile_enable(int(on)), "dc_profile_enable")


def profile_read(max_entries: int = 64) -> dict:
    """{kernel name: (total ms, launches)} of the launches recorded so far."""
    import ctypes

    names = ctypes.create_string_buffer(64 * max_entries)
    ms = (ctypes.c_float * max_entries)()
    cnt = (c_int * max_entries)()
    n = lib().dc_profile_read(names, ms, cnt, max_entries)
    out = {}
    for k in range(min(n, max_entries)):
        name = names.raw[64 * k: 64 * (k + 1)].split(b"\0", 1)[0].decode()
        out[name] = (float(ms[k]), int(cnt[k]))
    return out


def aft_trace(enable: bool = True, modes: int = 0xF, device=None):
    """Turn on the per-tile timeline of the AFT tensor-core kernels (mode bits:
    1 forward, 2 backward recompute, 4 dK/dV, 8 dW).  Returns the trace tensor
    [SMs, 64, 8] (uint64 stored as int64) that later launches fill, or None."""
    if not enable:
        check(lib().dc_aft_trace(None, 0, 0), "dc_aft_trace")
        return None
    props = torch.cuda.get_device_properties(device or torch.cuda.current_device())
    buf = torch.zeros(props.multi_processor_count, 64, 8, dtype=torch.int64, device=device or "cuda")
    check(lib().dc_aft_trace(buf.data_ptr(), buf.numel() * 8, int(modes)), "dc_aft_trace")
    return buf
