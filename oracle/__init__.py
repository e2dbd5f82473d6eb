"""CPU oracle for the AFT-full training hot path — TEST INFRASTRUCTURE ONLY.

This package is the checker.  Only ``tests/``, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` may import it; the product library under
``dart_cuda_b200/`` never does.

Two independent restatements live here:

* ``liboracle.so`` (built from ``aft_oracle.c`` by ``make -C oracle``): a
  line-for-line fp32 C restatement of the reference kernels, parallel over
  rows with OpenMP.  Each function in ``aft_oracle.c`` cites the reference
  file:line it follows.
* ``aft_f64`` / ``*_f64`` below: float64 numpy formulations of the same maths,
  used to check the C restatement and for finite-difference gradient checks.

``ref_lib()`` optionally opens ``oracle/_ref/libmat_mul_ref.so`` — the
reference engine compiled from its own sources by ``make -C oracle ref`` — and
drives it through its own C ABI (``create_tensor``/``aft_forward``/
``backward``/``get_tensor_grad``), exactly as its Python front end does
(python/dart_cuda/core/tensor/cuda_engine.py:92-199).  That library needs a GPU.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_bool, c_float, c_int, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libmat_mul_ref.so"

_FP = POINTER(c_float)
_IP = POINTER(c_int)

_lib = None


def build() -> None:
    """Compile ``liboracle.so`` with gcc (no GPU needed)."""
    import subprocess

    subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True,
                   stdout=subprocess.DEVNULL)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        sig = {
            "oracle_aft_full_fwd": [_FP] * 5 + [c_int] * 5,
            "oracle_aft_full_bwd": [_FP] * 9 + [c_int] * 5,
            "oracle_aft_cross_fwd": [_FP] * 5 + [c_int] * 3,
            "oracle_aft_cross_bwd": [_FP] * 9 + [c_int] * 3,
            "oracle_layernorm_fwd": [_FP] * 4 + [c_int, c_int, c_float],
            "oracle_layernorm_bwd": [_FP] * 6 + [c_int, c_int, c_float],
            "oracle_add_row_broadcast_fwd": [_FP] * 3 + [c_int, c_int],
            "oracle_add_row_broadcast_bwd": [_FP] * 3 + [c_int, c_int],
            "oracle_ce_fwd": [_FP, _IP, _FP, c_int, c_int, c_float],
            "oracle_ce_bwd": [_FP, _IP, _FP, c_int, c_int, c_float, c_float],
            "oracle_adam": [_FP] * 4 + [c_int, c_int] + [c_float] * 4,
            "oracle_set_threads": [c_int],
            "oracle_num_threads": [],
        }
        for name, args in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = None
        L.oracle_ce_mean.argtypes = [_FP, c_int]
        L.oracle_ce_mean.restype = c_float
        L.oracle_num_threads.restype = c_int
        _lib = L
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_FP)


def _i(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_IP)


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def num_threads() -> int:
    return int(lib().oracle_num_threads())


# ---------------------------------------------------------------------------
# fp32 C restatement
# ---------------------------------------------------------------------------
def aft_full_fwd(Q, K, V, W, masked=True, ldw=None):
    """Z for Q,K,V [B,T,D] (or [T,D]) fp32 and W [T, ldw] fp32."""
    Q3, K3, V3 = (np.ascontiguousarray(x, np.float32).reshape((-1,) + x.shape[-2:]) for x in (Q, K, V))
    B, T, D = Q3.shape
    W = np.ascontiguousarray(W, np.float32)
    ldw = T if ldw is None else ldw
    Z = np.empty_like(Q3)
    lib().oracle_aft_full_fwd(_f(Q3), _f(K3), _f(V3), _f(W), _f(Z), B, T, D, int(masked), ldw)
    return Z.reshape(np.shape(Q))


def aft_full_bwd(Q, K, V, W, dZ, masked=True, ldw=None, grads=None):
    """(dQ, dK, dV, dW) accumulated into ``grads`` (zeros when None)."""
    Q3, K3, V3, G3 = (np.ascontiguousarray(x, np.float32).reshape((-1,) + x.shape[-2:]) for x in (Q, K, V, dZ))
    B, T, D = Q3.shape
    W = np.ascontiguousarray(W, np.float32)
    ldw = T if ldw is None else ldw
    if grads is None:
        grads = (np.zeros_like(Q3), np.zeros_like(K3), np.zeros_like(V3), np.zeros_like(W))
    dQ, dK, dV, dW = grads
    lib().oracle_aft_full_bwd(_f(Q3), _f(K3), _f(V3), _f(W), _f(G3), _f(dQ), _f(dK), _f(dV), _f(dW),
                              B, T, D, int(masked), ldw)
    return dQ, dK, dV, dW


def aft_cross_fwd(Q, K, V, W):
    Q, K, V, W = (np.ascontiguousarray(x, np.float32) for x in (Q, K, V, W))
    TDec, D = Q.shape
    TEnc = K.shape[0]
    Z = np.empty_like(Q)
    lib().oracle_aft_cross_fwd(_f(Q), _f(K), _f(V), _f(W), _f(Z), TDec, TEnc, D)
    return Z


def aft_cross_bwd(Q, K, V, W, dZ):
    Q, K, V, W, dZ = (np.ascontiguousarray(x, np.float32) for x in (Q, K, V, W, dZ))
    TDec, D = Q.shape
    TEnc = K.shape[0]
    dQ, dK, dV, dW = (np.zeros_like(x) for x in (Q, K, V, W))
    lib().oracle_aft_cross_bwd(_f(Q), _f(K), _f(V), _f(W), _f(dZ), _f(dQ), _f(dK), _f(dV), _f(dW),
                               TDec, TEnc, D)
    return dQ, dK, dV, dW


def layernorm_fwd(x, gamma, beta, eps=1e-5):
    x, gamma, beta = (np.ascontiguousarray(a, np.float32) for a in (x, gamma, beta))
    R, C = x.shape
    y = np.empty_like(x)
    lib().oracle_layernorm_fwd(_f(x), _f(gamma), _f(beta), _f(y), R, C, eps)
    return y


def layernorm_bwd(x, gamma, go, eps=1e-5):
    x, gamma, go = (np.ascontiguousarray(a, np.float32) for a in (x, gamma, go))
    R, C = x.shape
    gx = np.zeros_like(x)
    gg = np.zeros(C, np.float32)
    gb = np.zeros(C, np.float32)
    lib().oracle_layernorm_bwd(_f(x), _f(gamma), _f(go), _f(gx), _f(gg), _f(gb), R, C, eps)
    return gx, gg, gb


def bias_fwd(a, b):
    a, b = (np.ascontiguousarray(x, np.float32) for x in (a, b))
    M, N = a.shape
    out = np.empty_like(a)
    lib().oracle_add_row_broadcast_fwd(_f(a), _f(b), _f(out), M, N)
    return out


def bias_bwd(go):
    go = np.ascontiguousarray(go, np.float32)
    M, N = go.shape
    ga = np.zeros_like(go)
    gb = np.zeros(N, np.float32)
    lib().oracle_add_row_broadcast_bwd(_f(go), _f(ga), _f(gb), M, N)
    return ga, gb


def ce_fwd(logits, targets, eps=0.1):
    """(mean loss, per-row losses)."""
    logits = np.ascontiguousarray(logits, np.float32)
    targets = np.ascontiguousarray(targets, np.int32)
    T, V = logits.shape
    rows = np.empty(T, np.float32)
    lib().oracle_ce_fwd(_f(logits), _i(targets), _f(rows), T, V, eps)
    return float(lib().oracle_ce_mean(_f(rows), T)), rows


def ce_bwd(logits, targets, grad_output=1.0, eps=0.1):
    logits = np.ascontiguousarray(logits, np.float32)
    targets = np.ascontiguousarray(targets, np.int32)
    T, V = logits.shape
    g = np.empty_like(logits)
    lib().oracle_ce_bwd(_f(logits), _i(targets), _f(g), T, V, float(grad_output), eps)
    return g


def adam(p, g, m, v, t, lr, b1=0.9, b2=0.999, eps=1e-8):
    """In-place AdamW update of p, m, v (fp32 arrays)."""
    lib().oracle_adam(_f(p), _f(np.ascontiguousarray(g, np.float32)), _f(m), _f(v), p.size, int(t),
                      lr, b1, b2, eps)


# ---------------------------------------------------------------------------
# float64 formulations (independent of the C code)
# ---------------------------------------------------------------------------
def aft_f64(Q, K, V, W, masked=True):
    """Z for [B,T,D] (or [T,D]) inputs; joint-max stabilised, float64."""
    Q, K, V = (np.asarray(x, np.float64) for x in (Q, K, V))
    squeeze = Q.ndim == 2
    if squeeze:
        Q, K, V = Q[None], K[None], V[None]
    T = Q.shape[1]
    Tk = K.shape[1]
    W = np.asarray(W, np.float64)[:T, :Tk]
    # e[b,t,i,d] = K[b,i,d] + W[t,i]
    e = K[:, None, :, :] + W[None, :, :, None]
    if masked:
        mask = np.tril(np.ones((T, Tk), bool))[None, :, :, None]
        e = np.where(mask, e, -np.inf)
    mx = e.max(axis=2, keepdims=True)
    p = np.exp(e - mx)
    num = (p * V[:, None, :, :]).sum(2)
    den = p.sum(2)
    Z = 1.0 / (1.0 + np.exp(-Q)) * num / den
    return Z[0] if squeeze else Z


def aft_grads_f64(Q, K, V, W, dZ, masked=True):
    """(dQ, dK, dV, dW) in float64, closed form; dW sums over the batch."""
    Q, K, V, dZ = (np.asarray(x, np.float64) for x in (Q, K, V, dZ))
    squeeze = Q.ndim == 2
    if squeeze:
        Q, K, V, dZ = Q[None], K[None], V[None], dZ[None]
    T = Q.shape[1]
    Tk = K.shape[1]
    W = np.asarray(W, np.float64)[:T, :Tk]
    e = K[:, None, :, :] + W[None, :, :, None]
    if masked:
        mask = np.tril(np.ones((T, Tk), bool))[None, :, :, None]
        e = np.where(mask, e, -np.inf)
    mx = e.max(axis=2, keepdims=True)
    p = np.exp(e - mx)                       # [B,T,I,D]
    den = p.sum(2)                           # [B,T,D]
    num = (p * V[:, None]).sum(2)
    r = num / den
    s = 1.0 / (1.0 + np.exp(-Q))
    dQ = dZ * r * s * (1 - s)
    g = dZ * s / den                         # [B,T,D]
    # d/d(exponent) of num/den for entry (t,i,d): p*(V_i - r_t)/den
    coef = p * (V[:, None] - r[:, :, None]) * g[:, :, None]   # [B,T,I,D]
    dK = coef.sum(1)
    dV = (p * g[:, :, None]).sum(1)
    dW = coef.sum(axis=(0, 3))
    if squeeze:
        return dQ[0], dK[0], dV[0], dW
    return dQ, dK, dV, dW


# ---------------------------------------------------------------------------
# reference engine driven through its own C ABI (needs a GPU)
# ---------------------------------------------------------------------------
class RefEngine:
    """The reference ``libmat_mul`` driven through its own exported symbols."""

    def __init__(self, path: str | os.PathLike = REF_LIB_PATH):
        L = ctypes.CDLL(str(path))
        VP = c_void_p
        L.create_tensor.restype = VP
        L.create_tensor.argtypes = [c_int, c_int, _FP]
        L.destroy_tensor.argtypes = [VP]
        L.get_tensor_data.argtypes = [VP, _FP]
        L.get_tensor_grad.argtypes = [VP, _FP]
        L.set_tensor_data.argtypes = [VP, _FP]
        L.aft_forward.restype = VP
        L.aft_forward.argtypes = [VP, VP, VP, VP, c_bool]
        L.aft_cross_forward.restype = VP
        L.aft_cross_forward.argtypes = [VP, VP, VP, VP]
        L.backward.argtypes = [VP]
        L.zero_grad.argtypes = [VP]
        L.layernorm_forward.restype = VP
        L.layernorm_forward.argtypes = [VP, VP, VP, c_float]
        L.add_tensor_row_broadcast.restype = VP
        L.add_tensor_row_broadcast.argtypes = [VP, VP]
        L.cross_entropy_loss.restype = VP
        L.cross_entropy_loss.argtypes = [VP, _IP, c_int, c_int]
        L.mul_tensors.restype = VP
        L.mul_tensors.argtypes = [VP, VP]
        L.sum_tensor.restype = VP
        L.sum_tensor.argtypes = [VP]
        L.matmul_tensors.restype = VP
        L.matmul_tensors.argtypes = [VP, VP]
        L.gelu_tensor.restype = VP
        L.gelu_tensor.argtypes = [VP]
        L.add_tensors.restype = VP
        L.add_tensors.argtypes = [VP, VP]
        L.embedding_forward.restype = VP
        L.embedding_forward.argtypes = [_IP, VP, VP, c_int, c_int]
        L.adam_step.restype = None
        L.adam_step.argtypes = [VP, VP, VP, c_int, c_float, c_float, c_float, c_float]
        L.concat_tensors_gpu.restype = VP
        L.concat_tensors_gpu.argtypes = [POINTER(VP), c_int]
        self.L = L

    def tensor(self, a: np.ndarray):
        a = np.ascontiguousarray(a, np.float32)
        r = a.shape[0]
        c = int(np.prod(a.shape[1:])) if a.ndim > 1 else 1
        return self.L.create_tensor(r, c, _f(a)), a.shape

    def data(self, h, shape):
        out = np.empty(shape, np.float32)
        self.L.get_tensor_data(h, _f(out))
        return out

    def grad(self, h, shape):
        out = np.empty(shape, np.float32)
        self.L.get_tensor_grad(h, _f(out))
        return out

    def free(self, *hs):
        for h in hs:
            self.L.destroy_tensor(h)

    def weighted_sum(self, out_h, out_shape, dZ):
        """Scalar L = sum(out * dZ) so that backward seeds out.grad = dZ."""
        g, _ = self.tensor(dZ)
        prod = self.L.mul_tensors(out_h, g)
        s = self.L.sum_tensor(prod)
        return s, [g, prod]

    def aft(self, Q, K, V, W, dZ, masked=True):
        """One [T,D] sequence through aft_forward + backward; returns
        (Z, dQ, dK, dV, dW).  W must already be [T, T] (row stride T)."""
        hq, sq = self.tensor(Q)
        hk, sk = self.tensor(K)
        hv, sv = self.tensor(V)
        hw, sw = self.tensor(W)
        hz = self.L.aft_forward(hq, hk, hv, hw, bool(masked))
        Z = self.data(hz, sq)
        s, extra = self.weighted_sum(hz, sq, dZ)
        self.L.backward(s)
        res = (Z, self.grad(hq, sq), self.grad(hk, sk), self.grad(hv, sv), self.grad(hw, sw))
        self.free(s, *extra, hz, hq, hk, hv, hw)
        return res
