"""Generate golden vectors by running the REFERENCE engine itself.

The reference library (``oracle/_ref/libmat_mul_ref.so``, compiled from the
reference's own ``native/src/engine.cu`` by ``make -C oracle ref``) is driven
through its own C ABI — ``create_tensor``, ``aft_forward``,
``aft_cross_forward``, ``layernorm_forward``, ``add_tensor_row_broadcast``,
``cross_entropy_loss``, ``mul_tensors``, ``sum_tensor``, ``backward``,
``get_tensor_data`` / ``get_tensor_grad`` — the same calls its Python front end
makes (python/dart_cuda/core/tensor/gpu_tensor.py:261-266).  Gradients are
obtained by back-propagating ``L = sum(out * dOut)`` so that the op under test
receives ``dOut`` as its upstream gradient.

The reference kernels need a GPU, so this script runs on a GPU machine:

    python tests/golden/make_golden.py --out <dir>

and the ``.npz`` files it writes are committed under ``tests/golden/``.
Inputs are seeded (numpy ``default_rng``) and stored next to the outputs.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402


def aft_case(E: oracle.RefEngine, seed: int, B: int, T: int, D: int, masked: bool, wscale: float):
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((B, T, D)).astype(np.float32)
    K = rng.standard_normal((B, T, D)).astype(np.float32)
    V = rng.standard_normal((B, T, D)).astype(np.float32)
    W = (wscale * rng.standard_normal((T, T))).astype(np.float32)
    dZ = rng.standard_normal((B, T, D)).astype(np.float32)
    Z = np.empty_like(Q)
    dQ = np.empty_like(Q)
    dK = np.empty_like(Q)
    dV = np.empty_like(Q)
    dW = np.zeros_like(W)
    # B sequential reference calls, one per sequence; the bias gradient of the
    # shared W is the sum of the per-sequence gradients.
    for b in range(B):
        z, q, k, v, w = E.aft(Q[b], K[b], V[b], W, dZ[b], masked)
        Z[b], dQ[b], dK[b], dV[b] = z, q, k, v
        dW += w
    return dict(Q=Q, K=K, V=V, W=W, dZ=dZ, Z=Z, dQ=dQ, dK=dK, dV=dV, dW=dW,
                masked=np.int32(masked), seed=np.int32(seed))


def cross_case(E: oracle.RefEngine, seed: int, TDec: int, TEnc: int, D: int):
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((TDec, D)).astype(np.float32)
    K = rng.standard_normal((TEnc, D)).astype(np.float32)
    V = rng.standard_normal((TEnc, D)).astype(np.float32)
    W = (0.3 * rng.standard_normal((TDec, TEnc))).astype(np.float32)
    dZ = rng.standard_normal((TDec, D)).astype(np.float32)
    L = E.L
    hq, _ = E.tensor(Q); hk, _ = E.tensor(K); hv, _ = E.tensor(V); hw, _ = E.tensor(W)
    hz = L.aft_cross_forward(hq, hk, hv, hw)
    Z = E.data(hz, Q.shape)
    s, extra = E.weighted_sum(hz, Q.shape, dZ)
    L.backward(s)
    out = dict(Q=Q, K=K, V=V, W=W, dZ=dZ, Z=Z, dQ=E.grad(hq, Q.shape), dK=E.grad(hk, K.shape),
               dV=E.grad(hv, V.shape), dW=E.grad(hw, W.shape), seed=np.int32(seed))
    E.free(s, *extra, hz, hq, hk, hv, hw)
    return out


def layernorm_case(E: oracle.RefEngine, seed: int, R: int, C: int):
    rng = np.random.default_rng(seed)
    x = (2 * rng.standard_normal((R, C)) + 0.5).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal((1, C))).astype(np.float32)
    beta = (0.1 * rng.standard_normal((1, C))).astype(np.float32)
    dy = rng.standard_normal((R, C)).astype(np.float32)
    L = E.L
    hx, _ = E.tensor(x); hg, _ = E.tensor(gamma); hb, _ = E.tensor(beta)
    hy = L.layernorm_forward(hx, hg, hb, 1e-5)
    y = E.data(hy, x.shape)
    s, extra = E.weighted_sum(hy, x.shape, dy)
    L.backward(s)
    out = dict(x=x, gamma=gamma, beta=beta, dy=dy, y=y, dx=E.grad(hx, x.shape),
               dgamma=E.grad(hg, gamma.shape), dbeta=E.grad(hb, beta.shape), seed=np.int32(seed))
    E.free(s, *extra, hy, hx, hg, hb)
    return out


def bias_case(E: oracle.RefEngine, seed: int, M: int, N: int):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, N)).astype(np.float32)
    b = rng.standard_normal((1, N)).astype(np.float32)
    dy = rng.standard_normal((M, N)).astype(np.float32)
    L = E.L
    ha, _ = E.tensor(a); hb, _ = E.tensor(b)
    hy = L.add_tensor_row_broadcast(ha, hb)
    y = E.data(hy, a.shape)
    s, extra = E.weighted_sum(hy, a.shape, dy)
    L.backward(s)
    out = dict(a=a, b=b, dy=dy, y=y, da=E.grad(ha, a.shape), db=E.grad(hb, b.shape), seed=np.int32(seed))
    E.free(s, *extra, hy, ha, hb)
    return out


def ce_case(E: oracle.RefEngine, seed: int, T: int, V: int):
    rng = np.random.default_rng(seed)
    x = (2 * rng.standard_normal((T, V))).astype(np.float32)
    y = rng.integers(0, V, T).astype(np.int32)
    L = E.L
    hx, _ = E.tensor(x)
    hl = L.cross_entropy_loss(hx, y.ctypes.data_as(oracle._IP), T, V)
    loss = E.data(hl, (1, 1))
    L.backward(hl)
    out = dict(logits=x, targets=y, loss=loss, dlogits=E.grad(hx, x.shape), seed=np.int32(seed))
    E.free(hl, hx)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent))
    ap.add_argument("--lib", default=str(oracle.REF_LIB_PATH))
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    E = oracle.RefEngine(args.lib)

    cases = {
        # the fp32 AFT-full workload: B=4, T=64, d=128, w ~ N(0, 0.02)
        "aft_full_b4_t64_d128_causal": aft_case(E, 101, 4, 64, 128, True, 0.02),
        "aft_full_b2_t64_d128_full": aft_case(E, 102, 2, 64, 128, False, 0.02),
        # ragged and degenerate shapes, larger bias spread
        "aft_full_b1_t1_d1_causal": aft_case(E, 103, 1, 1, 1, True, 0.5),
        "aft_full_b3_t7_d5_causal": aft_case(E, 104, 3, 7, 5, True, 0.5),
        "aft_full_b2_t130_d24_causal": aft_case(E, 105, 2, 130, 24, True, 0.5),
        "aft_full_b1_t33_d9_full": aft_case(E, 106, 1, 33, 9, False, 0.5),
        "aft_cross_t9_te5_d12": cross_case(E, 107, 9, 5, 12),
        "aft_cross_t16_te1_d8": cross_case(E, 108, 16, 1, 8),
        "layernorm_r64_c256": layernorm_case(E, 109, 64, 256),
        "layernorm_r3_c7": layernorm_case(E, 110, 3, 7),
        "bias_m64_n96": bias_case(E, 111, 64, 96),
        "bias_m5_n3": bias_case(E, 112, 5, 3),
        "ce_t64_v65": ce_case(E, 113, 64, 65),
        "ce_t4_v8192": ce_case(E, 114, 4, 8192),
    }
    for name, arrs in cases.items():
        np.savez_compressed(out / f"{name}.npz", **arrs)
        print("wrote", name, {k: v.shape for k, v in arrs.items()})


if __name__ == "__main__":
    main()
