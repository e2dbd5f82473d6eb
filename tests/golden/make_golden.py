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
import ctypes
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


def matmul_case(E: oracle.RefEngine, seed: int, M: int, K: int, N: int):
    """matmul_tensors (native/src/engine.cu:480-507, matmul.cuh:27-131) and
    its two backward products."""
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    dC = rng.standard_normal((M, N)).astype(np.float32)
    ha, _ = E.tensor(A); hb, _ = E.tensor(B)
    hc = E.L.matmul_tensors(ha, hb)
    C = E.data(hc, (M, N))
    s, extra = E.weighted_sum(hc, (M, N), dC)
    E.L.backward(s)
    out = dict(A=A, B=B, dC=dC, C=C, dA=E.grad(ha, A.shape), dB=E.grad(hb, B.shape), seed=np.int32(seed))
    E.free(s, *extra, hc, ha, hb)
    return out


def gelu_case(E: oracle.RefEngine, seed: int, R: int, C: int):
    """gelu_tensor (native/src/engine.cu:445-458, elementwise.cuh gelu_fwd/bwd)."""
    rng = np.random.default_rng(seed)
    x = (2 * rng.standard_normal((R, C))).astype(np.float32)
    dy = rng.standard_normal((R, C)).astype(np.float32)
    hx, _ = E.tensor(x)
    hy = E.L.gelu_tensor(hx)
    y = E.data(hy, x.shape)
    s, extra = E.weighted_sum(hy, x.shape, dy)
    E.L.backward(s)
    out = dict(x=x, dy=dy, y=y, dx=E.grad(hx, x.shape), seed=np.int32(seed))
    E.free(s, *extra, hy, hx)
    return out


def embedding_case(E: oracle.RefEngine, seed: int, V: int, Tmax: int, T: int, D: int):
    """embedding_forward (native/src/engine.cu:794-822): out[t] = wte[idx[t]] +
    wpe[t]; the backward scatters into wte's rows (repeated ids add up) and
    wpe's first T rows."""
    rng = np.random.default_rng(seed)
    wte = rng.standard_normal((V, D)).astype(np.float32)
    wpe = rng.standard_normal((Tmax, D)).astype(np.float32)
    idx = rng.integers(0, V, T).astype(np.int32)
    idx[: min(3, T)] = idx[0]  # repeated ids
    dy = rng.standard_normal((T, D)).astype(np.float32)
    hte, _ = E.tensor(wte); hpe, _ = E.tensor(wpe)
    hy = E.L.embedding_forward(idx.ctypes.data_as(oracle._IP), hte, hpe, T, D)
    y = E.data(hy, (T, D))
    s, extra = E.weighted_sum(hy, (T, D), dy)
    E.L.backward(s)
    out = dict(wte=wte, wpe=wpe, idx=idx, dy=dy, y=y, dwte=E.grad(hte, wte.shape),
               dwpe=E.grad(hpe, wpe.shape), seed=np.int32(seed))
    E.free(s, *extra, hy, hte, hpe)
    return out


def adam_case(E: oracle.RefEngine, seed: int, R: int, C: int, steps: int, lr: float):
    """adam_step (native/src/engine.cu:887-905, loss_optim.cuh:255-298) for
    `steps` consecutive steps t = 1..steps (the value the front end passes,
    lib/core/optimizers/adam.dart:603-637); p's gradient of step k is set by
    back-propagating sum(p * G_k) after zero_grad."""
    rng = np.random.default_rng(seed)
    p = rng.standard_normal((R, C)).astype(np.float32)
    Gs = (0.5 * rng.standard_normal((steps, R, C))).astype(np.float32)
    hp, _ = E.tensor(p)
    hm, _ = E.tensor(np.zeros((R, C), np.float32))
    hv, _ = E.tensor(np.zeros((R, C), np.float32))
    ps, ms, vs = [], [], []
    for k in range(steps):
        E.L.zero_grad(hp)
        s, extra = E.weighted_sum(hp, (R, C), Gs[k])
        E.L.backward(s)
        E.L.adam_step(hp, hm, hv, k + 1, lr, 0.9, 0.999, 1e-8)
        ps.append(E.data(hp, (R, C)))
        ms.append(E.data(hm, (R, C)))
        vs.append(E.data(hv, (R, C)))
        E.free(s, *extra)
    E.free(hp, hm, hv)
    return dict(p0=p, G=Gs, p=np.stack(ps), m=np.stack(ms), v=np.stack(vs), lr=np.float32(lr),
                seed=np.int32(seed))


def decoder_case(E: oracle.RefEngine, seed: int, vocab: int, d: int, n_layers: int, n_heads: int, T: int):
    """One sequence through a TransformerDecoder built from the reference
    engine's own handle ops, composed as the reference's layers compose them
    (lib/core/transformers/aft/transformer_decoder.dart, transformer_decoder_block.dart:
    pre-LN blocks; MultiHeadAFT: per-head Q/K/V Layers, aft_forward on the
    head's posBias, concat, projection; MultiHeadAFTCross against the dummy
    [1, d] zero encoder with aft_cross_forward; FeedForward with gelu_tensor;
    residual add_tensors; final LayerNorm; LM head; cross_entropy_loss),
    then backward from the loss.  A Layer is matmul_tensors followed by
    add_tensor_row_broadcast of its [1, out] bias.  Parameters are N(0, 0.2)
    (LayerNorm gains 1 + N(0, 0.1)) in the reference's parameters() order;
    names and shapes come from the decoder's reference-order view."""
    from dart_cuda_b200.decoder import AftDecoder, DecoderConfig

    cfg = DecoderConfig(vocab=vocab, d_model=d, n_layers=n_layers, n_heads=n_heads, block_size=T)
    names = [(n, tuple(v.shape)) for n, v in AftDecoder(cfg, device="cpu").reference_parameters()]
    rng = np.random.default_rng(seed)
    P = {}
    for n, shp in names:
        if n.endswith("gamma"):
            P[n] = (1 + 0.1 * rng.standard_normal(shp)).astype(np.float32)
        else:
            P[n] = (0.2 * rng.standard_normal(shp)).astype(np.float32)
    idx = rng.integers(0, vocab, T).astype(np.int32)
    tgt = rng.integers(0, vocab, T).astype(np.int32)
    L = E.L
    H = {n: E.tensor(a)[0] for n, a in P.items()}
    keep = []

    def k(h):
        keep.append(h)
        return h

    def layer(x, pre):
        return k(L.add_tensor_row_broadcast(k(L.matmul_tensors(x, H[pre + ".w"])), H[pre + ".b"]))

    def concat(hs):
        arr = (ctypes.c_void_p * len(hs))(*hs)
        return k(L.concat_tensors_gpu(ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)), len(hs)))

    def ln(x, pre):
        return k(L.layernorm_forward(x, H[pre + ".gamma"], H[pre + ".beta"], 1e-5))

    x = k(L.embedding_forward(idx.ctypes.data_as(oracle._IP), H["wte"], H["wpe"], T, d))
    enc = k(E.tensor(np.zeros((1, cfg.enc), np.float32))[0])
    for l in range(n_layers):
        pre = f"blocks[{l}]"
        a1 = ln(x, pre + ".ln1")
        zs = []
        for h in range(n_heads):
            hp = f"{pre}.self.heads[{h}]"
            q, kk, v = (layer(a1, f"{hp}.{nm}") for nm in "qkv")
            zs.append(k(L.aft_forward(q, kk, v, H[hp + ".posBias"], True)))
        x1 = k(L.add_tensors(x, layer(concat(zs), pre + ".self.proj")))
        a2 = ln(x1, pre + ".ln2")
        cs = []
        for h in range(n_heads):
            hp = f"{pre}.cross.heads[{h}]"
            q = layer(a2, hp + ".q")
            kk, v = layer(enc, hp + ".k"), layer(enc, hp + ".v")
            cs.append(k(L.aft_cross_forward(q, kk, v, H[hp + ".posBias"])))
        x2 = k(L.add_tensors(x1, layer(concat(cs), pre + ".cross.proj")))
        a3 = ln(x2, pre + ".ln3")
        f = k(L.gelu_tensor(layer(a3, pre + ".ffn.w1")))
        x = k(L.add_tensors(x2, layer(f, pre + ".ffn.w2")))
    af = ln(x, "finalLayerNorm")
    logits = layer(af, "lmHead")
    hl = k(L.cross_entropy_loss(logits, tgt.ctypes.data_as(oracle._IP), T, vocab))
    loss = E.data(hl, (1, 1))
    lg = E.data(logits, (T, vocab))
    L.backward(hl)
    out = {"idx": idx, "targets": tgt, "loss": loss, "logits": lg, "seed": np.int32(seed),
           "dims": np.array([vocab, d, n_layers, n_heads, T], np.int32),
           "names": np.array([n for n, _ in names])}
    for n, _ in names:
        out["p:" + n] = P[n]
        out["g:" + n] = E.grad(H[n], P[n].shape)
    E.free(*keep, *H.values())
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent))
    ap.add_argument("--lib", default=str(oracle.REF_LIB_PATH))
    ap.add_argument("--only", default="", help="comma-separated fixture names to (re)write")
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
        "matmul_m37_k50_n29": matmul_case(E, 115, 37, 50, 29),
        "matmul_m128_k256_n65": matmul_case(E, 116, 128, 256, 65),
        "gelu_r64_c96": gelu_case(E, 117, 64, 96),
        "embedding_v65_t13_d16": embedding_case(E, 118, 65, 20, 13, 16),
        "adam_r50_c7_s3": adam_case(E, 119, 50, 7, 3, 1e-2),
        "decoder_v11_d32_l2_h2_t16": decoder_case(E, 120, 11, 32, 2, 2, 16),
    }
    only = set(args.only.split(",")) if args.only else None
    cases = {k: v for k, v in cases.items() if only is None or k in only}
    for name, arrs in cases.items():
        np.savez_compressed(out / f"{name}.npz", **arrs)
        print("wrote", name, {k: v.shape for k, v in arrs.items()})


if __name__ == "__main__":
    main()
