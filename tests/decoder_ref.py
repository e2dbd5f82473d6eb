"""Float64 restatement of the AFT decoder step for the decoder tests (test
infrastructure: the checker, never the product).

Follows the reference's layers: pre-LN blocks (transformer_decoder_block.dart:56-79),
LayerNorm eps 1e-5 (layer_norm.dart:9), AFT-full per head
(native/src/kernels/attention.cuh:6-40), cross-AFT against one encoder row
(sigmoid(q) * v0, attention.cuh:41-128 at TEnc = 1), tanh GELU
(native/src/kernels/elementwise.cuh:328-337), label-smoothed cross-entropy
with eps 0.1 (native/src/engine.cu:825-877), mean over all tokens."""
import math

import torch


def layer_norm(x, g, b, eps=1e-5):
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    return (x - mu) / torch.sqrt(var + eps) * g + b


def gelu(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608 * (x + 0.044715 * x ** 3)))


def aft_causal(q, k, v, w):
    """q, k, v [B, T, D]; w [T, T] -> Z [B, T, D]."""
    T = q.shape[1]
    s = k[:, None, :, :] + w[None, :, :, None]  # [B, t, i, D]
    mask = torch.tril(torch.ones(T, T, dtype=torch.bool))
    s = torch.where(mask[None, :, :, None], s, torch.tensor(-math.inf, dtype=s.dtype))
    a = torch.softmax(s, dim=2)
    return torch.sigmoid(q) * (a * v[:, None, :, :]).sum(2)


def forward(P, cfg, idx, targets=None, eps=0.1):
    """P: name -> float64 tensor (internal layout of AftDecoder).  Returns
    (logits [B*T, V], loss)."""
    B, T = idx.shape
    d, H, hs, V = cfg.d_model, cfg.n_heads, cfg.head, cfg.vocab
    x = P["wte"][idx.long()] + P["wpe"][:T]
    for l in range(cfg.n_layers):
        a1 = layer_norm(x, P[f"{l}.ln1g"], P[f"{l}.ln1b"])
        qkv = a1 @ P[f"{l}.wqkv"] + P[f"{l}.bqkv"]
        zs = []
        for h in range(H):
            q, k, v = (qkv[..., j * d + h * hs: j * d + (h + 1) * hs] for j in range(3))
            zs.append(aft_causal(q, k, v, P[f"{l}.pos"][h][:T, :T]))
        z = torch.cat(zs, -1)
        x1 = x + z @ P[f"{l}.wo"] + P[f"{l}.bo"]
        a2 = layer_norm(x1, P[f"{l}.ln2g"], P[f"{l}.ln2b"])
        qc = a2 @ P[f"{l}.wcq"] + P[f"{l}.bcq"]
        cg = torch.sigmoid(qc) * P[f"{l}.bcv"]
        x2 = x1 + cg @ P[f"{l}.wco"] + P[f"{l}.bco"]
        a3 = layer_norm(x2, P[f"{l}.ln3g"], P[f"{l}.ln3b"])
        x = x2 + gelu(a3 @ P[f"{l}.w1"] + P[f"{l}.b1"]) @ P[f"{l}.w2"] + P[f"{l}.b2"]
    af = layer_norm(x, P["lnfg"], P["lnfb"])
    logits = (af @ P["wlm"][:, :V] + P["blm"]).reshape(B * T, V)
    if targets is None:
        return logits, None
    lse = torch.logsumexp(logits, -1)
    nll = lse - logits.gather(1, targets.reshape(-1, 1).long())[:, 0]
    smooth = lse - logits.mean(-1)
    return logits, ((1 - eps) * nll + eps * smooth).mean()
