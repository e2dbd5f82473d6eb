"""The reference's AFT decoder on the library's batched kernels.

Mirrors ``TransformerDecoder`` and its parts
(lib/core/transformers/aft/transformer_decoder.dart,
lib/core/transformers/aft/transformer_decoder_block.dart,
lib/core/attention/aft_multi_head_attention.dart,
lib/core/attention/aft_multi_head_cross_attention.dart,
lib/core/attention/aft.dart, lib/core/attention/aft_cross_attention.dart,
lib/core/layers/feed_forward.dart, lib/core/layers/layer_norm.dart,
lib/core/layers/nn.dart) for B sequences per call instead of one:

    block(x) = x1 + FFN(LN3(x2)),  x2 = x1 + CrossAFT(LN2(x1), enc),
               x1 = x + MultiHeadAFT(LN1(x))          (pre-LN, causal self-AFT)

* ``train_step``: forward, label-smoothed cross-entropy (eps 0.1, mean over
  all B*T tokens), backward, an optional all-reduce of the gradients (one
  flat buffer), and one AdamW launch over every parameter
  (native/src/kernels/loss_optim.cuh:255-298, weight decay 0.001).
* ``generate``: the prompt through the batched forward (filling each layer's
  k/v history), then one cached decode step per new token, greedy.  The
  reference re-runs the whole context per token
  (example/bin/shakespear4.dart:176-214).
* ``save`` / ``load``: the reference's checkpoint, flat fp32 in its
  ``parameters()`` order (lib/core/utils/persistence.dart:8-70).

Every computation runs in ``libmat_mul.so``: tcgen05 GEMMs with fused bias /
residual / GELU (dc_gemm), the AFT operator (dc_aft_*_strided, reading each
head's columns out of the fused Q|K|V projection), LayerNorm, cross-entropy,
embedding, the single-row cross-attention gate and AdamW.  PyTorch only
allocates the buffers and supplies the stream.

Parameters are stored for the kernels, not in the reference's order: each
block's per-head Q/K/V layers are one [d, 3d] matrix (columns q heads | k
heads | v heads) and the LM head's rows are padded to a 16-byte stride; the
checkpoint functions translate.  The cross-attention runs against one
encoder row (the reference's dummy ``[1, D]`` zeros): with a single key the
AFT weight cancels and the output is sigmoid(q) * v0 exactly, so its key
projection and bias matrix receive zero gradient, as in the reference.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from . import ops
from ._lib import (DC_AFT_CAUSAL, DC_AFT_SAVE_STATS, DC_AFT_SPARE_SMS, DC_AFT_WS_VALID, DC_F32, check,
                   lib)

_ALIGN = 32  # elements: every parameter starts on a 128-byte boundary


def _up(n, a):
    return (n + a - 1) // a * a


@dataclass
class DecoderConfig:
    vocab: int = 65
    d_model: int = 256
    n_layers: int = 4
    n_heads: int = 4
    block_size: int = 256  # maxSeqLen: rows of wpe and of every posBias
    ffn_mult: int = 4
    enc_dim: int | None = None  # encoderEmbedSize (defaults to d_model)

    @property
    def head(self):
        return self.d_model // self.n_heads

    @property
    def enc(self):
        return self.enc_dim or self.d_model


class AftDecoder:
    # sequence length from which the AFT forward keeps r and 1/den' for the
    # backward instead of the backward repeating the forward contraction
    STATS_FROM_T = 256

    def __init__(self, cfg: DecoderConfig, device="cuda", seed=0, std=0.02):
        if cfg.d_model % cfg.n_heads:
            raise ValueError("d_model must be a multiple of n_heads")
        self.cfg = c = cfg
        self.device = torch.device(device)
        d, H, Tm, E, F, V = c.d_model, c.n_heads, c.block_size, c.enc, c.ffn_mult * c.d_model, c.vocab
        self.Vp = _up(V, 4)
        specs = [("wte", (V, d)), ("wpe", (Tm, d))]
        for l in range(c.n_layers):
            specs += [(f"{l}.wqkv", (d, 3 * d)), (f"{l}.bqkv", (3 * d,)), (f"{l}.pos", (H, Tm, Tm)),
                      (f"{l}.wo", (d, d)), (f"{l}.bo", (d,)),
                      (f"{l}.wcq", (d, d)), (f"{l}.bcq", (d,)), (f"{l}.wck", (E, d)), (f"{l}.bck", (d,)),
                      (f"{l}.wcv", (E, d)), (f"{l}.bcv", (d,)), (f"{l}.cpos", (H, Tm, Tm)),
                      (f"{l}.wco", (d, d)), (f"{l}.bco", (d,)),
                      (f"{l}.w1", (d, F)), (f"{l}.b1", (F,)), (f"{l}.w2", (F, d)), (f"{l}.b2", (d,)),
                      (f"{l}.ln1g", (d,)), (f"{l}.ln1b", (d,)), (f"{l}.ln2g", (d,)), (f"{l}.ln2b", (d,)),
                      (f"{l}.ln3g", (d,)), (f"{l}.ln3b", (d,))]
        specs += [("lnfg", (d,)), ("lnfb", (d,)), ("wlm", (d, self.Vp)), ("blm", (V,))]
        self._offsets = {}
        off = 0
        for name, shape in specs:
            self._offsets[name] = (off, shape)
            off += _up(int(np.prod(shape)), _ALIGN)
        self.numel = off
        dev = self.device
        self.flat = torch.zeros(off, device=dev)
        self.grad = torch.zeros(off, device=dev)
        self.adam_m = torch.zeros(off, device=dev)
        self.adam_v = torch.zeros(off, device=dev)
        self.P = {n: self._view(self.flat, n) for n in self._offsets}
        self.G = {n: self._view(self.grad, n) for n in self._offsets}
        self.t = 0
        self._init(seed, std)
        self._bufs = None
        self._dec = None
        # heads 1.. of each AFT layer run on their own streams (head 0 on the
        # caller's): one head's launches leave most SMs idle at these sizes
        # (B*T/128 row tiles of 64 columns), so the heads run side by side
        self._head_streams = [torch.cuda.Stream(self.device) for _ in range(cfg.n_heads - 1)] \
            if self.device.type == "cuda" else []
        # with the heads on their own streams each head's AFT launch takes
        # 2 SMs / heads CTAs, leaving room for the others': a CTA then runs
        # two or more tiles through its two accumulators instead of paying
        # its set-up for one (decoder training step 2.81 -> 2.75 ms)
        self._head_spare = 0
        if self._head_streams:
            sms = torch.cuda.get_device_properties(self.device).multi_processor_count
            self._head_spare = DC_AFT_SPARE_SMS(min(255, max(0, sms - max(16, 2 * sms // cfg.n_heads))))
        # the backward's weight and bias gradients (off the input-gradient
        # chain) run on a second stream beside it
        self._wgrad_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        # False: every launch on the caller's stream (per-kernel timing)
        self.concurrent = True

    def _view(self, flat, name):
        off, shape = self._offsets[name]
        return flat[off: off + int(np.prod(shape))].view(shape)

    def _init(self, seed, std):
        """Weight matrices, embeddings and pairwise biases ~ N(0, std);
        Layer biases 0; LayerNorm gamma 1, beta 0 (seeded, on the host)."""
        g = torch.Generator().manual_seed(seed)
        for name, (_, shape) in self._offsets.items():
            base = name.split(".")[-1]
            if base.startswith("ln"):
                val = torch.ones(shape) if base.endswith("g") else torch.zeros(shape)
            elif base.startswith("b"):
                val = torch.zeros(shape)
            else:
                val = std * torch.randn(shape, generator=g)
            if name == "wlm":
                val[:, self.cfg.vocab:] = 0.0
            self.P[name].copy_(val)

    # ------------------------------------------------------------ checkpoint
    def reference_parameters(self, grads: bool = False):
        """[(name, view)] in the reference's parameters() order, each view in
        the reference's shape (lib/core/transformers/aft/transformer_decoder.dart:90-97,
        transformer_decoder_block.dart:101-108, aft.dart:71-76,
        aft_cross_attention.dart:39-45, aft_multi_head_*.dart, nn.dart:55).
        grads=True gives the same views of the gradient buffer."""
        c, P = self.cfg, (self.G if grads else self.P)
        d, hs = c.d_model, c.head
        out = [("wte", P["wte"]), ("wpe", P["wpe"])]
        for l in range(c.n_layers):
            pre = f"blocks[{l}]"
            wqkv, bqkv = P[f"{l}.wqkv"], P[f"{l}.bqkv"]
            for h in range(c.n_heads):
                s = slice(h * hs, (h + 1) * hs)
                for j, nm in enumerate("qkv"):
                    cs = slice(j * d + h * hs, j * d + (h + 1) * hs)
                    out += [(f"{pre}.self.heads[{h}].{nm}.w", wqkv[:, cs]),
                            (f"{pre}.self.heads[{h}].{nm}.b", bqkv[cs].view(1, hs))]
                out.append((f"{pre}.self.heads[{h}].posBias", P[f"{l}.pos"][h]))
                del s
            out += [(f"{pre}.self.proj.w", P[f"{l}.wo"]), (f"{pre}.self.proj.b", P[f"{l}.bo"].view(1, d))]
            for h in range(c.n_heads):
                s = slice(h * hs, (h + 1) * hs)
                # AFTCrossAttention.parameters(): key, query, value, posBias
                for nm, w, b in (("k", "wck", "bck"), ("q", "wcq", "bcq"), ("v", "wcv", "bcv")):
                    out += [(f"{pre}.cross.heads[{h}].{nm}.w", P[f"{l}.{w}"][:, s]),
                            (f"{pre}.cross.heads[{h}].{nm}.b", P[f"{l}.{b}"][s].view(1, hs))]
                out.append((f"{pre}.cross.heads[{h}].posBias", P[f"{l}.cpos"][h]))
            out += [(f"{pre}.cross.proj.w", P[f"{l}.wco"]), (f"{pre}.cross.proj.b", P[f"{l}.bco"].view(1, d))]
            F = P[f"{l}.w1"].shape[1]
            out += [(f"{pre}.ffn.w1.w", P[f"{l}.w1"]), (f"{pre}.ffn.w1.b", P[f"{l}.b1"].view(1, F)),
                    (f"{pre}.ffn.w2.w", P[f"{l}.w2"]), (f"{pre}.ffn.w2.b", P[f"{l}.b2"].view(1, d))]
            for k in (1, 2, 3):
                out += [(f"{pre}.ln{k}.gamma", P[f"{l}.ln{k}g"].view(1, d)),
                        (f"{pre}.ln{k}.beta", P[f"{l}.ln{k}b"].view(1, d))]
        out += [("finalLayerNorm.gamma", P["lnfg"].view(1, d)), ("finalLayerNorm.beta", P["lnfb"].view(1, d)),
                ("lmHead.w", P["wlm"][:, : c.vocab]), ("lmHead.b", P["blm"].view(1, c.vocab))]
        return out

    def save(self, path):
        """The reference's saveModuleBinary format: every parameter's fp32
        values, row-major, concatenated in parameters() order, no header."""
        parts = [v.detach().contiguous().view(-1).cpu() for _, v in self.reference_parameters()]
        np.concatenate([p.numpy() for p in parts]).astype("<f4").tofile(str(path))

    def load(self, path):
        """loadModuleBinary: the file must hold exactly the model's floats."""
        data = np.fromfile(str(path), dtype="<f4")
        params = self.reference_parameters()
        need = sum(v.numel() for _, v in params)
        if data.size != need:
            raise ValueError(f"weight file holds {data.size} floats, the model expects {need}")
        off = 0
        for _, v in params:
            n = v.numel()
            v.copy_(torch.from_numpy(data[off: off + n].copy()).view(v.shape))
            off += n

    # ------------------------------------------------------------ buffers
    def _buffers(self, B, T):
        if self._bufs is not None and self._bufs["shape"] == (B, T):
            return self._bufs
        c, dev = self.cfg, self.device
        d, F, V, M = c.d_model, c.ffn_mult * c.d_model, c.vocab, B * T
        if T > c.block_size:
            raise ValueError(f"sequence length {T} exceeds block size {c.block_size}")
        z = lambda *s: torch.zeros(*s, device=dev)
        L = c.n_layers
        b = {"shape": (B, T)}
        b["x"] = [z(M, d) for _ in range(L + 1)]
        for k in ("a1", "z", "x1", "a2", "qc", "cg", "x2", "a3"):
            b[k] = [z(M, d) for _ in range(L)]
        b["qkv"] = [z(M, 3 * d) for _ in range(L)]
        b["u"] = [z(M, F) for _ in range(L)]
        b["h"] = [z(M, F) for _ in range(L)]
        b["af"] = z(M, d)
        b["logits"] = z(M, V)
        b["dX"], b["da"], b["dz"] = z(M, d), z(M, d), z(M, d)
        b["dqkv"], b["dh"] = z(M, 3 * d), z(M, F)
        b["dlog"], b["dlog_pad"] = z(M, V), z(M, self.Vp)
        b["scale"] = torch.ones(1, device=dev)
        b["loss"] = torch.zeros(1, device=dev)
        # one AFT workspace per (layer, head): the forward's panels are reused
        # by the backward; r and 1/den are kept from T >= STATS_FROM_T on
        self._aft_flags = DC_AFT_CAUSAL | (DC_AFT_SAVE_STATS if T >= self.STATS_FROM_T else 0)
        n = ctypes.c_size_t(0)
        check(lib().dc_aft_workspace_size(B, T, T, c.head, DC_F32, self._aft_flags, ctypes.byref(n)),
              "dc_aft_workspace_size")
        self._ws_bytes = _up(int(n.value), 1024)
        b["ws"] = torch.empty(self._ws_bytes * L * c.n_heads + 1024, dtype=torch.uint8, device=dev)
        self._bufs = b
        return b

    def _ws(self, l, h):
        base = (self._bufs["ws"].data_ptr() + 1023) // 1024 * 1024
        return base + (l * self.cfg.n_heads + h) * self._ws_bytes

    # ------------------------------------------------------------ pieces
    def _aft(self, l, qkv, z, B, T, backward=False, dz=None, dqkv=None):
        c = self.cfg
        d, hs, Tm = c.d_model, c.head, c.block_size
        pos, dpos = self.P[f"{l}.pos"], self.G[f"{l}.pos"]
        q0 = qkv.data_ptr()
        main = torch.cuda.current_stream()
        side = self._head_streams if self.concurrent else []
        flags = self._aft_flags | (self._head_spare if side else 0)
        if side:  # fork: the head streams start after what the caller queued
            fork = torch.cuda.Event()
            fork.record(main)
            for s in side:
                s.wait_event(fork)
        for h in range(c.n_heads):
            st = (side[h - 1] if h and side else main).cuda_stream
            Q, K, Vv = (q0 + 4 * (j * d + h * hs) for j in range(3))
            w = pos[h].data_ptr()
            if not backward:
                check(lib().dc_aft_fwd_strided(Q, K, Vv, w, Tm, z.data_ptr() + 4 * h * hs, B, T, T, hs,
                                               3 * d, d, DC_F32, flags, self._ws(l, h),
                                               self._ws_bytes, st), "dc_aft_fwd_strided")
            else:
                g0 = dqkv.data_ptr()
                dQ, dK, dV = (g0 + 4 * (j * d + h * hs) for j in range(3))
                check(lib().dc_aft_bwd_strided(Q, K, Vv, w, Tm, dz.data_ptr() + 4 * h * hs, dQ, dK, dV,
                                               dpos[h].data_ptr(), B, T, T, hs, 3 * d, d, DC_F32,
                                               flags | DC_AFT_WS_VALID, self._ws(l, h),
                                               self._ws_bytes, st), "dc_aft_bwd_strided")
        for s in side:  # join
            done = torch.cuda.Event()
            done.record(s)
            main.wait_event(done)

    def _gate(self, q, v0, out):
        M, N = q.shape
        check(lib().dc_gate_fwd(q.data_ptr(), q.stride(0), v0.data_ptr(), out.data_ptr(), out.stride(0), M, N,
                                ops._stream()), "dc_gate_fwd")

    def _v0(self, l):
        """The cross-attention value of the single encoder row,
        v0 = enc . Wcv + bcv; the dummy encoder is zeros, so v0 = bcv."""
        return self.P[f"{l}.bcv"]

    # ------------------------------------------------------------ training
    def forward(self, idx: torch.Tensor, targets: torch.Tensor | None = None, lm_head: bool = True):
        """Logits [B*T, V] of token ids idx [B, T] (int32, on the device) and,
        with targets, the mean label-smoothed cross-entropy (device scalar).
        Without ``lm_head`` the forward stops after the final LayerNorm."""
        c, P = self.cfg, self.P
        B, T = idx.shape
        b = self._buffers(B, T)
        d, F, V = c.d_model, c.ffn_mult * c.d_model, c.vocab
        st = ops._stream()
        check(lib().dc_embedding_fwd(idx.data_ptr(), P["wte"].data_ptr(), P["wpe"].data_ptr(),
                                     b["x"][0].data_ptr(), B, T, d, V, st), "dc_embedding_fwd")
        for l in range(c.n_layers):
            x = b["x"][l]
            ops.layernorm_fwd(x, P[f"{l}.ln1g"], P[f"{l}.ln1b"], out=b["a1"][l])
            ops.gemm(b["a1"][l], P[f"{l}.wqkv"], out=b["qkv"][l], bias=P[f"{l}.bqkv"])
            self._aft(l, b["qkv"][l], b["z"][l], B, T)
            ops.gemm(b["z"][l], P[f"{l}.wo"], out=b["x1"][l], bias=P[f"{l}.bo"], residual=x)
            ops.layernorm_fwd(b["x1"][l], P[f"{l}.ln2g"], P[f"{l}.ln2b"], out=b["a2"][l])
            ops.gemm(b["a2"][l], P[f"{l}.wcq"], out=b["qc"][l], bias=P[f"{l}.bcq"])
            self._gate(b["qc"][l], self._v0(l), b["cg"][l])
            ops.gemm(b["cg"][l], P[f"{l}.wco"], out=b["x2"][l], bias=P[f"{l}.bco"], residual=b["x1"][l])
            ops.layernorm_fwd(b["x2"][l], P[f"{l}.ln3g"], P[f"{l}.ln3b"], out=b["a3"][l])
            ops.gemm(b["a3"][l], P[f"{l}.w1"], out=b["h"][l], bias=P[f"{l}.b1"], gelu=True, gelu_aux=b["u"][l])
            ops.gemm(b["h"][l], P[f"{l}.w2"], out=b["x"][l + 1], bias=P[f"{l}.b2"], residual=b["x2"][l])
        ops.layernorm_fwd(b["x"][c.n_layers], P["lnfg"], P["lnfb"], out=b["af"])
        if not lm_head:
            return None, None
        ops.gemm(b["af"], P["wlm"][:, :V], out=b["logits"], bias=P["blm"])
        if targets is None:
            return b["logits"], None
        b["idx"], b["targets"] = idx, targets.view(-1)
        return b["logits"], ops.ce_fwd(b["logits"], b["targets"], out=b["loss"])

    def grad_buckets(self):
        """[(start, end)] ranges of ``self.grad`` in the order the backward
        completes them: the LM head, final LayerNorm and last block together,
        then one per earlier block, then the embeddings.  Each range is
        contiguous in the flat buffer."""
        c = self.cfg
        start = [self._offsets[f"{l}.wqkv"][0] for l in range(c.n_layers)] + [self._offsets["lnfg"][0]]
        out = [(start[c.n_layers - 1], self.numel)]
        for l in reversed(range(c.n_layers - 1)):
            out.append((start[l], start[l + 1]))
        out.append((0, start[0]))
        return out

    def backward(self, grad_scale: float = 1.0, bucket_done=None):
        """Gradients of the last forward's loss (times grad_scale) into
        ``self.grad`` (overwritten).  ``bucket_done(k)``, when given, is called
        once the launches that complete bucket k of grad_buckets() have all
        been queued on the caller's stream (every side stream joined back), so
        a data-parallel caller can start that bucket's reduction while the
        rest of the backward runs."""
        c, P, G = self.cfg, self.P, self.G
        b = self._bufs
        B, T = b["shape"]
        d, V = c.d_model, c.vocab
        st = ops._stream()
        self.grad.zero_()
        b["scale"].fill_(grad_scale)
        ops.ce_bwd(b["logits"], b["targets"], grad_scale=b["scale"], out=b["dlog"])
        check(lib().dc_copy2d(b["dlog_pad"].data_ptr(), self.Vp * 4, b["dlog"].data_ptr(), V * 4, V * 4,
                              B * T, st), "dc_copy2d")
        main = torch.cuda.current_stream()
        side = self._wgrad_stream if self.concurrent else main

        def fork():
            """Side work queued after this point sees what main has queued so far."""
            ev = torch.cuda.Event()
            ev.record(main)
            side.wait_event(ev)

        def join():
            """Main waits for all side work queued so far: called before main
            overwrites a buffer the side work reads (dX by the LayerNorm
            backward's accumulation; dh, da and dqkv are rewritten only after
            a later join)."""
            ev = torch.cuda.Event()
            ev.record(side)
            main.wait_event(ev)

        fork()
        with torch.cuda.stream(side):
            ops.gemm(b["af"], b["dlog_pad"], trans_a=True, out=G["wlm"])
            ops.bias_bwd(b["dlog"], grads=(None, G["blm"]))
        ops.gemm(b["dlog_pad"], P["wlm"], trans_b=True, out=b["da"])
        dX = b["dX"]
        ops.layernorm_bwd(b["x"][c.n_layers], P["lnfg"], b["da"], grads=(dX, G["lnfg"], G["lnfb"]))
        for l in reversed(range(c.n_layers)):
            # FFN: x3 = x2 + gelu(a3 W1 + b1) W2 + b2
            fork()
            with torch.cuda.stream(side):
                ops.gemm(b["h"][l], dX, trans_a=True, out=G[f"{l}.w2"])
                ops.bias_bwd(dX, grads=(None, G[f"{l}.b2"]))
            ops.gemm(dX, P[f"{l}.w2"], trans_b=True, out=b["dh"], gelu_bwd_aux=b["u"][l])
            fork()
            with torch.cuda.stream(side):
                ops.gemm(b["a3"][l], b["dh"], trans_a=True, out=G[f"{l}.w1"])
                ops.bias_bwd(b["dh"], grads=(None, G[f"{l}.b1"]))
            ops.gemm(b["dh"], P[f"{l}.w1"], trans_b=True, out=b["da"])
            join()
            ops.layernorm_bwd(b["x2"][l], P[f"{l}.ln3g"], b["da"], grads=(dX, G[f"{l}.ln3g"], G[f"{l}.ln3b"]),
                              accumulate=True)
            # cross: x2 = x1 + (sigmoid(qc) * v0) Wco + bco, qc = a2 Wcq + bcq
            fork()
            with torch.cuda.stream(side):
                ops.gemm(b["cg"][l], dX, trans_a=True, out=G[f"{l}.wco"])
                ops.bias_bwd(dX, grads=(None, G[f"{l}.bco"]))
            ops.gemm(dX, P[f"{l}.wco"], trans_b=True, out=b["dz"])
            check(lib().dc_gate_bwd(b["qc"][l].data_ptr(), d, self._v0(l).data_ptr(), b["dz"].data_ptr(), d,
                                    b["da"].data_ptr(), d, G[f"{l}.bcv"].data_ptr(), B * T, d, st), "dc_gate_bwd")
            fork()
            with torch.cuda.stream(side):
                ops.gemm(b["a2"][l], b["da"], trans_a=True, out=G[f"{l}.wcq"])
                ops.bias_bwd(b["da"], grads=(None, G[f"{l}.bcq"]))
            ops.gemm(b["da"], P[f"{l}.wcq"], trans_b=True, out=b["dz"])
            join()
            ops.layernorm_bwd(b["x1"][l], P[f"{l}.ln2g"], b["dz"], grads=(dX, G[f"{l}.ln2g"], G[f"{l}.ln2b"]),
                              accumulate=True)
            # self: x1 = x + AFT(a1 Wqkv + bqkv) Wo + bo
            fork()
            with torch.cuda.stream(side):
                ops.gemm(b["z"][l], dX, trans_a=True, out=G[f"{l}.wo"])
                ops.bias_bwd(dX, grads=(None, G[f"{l}.bo"]))
            ops.gemm(dX, P[f"{l}.wo"], trans_b=True, out=b["dz"])
            self._aft(l, b["qkv"][l], None, B, T, backward=True, dz=b["dz"], dqkv=b["dqkv"])
            fork()
            with torch.cuda.stream(side):
                ops.gemm(b["a1"][l], b["dqkv"], trans_a=True, out=G[f"{l}.wqkv"])
                ops.bias_bwd(b["dqkv"], grads=(None, G[f"{l}.bqkv"]))
            ops.gemm(b["dqkv"], P[f"{l}.wqkv"], trans_b=True, out=b["da"])
            join()
            ops.layernorm_bwd(b["x"][l], P[f"{l}.ln1g"], b["da"], grads=(dX, G[f"{l}.ln1g"], G[f"{l}.ln1b"]),
                              accumulate=True)
            if bucket_done is not None:  # block l (and, for the last, the LM head) complete
                bucket_done(c.n_layers - 1 - l)
        check(lib().dc_embedding_bwd(b["idx"].data_ptr(), dX.data_ptr(), G["wte"].data_ptr(), G["wpe"].data_ptr(),
                                     B, T, d, V, st), "dc_embedding_bwd")
        if bucket_done is not None:
            bucket_done(c.n_layers)

    def optimizer_step(self, lr=3e-4, b1=0.9, b2=0.999, eps=1e-8, weight_decay=0.001):
        """AdamW over every parameter in one launch, with the reference's step
        count convention (Adam.step increments t before adam_step,
        lib/core/optimizers/adam.dart:603-637)."""
        self.t += 1
        ops.adam_step(self.flat, self.grad, self.adam_m, self.adam_v, self.t, lr, b1, b2, eps, weight_decay)

    def train_step(self, idx, targets, lr=3e-4, process_group=None, overlap=True):
        """One data-parallel step: the loss is the mean over this rank's B*T
        tokens; with a process group the gradients are averaged over ranks.
        overlap=True all-reduces them bucket by bucket (grad_buckets()) on a
        comm stream while the rest of the backward runs; otherwise with one
        all-reduce of the flat gradient buffer after it."""
        world = 1
        if process_group is not None:
            import torch.distributed as dist
            world = dist.get_world_size(process_group)
        _, loss = self.forward(idx, targets)
        if world > 1 and overlap:
            import torch.distributed as dist
            main = torch.cuda.current_stream()
            if getattr(self, "_comm_stream", None) is None:
                self._comm_stream = torch.cuda.Stream(self.device)
            comm = self._comm_stream
            buckets = self.grad_buckets()

            def done(k):
                a, b = buckets[k]
                ev = torch.cuda.Event()
                ev.record(main)
                comm.wait_event(ev)
                with torch.cuda.stream(comm):
                    dist.all_reduce(self.grad[a:b], group=process_group)

            self.backward(grad_scale=1.0 / world, bucket_done=done)
            main.wait_stream(comm)
        else:
            self.backward(grad_scale=1.0 / world)
            if world > 1:
                import torch.distributed as dist
                dist.all_reduce(self.grad, group=process_group)
        self.optimizer_step(lr)
        return loss

    # ------------------------------------------------------------ decoding
    def _decode_state(self, B):
        if self._dec is not None and self._dec["B"] == B:
            return self._dec
        c, dev = self.cfg, self.device
        d, F, Tm = c.d_model, c.ffn_mult * c.d_model, c.block_size
        z = lambda *s: torch.zeros(*s, device=dev)
        s = {"B": B}
        s["cache"] = [z(Tm, B * d * 2) for _ in range(c.n_layers)]
        s["x"], s["a"], s["zd"], s["cg"] = (z(B, d) for _ in range(4))
        s["qkv"], s["h"] = z(B, 3 * d), z(B, F)
        s["logits"] = z(B, c.vocab)
        s["v0"] = [self.P[f"{l}.bcv"] for l in range(c.n_layers)]
        s["tokens"] = torch.zeros(B, Tm, dtype=torch.int32, device=dev)
        s["pos"] = torch.zeros(1, dtype=torch.int32, device=dev)
        nb = lib().dc_aft_decode_workspace_size(B, d, Tm)
        s["ws"] = torch.zeros(nb, dtype=torch.uint8, device=dev)  # counters start at zero
        s["ws_bytes"] = nb
        self._dec = s
        return s

    def prefill(self, prompt: torch.Tensor):
        """Run the prompt [B, T0] (int32) through the batched forward, keep
        every layer's k/v history and pick the first new token (greedy)."""
        c, P = self.cfg, self.P
        B, T0 = prompt.shape
        s = self._decode_state(B)
        d, V, Tm = c.d_model, c.vocab, c.block_size
        st = ops._stream()
        self.forward(prompt, lm_head=False)
        b = self._bufs
        for l in range(c.n_layers):
            check(lib().dc_kv_cache_fill(b["qkv"][l].data_ptr(), 3 * d, B, T0, d, s["cache"][l].data_ptr(), st),
                  "dc_kv_cache_fill")
        # LM head on the last position only: rows b*T0 + T0-1 of the final LN
        last = b["af"].view(B, T0, d)[:, T0 - 1, :]
        ops.gemm(last, P["wlm"][:, :V], out=s["logits"], bias=P["blm"])
        check(lib().dc_copy2d(s["tokens"].data_ptr(), Tm * 4, prompt.data_ptr(), T0 * 4, T0 * 4, B, st), "dc_copy2d")
        s["pos"].fill_(T0 - 1)
        self._greedy(s)

    def _greedy(self, s):
        c, P = self.cfg, self.P
        check(lib().dc_greedy_embed(s["logits"].data_ptr(), c.vocab, s["B"], c.vocab, P["wte"].data_ptr(),
                                    P["wpe"].data_ptr(), s["pos"].data_ptr(), c.d_model, s["tokens"].data_ptr(),
                                    c.block_size, s["x"].data_ptr(), ops._stream()), "dc_greedy_embed")

    def decode_step(self):
        """Consume the token at position t = pos (its embedding is in s['x']),
        append its k/v to every layer's history, emit the token of t+1."""
        c, P = self.cfg, self.P
        s = self._dec
        B = s["B"]
        d, hs, Tm = c.d_model, c.head, c.block_size
        st = ops._stream()
        x = s["x"]
        for l in range(c.n_layers):
            ops.layernorm_fwd(x, P[f"{l}.ln1g"], P[f"{l}.ln1b"], out=s["a"])
            ops.gemm(s["a"], P[f"{l}.wqkv"], out=s["qkv"], bias=P[f"{l}.bqkv"])
            check(lib().dc_aft_decode(s["qkv"].data_ptr(), 3 * d, P[f"{l}.pos"].data_ptr(), Tm, Tm * Tm,
                                      s["cache"][l].data_ptr(), B, c.n_heads, hs, s["pos"].data_ptr(), Tm,
                                      s["zd"].data_ptr(), d, s["ws"].data_ptr(), s["ws_bytes"], st), "dc_aft_decode")
            # residual adds in place on x (the step keeps no activations), so a
            # split-K GEMM starts from x itself rather than from a copy
            ops.gemm(s["zd"], P[f"{l}.wo"], out=x, bias=P[f"{l}.bo"], residual=x)
            # cross-attention against the one encoder row, sigmoid(q) * v0, in
            # the query projection's epilogue
            ops.layernorm_fwd(x, P[f"{l}.ln2g"], P[f"{l}.ln2b"], out=s["a"])
            ops.gemm(s["a"], P[f"{l}.wcq"], out=s["cg"], bias=P[f"{l}.bcq"], gate=s["v0"][l])
            ops.gemm(s["cg"], P[f"{l}.wco"], out=x, bias=P[f"{l}.bco"], residual=x)
            ops.layernorm_fwd(x, P[f"{l}.ln3g"], P[f"{l}.ln3b"], out=s["a"])
            ops.gemm(s["a"], P[f"{l}.w1"], out=s["h"], bias=P[f"{l}.b1"], gelu=True)
            ops.gemm(s["h"], P[f"{l}.w2"], out=x, bias=P[f"{l}.b2"], residual=x)
        ops.layernorm_fwd(x, P["lnfg"], P["lnfb"], out=s["a"])
        ops.gemm(s["a"], P["wlm"][:, : c.vocab], out=s["logits"], bias=P["blm"])
        self._greedy(s)

    def generate(self, prompt: torch.Tensor, n_new: int, graph: bool = True):
        """Greedy continuation of prompt [B, T0]: tokens [B, T0 + n_new].
        With ``graph`` the decode step is captured once as a CUDA graph and
        replayed (the position advances on the device)."""
        B, T0 = prompt.shape
        if T0 + n_new > self.cfg.block_size:
            raise ValueError("prompt + new tokens exceed the block size")
        self.prefill(prompt)
        steps = n_new - 1
        if steps > 0:
            self.decode_step()  # eager first step: one-time library setup happens here
            if graph and steps > 1:
                g = self.capture_decode_step()
                for _ in range(steps - 1):
                    g.replay()
            else:
                for _ in range(steps - 1):
                    self.decode_step()
        return self._dec["tokens"][:, : T0 + n_new]

    def capture_decode_step(self):
        """A CUDA graph of one decode step.  Capturing does not run it; each
        replay decodes the position held in device memory and advances it."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.decode_step()
        return g
