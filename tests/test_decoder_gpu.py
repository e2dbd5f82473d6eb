"""The decoder path: cached AFT decode against the oracle, the training step
against a float64 restatement, cached generation against full recompute."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from tests import decoder_ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mods():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dart_cuda_b200 import decoder, ops
    from dart_cuda_b200._lib import check, lib
    return decoder, ops, check, lib


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("B,H,hs,T,T0", [(3, 2, 16, 40, 0), (2, 4, 32, 70, 33), (64, 4, 128, 24, 8)])
def test_decode_matches_oracle(mods, B, H, hs, T, T0):
    """Positions T0..T-1 decoded one at a time (rows < T0 filled from a
    prefill projection) give the oracle's causal AFT rows."""
    _, ops, check, lib = mods
    D, Tmax = H * hs, T + 8
    rng = np.random.default_rng(B * 100 + T)
    Q, K, V = (rng.standard_normal((B, T, D)).astype(np.float32) for _ in range(3))
    W = (0.3 * rng.standard_normal((H, Tmax, Tmax))).astype(np.float32)
    ref = np.concatenate([oracle.aft_full_fwd(Q[..., h * hs:(h + 1) * hs], K[..., h * hs:(h + 1) * hs],
                                              V[..., h * hs:(h + 1) * hs],
                                              np.ascontiguousarray(W[h, :T, :T]), True) for h in range(H)], -1)
    qkv_all = torch.from_numpy(np.concatenate([Q, K, V], -1)).cuda()  # [B, T, 3D]
    w = torch.from_numpy(W).cuda()
    cache = torch.zeros(Tmax, B * D * 2, device="cuda")
    nb = lib().dc_aft_decode_workspace_size(B, D, Tmax)
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = ops._stream()
    if T0:
        pre = qkv_all[:, :T0].reshape(B * T0, 3 * D).contiguous()
        check(lib().dc_kv_cache_fill(pre.data_ptr(), 3 * D, B, T0, D, cache.data_ptr(), st), "fill")
    Z = torch.zeros(B, T, D, device="cuda")
    for t in range(T0, T):
        qkv = qkv_all[:, t].contiguous()
        pos.fill_(t)
        zt = torch.empty(B, D, device="cuda")
        check(lib().dc_aft_decode(qkv.data_ptr(), 3 * D, w.data_ptr(), Tmax, Tmax * Tmax, cache.data_ptr(), B, H,
                                  hs, pos.data_ptr(), Tmax, zt.data_ptr(), D, ws.data_ptr(), nb, st), "decode")
        Z[:, t] = zt
    torch.cuda.synchronize()
    got = Z[:, T0:].cpu().numpy()
    assert rel(got, ref[:, T0:]) < 1e-5
    assert np.abs(got - ref[:, T0:]).max() < 1e-4
    assert ops.device_status() == 0
    assert torch.count_nonzero(ws[:64]) == 0  # counters left at zero


def tiny_cfg(decoder, **kw):
    base = dict(vocab=11, d_model=32, n_layers=2, n_heads=2, block_size=16)
    base.update(kw)
    return decoder.DecoderConfig(**base)


def test_train_step_matches_float64(mods):
    decoder, ops, _, _ = mods
    cfg = tiny_cfg(decoder)
    m = decoder.AftDecoder(cfg, seed=3, std=0.2)
    # non-trivial biases / LN parameters so every gradient path is exercised
    g = torch.Generator().manual_seed(4)
    for name, v in m.P.items():
        base = name.split(".")[-1]
        if base.startswith("b") or base.startswith("ln"):
            v.add_(0.1 * torch.randn(v.shape, generator=g).cuda())
    B, T = 3, 16
    idx = torch.randint(0, cfg.vocab, (B, T), generator=g, dtype=torch.int32)
    tgt = torch.randint(0, cfg.vocab, (B, T), generator=g, dtype=torch.int32)
    logits, loss = m.forward(idx.cuda(), tgt.cuda())
    m.backward()
    torch.cuda.synchronize()
    P64 = {k: v.detach().double().cpu().requires_grad_(True) for k, v in m.P.items()}
    ref_logits, ref_loss = decoder_ref.forward(P64, cfg, idx, tgt)
    ref_loss.backward()
    assert rel(logits.cpu().numpy(), ref_logits.detach().numpy()) < 5e-3
    ref_l = float(ref_loss.detach())
    assert abs(float(loss) - ref_l) / ref_l < 1e-3
    for k, v in P64.items():
        gref = v.grad.numpy() if v.grad is not None else np.zeros(v.shape)
        got = m.G[k].cpu().numpy()
        if np.linalg.norm(gref) < 1e-12:
            assert np.abs(got).max() < 1e-7, k
        else:
            assert rel(got, gref) < 1.5e-2, (k, rel(got, gref))
    assert ops.device_status() == 0


def test_concurrent_streams_match_serial(mods):
    """Heads on their own streams and the weight gradients beside the
    input-gradient chain give the gradients of the all-on-one-stream step, in
    a captured CUDA graph too (up to the order of split-K atomics)."""
    decoder, ops, _, _ = mods
    cfg = tiny_cfg(decoder, vocab=29, d_model=128, n_heads=4, block_size=64)
    m = decoder.AftDecoder(cfg, seed=7, std=0.1)
    g = torch.Generator().manual_seed(8)
    idx = torch.randint(0, cfg.vocab, (16, 64), generator=g, dtype=torch.int32).cuda()
    tgt = torch.randint(0, cfg.vocab, (16, 64), generator=g, dtype=torch.int32).cuda()

    def step():
        m.forward(idx, tgt)
        m.backward()

    def close(a, b):
        # per parameter, normwise.  Two all-on-one-stream steps already differ
        # by up to 5e-4 here (split-K atomics add in a different order every
        # run, and the differences travel down the input-gradient chain); a
        # stream race would hand a kernel a stale or half-written buffer.
        for k in m.G:
            off, shape = m._offsets[k]
            n = int(np.prod(shape))
            x, y = a[off:off + n].double(), b[off:off + n].double()
            assert float((x - y).norm()) <= 2e-3 * float(y.norm()) + 1e-9, k

    m.concurrent = False
    step()
    serial = m.grad.clone()
    m.concurrent = True
    step()
    torch.cuda.synchronize()
    close(m.grad, serial)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # warm the graph's allocations on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    m.grad.zero_()
    graph.replay()
    torch.cuda.synchronize()
    close(m.grad, serial)
    del graph
    assert ops.device_status() == 0


def test_loss_decreases(mods):
    decoder, _, _, _ = mods
    cfg = tiny_cfg(decoder, vocab=13, d_model=64, n_heads=4, block_size=32)
    m = decoder.AftDecoder(cfg, seed=5)
    g = torch.Generator().manual_seed(6)
    idx = torch.randint(0, cfg.vocab, (8, 32), generator=g, dtype=torch.int32).cuda()
    tgt = torch.roll(idx, -1, dims=1)  # learnable: predict the next token of a fixed batch
    losses = [float(m.train_step(idx, tgt, lr=3e-3)) for _ in range(30)]
    assert losses[-1] < 0.7 * losses[0], losses


@pytest.mark.parametrize("graph", [False, True])
def test_generate_matches_full_recompute(mods, graph):
    """Cached greedy decoding emits the tokens a full forward over the growing
    context picks, and its logits agree with that forward's last row."""
    decoder, ops, _, _ = mods
    cfg = tiny_cfg(decoder, vocab=17, d_model=64, n_heads=2, block_size=40, n_layers=3)
    m = decoder.AftDecoder(cfg, seed=7, std=0.3)
    g = torch.Generator().manual_seed(8)
    B, T0, n_new = 5, 12, 20
    prompt = torch.randint(0, cfg.vocab, (B, T0), generator=g, dtype=torch.int32).cuda()
    toks = m.generate(prompt, n_new, graph=graph).clone()
    torch.cuda.synchronize()
    assert torch.equal(toks[:, :T0], prompt)
    agree = 0
    for p in range(T0, T0 + n_new):
        logits, _ = m.forward(toks[:, :p].contiguous())
        last = logits.view(B, p, cfg.vocab)[:, p - 1]
        top2 = torch.topk(last, 2, dim=1).values
        sure = (top2[:, 0] - top2[:, 1]) > 1e-2
        pick = last.argmax(1).int()
        assert torch.equal(pick[sure], toks[sure, p])
        agree += int(sure.sum())
    assert agree >= B * n_new * 0.8
    assert ops.device_status() == 0


def test_decode_logits_match_forward(mods):
    decoder, ops, _, _ = mods
    cfg = tiny_cfg(decoder, vocab=19, d_model=64, n_heads=4, block_size=32)
    m = decoder.AftDecoder(cfg, seed=9, std=0.3)
    g = torch.Generator().manual_seed(10)
    B, T0 = 4, 9
    prompt = torch.randint(0, cfg.vocab, (B, T0), generator=g, dtype=torch.int32).cuda()
    m.prefill(prompt)
    for _ in range(6):
        m.decode_step()
        s = m._dec
        p = int(s["pos"])  # the step consumed position p-1 and emitted token p
        toks = s["tokens"][:, :p].contiguous()
        logits, _ = m.forward(toks)
        last = logits.view(B, p, cfg.vocab)[:, p - 1]
        assert rel(s["logits"].cpu().numpy(), last.cpu().numpy()) < 2e-3
