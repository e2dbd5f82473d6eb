"""Checkpoint interop with the reference's persistence format (flat fp32 in
parameters() order, lib/core/utils/persistence.dart:8-70).  Host-only: the
model's parameter storage is created on the CPU and no kernel runs."""
import numpy as np
import pytest
import torch

from dart_cuda_b200.decoder import AftDecoder, DecoderConfig


def make(seed=0, **kw):
    cfg = DecoderConfig(**{**dict(vocab=13, d_model=32, n_layers=2, n_heads=4, block_size=8), **kw})
    return AftDecoder(cfg, device="cpu", seed=seed)


def expected_count(c):
    d, H, hs, Tm, E, F, V = c.d_model, c.n_heads, c.head, c.block_size, c.enc, 4 * c.d_model, c.vocab
    head = 3 * (d * hs + hs) + Tm * Tm
    cross_head = (E * hs + hs) + (d * hs + hs) + (E * hs + hs) + Tm * Tm
    block = H * head + d * d + d + H * cross_head + d * d + d + d * F + F + F * d + d + 6 * d
    return V * d + Tm * d + c.n_layers * block + 2 * d + d * V + V


def test_parameter_order_and_shapes():
    m = make()
    c = m.cfg
    params = m.reference_parameters()
    names = [n for n, _ in params]
    hs = c.head
    # the first entries of the reference's TransformerDecoder.parameters()
    assert names[:2] == ["wte", "wpe"]
    assert names[2:9] == [f"blocks[0].self.heads[0].{x}" for x in ("q.w", "q.b", "k.w", "k.b", "v.w", "v.b", "posBias")]
    assert params[2][1].shape == (c.d_model, hs) and params[3][1].shape == (1, hs)
    assert params[8][1].shape == (c.block_size, c.block_size)
    # cross heads list key, query, value (AFTCrossAttention.parameters())
    k = names.index("blocks[0].cross.heads[0].k.w")
    assert names[k:k + 7] == [f"blocks[0].cross.heads[0].{x}" for x in ("k.w", "k.b", "q.w", "q.b", "v.w", "v.b", "posBias")]
    assert names[-4:] == ["finalLayerNorm.gamma", "finalLayerNorm.beta", "lmHead.w", "lmHead.b"]
    assert params[-2][1].shape == (c.d_model, c.vocab)
    assert sum(v.numel() for _, v in params) == expected_count(c)
    # views alias the kernels' fused storage: head 1's key weight is columns d+hs.. of wqkv
    v = dict(params)["blocks[1].self.heads[1].k.w"]
    assert torch.equal(v, m.P["1.wqkv"][:, c.d_model + hs: c.d_model + 2 * hs])


def test_save_load_round_trip(tmp_path):
    a, b = make(seed=1), make(seed=2)
    assert not torch.equal(a.flat, b.flat)
    f = tmp_path / "w.bin"
    a.save(f)
    assert f.stat().st_size == 4 * expected_count(a.cfg)
    data = np.fromfile(f, dtype="<f4")
    assert np.array_equal(data[: a.cfg.vocab * a.cfg.d_model], a.P["wte"].numpy().ravel())
    b.load(f)
    assert torch.equal(a.flat, b.flat)  # padding of the LM head stays zero on both


def test_load_rejects_wrong_size(tmp_path):
    a = make()
    f = tmp_path / "w.bin"
    np.zeros(10, dtype="<f4").tofile(f)
    with pytest.raises(ValueError, match="expects"):
        a.load(f)


def test_grad_buckets_cover_the_gradient_buffer():
    """The data-parallel reduction buckets are disjoint, contiguous and cover
    the whole flat gradient buffer, in the order the backward completes them
    (LM head with the last block first, embeddings last)."""
    m = make(n_layers=3)
    bk = m.grad_buckets()
    assert len(bk) == m.cfg.n_layers + 1
    assert bk[0][1] == m.numel and bk[-1][0] == 0
    for (a0, b0), (a1, b1) in zip(bk, bk[1:]):
        assert b1 == a0 and a1 < b1
    off = {n: o for n, (o, _) in m._offsets.items()}
    assert bk[0][0] == off["2.wqkv"] and bk[1] == (off["1.wqkv"], off["2.wqkv"])
    assert bk[-1] == (0, off["0.wqkv"])
