"""Data-parallel decoder step with two ranks (gloo, both on GPU 0; no kernel
waits on another rank): averaged gradients equal the single-process
gradient over the whole batch and the ranks stay in lockstep."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(0)
        from dart_cuda_b200 import decoder

        cfg = decoder.DecoderConfig(vocab=11, d_model=32, n_layers=2, n_heads=2, block_size=16)
        g = torch.Generator().manual_seed(21)
        idx = torch.randint(0, cfg.vocab, (4, 16), generator=g, dtype=torch.int32).cuda()
        tgt = torch.randint(0, cfg.vocab, (4, 16), generator=g, dtype=torch.int32).cuda()
        shard = slice(2 * rank, 2 * rank + 2)
        m = decoder.AftDecoder(cfg, seed=5, std=0.2)
        m.forward(idx[shard].contiguous(), tgt[shard].contiguous())
        # the gradients reduced bucket by bucket at the points the backward
        # reports them complete (on the caller's stream, so each reduction
        # sees exactly the work queued before it): a bucket reported too early
        # would reduce partial gradients and miss the single-process result
        buckets = m.grad_buckets()
        seen = []

        def done(k):
            seen.append(k)
            a, b = buckets[k]
            dist.all_reduce(m.grad[a:b])

        m.backward(grad_scale=1.0 / world, bucket_done=done)
        assert seen == list(range(len(buckets))), seen
        m.optimizer_step(lr=1e-2)
        flat = [torch.empty_like(m.flat) for _ in range(world)]
        dist.all_gather(flat, m.flat)
        if rank == 0:
            assert all(torch.equal(flat[0], f) for f in flat[1:]), "ranks diverged"
            ref = decoder.AftDecoder(cfg, seed=5, std=0.2)
            ref.forward(idx, tgt)
            ref.backward()
            err = float((m.grad - ref.grad).norm() / ref.grad.norm())
            assert err < 1e-4, err
            with open(os.path.join(out_dir, "ok"), "w") as f:
                f.write(str(err))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_step(tmp_path):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    mp.spawn(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert (tmp_path / "ok").exists()
