"""AFT-full fwd+bwd benchmark (tokens/s) on 1..N B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4|c2|c1|c3|c5]
                    [--scaling weak|strong]
    python bench.py --impl reference ...      # CPU oracle on the host cores

One step = forward + backward of the causal AFT-full operator over one batch
of synthetic sequences (seeded N(0,1) Q, K, V, dZ; w ~ N(0, 0.02)), the
backward reusing the forward's operand panels.  Default workload: the
long-context configuration B=8, T=4096, d=1024, bf16 tensors, fp32
accumulation (tensor-core bound); c2 is B=32, T=512, d=512 (HBM bound).
With N > 1 GPUs every rank runs its own batch shard (weak scaling: the
configuration's B per rank; strong: B split over the ranks) and the shared
bias gradient dW is summed across ranks with one NCCL all-reduce inside the
step.

`value`  : tokens/s of the whole job, inputs resident in HBM, device-timed
           with CUDA events, L2 flushed between steps (outside the events).
`e2e`    : the same through the C ABI with host (pinned) buffers: each step
           copies Q, K, V, dZ host->device and Z, dQ, dK, dV, dW back.
`roofline`: the dominant kernel's algorithmic FLOPs (or user-tensor bytes)
           per launch over its CUDA-event time against the measured peaks,
           and under `step` the whole step against t_roof = max(F / tensor
           peak, user bytes / HBM bandwidth).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # name: (B, T, d, dtype, description)
    "c1": (4, 64, 128, "f32", "AFT-full causal fwd+bwd fp32 B=4 T=64 d=128"),
    "c2": (32, 512, 512, "bf16", "AFT-full causal fwd+bwd bf16 B=32 T=512 d=512"),
    "c4": (8, 4096, 1024, "bf16", "AFT-full causal fwd+bwd bf16 B=8 T=4096 d=1024"),
}
METRIC = "AFT fwd+bwd tokens/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return dict(FALLBACK_PEAKS, bf16_tflops_sustained=1400.0, source="fallback")


def causal_flops(B, T, d):
    """Algorithmic tensor-core FLOPs of one fwd+bwd: three [num|den]-shaped
    contractions, each 2*B*d*T*(T+1) with the causal half skipped."""
    return 6.0 * B * d * T * (T + 1)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampled every 200 ms while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.rows.append([c.strip() for c in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------ CPU
class CpuSample:
    """The oracle port (fp32 C restatement of the reference loops, OpenMP over
    query rows) on the host cores, over a bounded sample of the workload.

    In the reference algorithm every channel d of every sequence is
    independent (only dW sums over them), so a sample of `dsub` channels of
    `nseq` sequences costs nseq/B * dsub/d of a full step; its rate in
    tokens/s is nseq * T * (dsub / d) / seconds."""

    def __init__(self, B, T, d, budget_s):
        import oracle

        self.oracle = oracle
        self.cores = os.cpu_count() or 1
        oracle.set_threads(self.cores)
        self.B, self.T, self.d = B, T, d
        rng = np.random.default_rng(0)
        self.W = (0.02 * rng.standard_normal((T, T))).astype(np.float32)
        self.rng = rng
        # size the sample from a probe of a few channels of one sequence
        dprobe = min(d, 8)
        t = self._run(1, dprobe)
        per_chan = t / dprobe  # seconds per channel of one sequence
        if per_chan * d <= budget_s:
            self.nseq, self.dsub = int(max(1, min(B, budget_s // (per_chan * d)))), d
        else:
            self.nseq, self.dsub = 1, int(max(1, min(d, budget_s // per_chan)))

    def _run(self, nseq, dsub):
        T = self.T
        Q, K, V, dZ = (self.rng.standard_normal((nseq, T, dsub)).astype(np.float32) for _ in range(4))
        t0 = time.perf_counter()
        self.oracle.aft_full_fwd(Q, K, V, self.W, True)
        self.oracle.aft_full_bwd(Q, K, V, self.W, dZ, True)
        return time.perf_counter() - t0

    def step(self):
        """One timed sample: (seconds, tokens/s of the whole workload's rate)."""
        t = self._run(self.nseq, self.dsub)
        return t, self.nseq * self.T * (self.dsub / self.d) / t

    def describe(self):
        return (f"{self.nseq} of {self.B} sequences x {self.dsub} of {self.d} channels (T={self.T}) "
                f"fwd+bwd per sample, fp32, {self.cores} threads; channels are independent in the "
                f"reference algorithm, so the rate scales to the whole workload by d/{self.dsub}")


def cpu_baseline(B, T, d, dtype_name, budget_s=10.0):
    """Returns (tokens/s, cores, sample description) of one bounded sample."""
    cs = CpuSample(B, T, d, budget_s)
    secs, rate = cs.step()
    return rate, cs.cores, cs.describe() + f", {secs:.2f} s"


# ------------------------------------------------------------------ host link
def _numa_of_gpu(torch, dev):
    try:
        bus = torch.cuda.get_device_properties(dev).pci_bus_id.lower()  # dddddddd:bb:dd.f
        dom, rest = bus.split(":", 1)
        for name in (bus, f"{int(dom, 16):04x}:{rest}"):  # sysfs uses a 4-digit domain
            f = Path(f"/sys/bus/pci/devices/{name}/numa_node")
            if f.exists():
                return int(f.read_text().strip())
        return -2
    except Exception:
        return -2


def _numa_of_cpus():
    """NUMA nodes of the CPUs this process may run on."""
    try:
        cpus = os.sched_getaffinity(0)
        nodes = set()
        for nd in Path("/sys/devices/system/node").glob("node[0-9]*"):
            for part in (nd / "cpulist").read_text().strip().split(","):
                lo, _, hi = part.partition("-")
                rng = range(int(lo), int(hi or lo) + 1)
                if any(c in cpus for c in rng):
                    nodes.add(int(nd.name[4:]))
        return sorted(nodes)
    except Exception:
        return []


def host_link(torch, dist, dev, bufset, host_inputs, h2d, d2h, e2e_step_ms, world, reps=3):
    """Achieved host<->device copy rates of this rank's step copies, each
    direction timed alone (pinned buffers, CUDA events on the copy stream),
    and where the GPU and this process's CPUs sit (NUMA nodes), gathered over
    the ranks: what bounds the end-to-end rate when every rank copies at once."""
    s = torch.cuda.Stream(device=dev)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    with torch.cuda.stream(s):
        e[0].record(s)
        for _ in range(reps):
            for dst, src in zip(bufset.inp, host_inputs):
                dst.copy_(src, non_blocking=True)
        e[1].record(s)
        for _ in range(reps):
            for dst, src in zip(bufset.host, bufset.out):
                dst.copy_(src, non_blocking=True)
        e[2].record(s)
    torch.cuda.synchronize()
    mine = [h2d * reps / (e[0].elapsed_time(e[1]) / 1e3) / 1e9, d2h * reps / (e[1].elapsed_time(e[2]) / 1e3) / 1e9,
            (h2d + d2h) / (e2e_step_ms / 1e3) / 1e9, float(_numa_of_gpu(torch, dev))]
    cpu_nodes = _numa_of_cpus()
    mine.append(float(cpu_nodes[0]) if len(cpu_nodes) == 1 else -1.0)
    t = torch.tensor(mine, device=dev, dtype=torch.float64)
    if dist is not None:
        allt = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allt, t)
    else:
        allt = [t]
    rows = [[float(x) for x in a.cpu()] for a in allt]
    return {"per_rank": [{"h2d_GB/s_alone": r[0], "d2h_GB/s_alone": r[1], "both_ways_GB/s_in_e2e": r[2],
                          "gpu_numa": int(r[3]), "cpu_numa": int(r[4])} for r in rows],
            "note": "alone: one direction of this rank's copies while the other ranks do the same; "
                    "in_e2e: the step's copy bytes over the e2e step time; cpu_numa -1: the process "
                    "may run on several NUMA nodes (pinned pages land where they are first touched)"}


# ------------------------------------------------------------------ row ops
def row_kernels(dev, P, reps=10):
    """HBM bandwidth of the training step's row kernels on tensors larger than
    L2 (no flush needed): LayerNorm and bias over [262144, 256] fp32 (the C3
    activation width), cross-entropy over [65536, 8192] fp32 logits (the C5
    vocabulary).  Bytes = one read of every input row and one write of every
    output row (parameter vectors are negligible)."""
    import torch
    from dart_cuda_b200 import ops

    torch.manual_seed(0)
    R, C = 262144, 256
    x = torch.randn(R, C, device=dev)
    dy = torch.randn(R, C, device=dev)
    gam, bet = torch.randn(C, device=dev), torch.randn(C, device=dev)
    y, dx = torch.empty_like(x), torch.empty_like(x)
    dg, db = torch.empty(C, device=dev), torch.empty(C, device=dev)
    T, V = 65536, 8192
    logits = torch.randn(T, V, device=dev)
    tgt = torch.randint(0, V, (T,), device=dev, dtype=torch.int32)
    g = torch.empty_like(logits)
    scale = torch.ones(1, device=dev)
    act = R * C * 4
    cases = {
        "layernorm_fwd": (lambda: ops.layernorm_fwd(x, gam, bet, out=y), 2 * act),
        "layernorm_bwd": (lambda: ops.layernorm_bwd(x, gam, dy, grads=(dx, dg, db)), 3 * act),
        "bias_fwd": (lambda: ops.bias_fwd(x, bet, out=y), 2 * act),
        "bias_bwd": (lambda: ops.bias_bwd(dy, grads=(dx, db)), 2 * act),
        "ce_fwd": (lambda: ops.ce_fwd(logits, tgt), T * V * 4),
        "ce_bwd": (lambda: ops.ce_bwd(logits, tgt, grad_scale=scale, out=g), 2 * T * V * 4),
    }
    out = {}
    stream = torch.cuda.current_stream()
    for name, (fn, nbytes) in cases.items():
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        gbs = nbytes / (ms / 1e3) / 1e9
        out[name] = {"us": ms * 1e3, "GB/s": gbs, "hbm_frac": gbs / P["hbm_gbs"], "bytes": nbytes}
    out["shapes"] = f"LN/bias [{R},{C}] fp32, CE [{T},{V}] fp32"
    return out


# ------------------------------------------------------------------ decoder
DECODER_CONFIGS = {
    # char-level decoder training step: vocab 65, 4 blocks, d_model 256, 4 heads, FFN 4x, T 256, B 64
    "c3": dict(vocab=65, d_model=256, n_layers=4, n_heads=4, block_size=256, B=64, T=256,
               desc="AFT decoder training step fp32 (tf32 tensor cores) vocab 65, 4 blocks, d_model 256, "
                    "4 heads, FFN 1024, T 256, B 64, CE eps 0.1, AdamW lr 3e-4",
               metric="decoder training step tokens/s"),
    # cached greedy decode: 6 blocks, d_model 512, vocab 8192, B 64, prompt 256, 256 new tokens
    "c5": dict(vocab=8192, d_model=512, n_layers=6, n_heads=4, block_size=512, B=64, T=256, new=256,
               desc="AFT decoder greedy decode fp32: 6 blocks, d_model 512, 4 heads, vocab 8192, B 64, "
                    "prompt 256 + 256 new tokens, k/v history cached",
               metric="decoder greedy decode tokens/s"),
}


def soak(step, barrier, seconds=0.5):
    """Untimed steps for `seconds` of wall time (in rounds of 20 steps; every
    rank runs the same number of rounds: rank 0 decides and broadcasts)."""
    import torch
    import torch.distributed as dist

    t0 = time.perf_counter()
    while True:
        for _ in range(20):
            step()
        barrier()
        go = torch.tensor([1 if time.perf_counter() - t0 < seconds else 0],
                          device=torch.cuda.current_device())
        if dist.is_available() and dist.is_initialized():
            dist.broadcast(go, 0)
        if not int(go):
            break


def _timed(torch, fn, steps, flush, stream):
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends))


def _max_over_ranks(torch, dist, dev, v):
    if dist is None:
        return v
    t = torch.tensor([v], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def _kernel_table(prof, steps, bytes_per=None, flops_per=None, P=None):
    out = {}
    total = max(sum(m for m, _ in prof.values()), 1e-9)
    for name, (ms, cnt) in prof.items():
        e = {"ms_per_step": ms / steps, "launches_per_step": cnt / steps, "share": ms / total}
        if bytes_per and name in bytes_per:
            e["GB/s"] = bytes_per[name] * steps / (ms / 1e3) / 1e9
            e["hbm_frac"] = e["GB/s"] / P["hbm_gbs"]
        if flops_per and name in flops_per:
            e["TFLOP/s"] = flops_per[name] * steps / (ms / 1e3) / 1e12
            e["tensor_frac"] = e["TFLOP/s"] / P["bf16_tflops"]
        out[name] = e
    return out


def bench_train(args, dev, rank, world, dist):
    """C3: one data-parallel training step of the AFT decoder per bench step
    (forward, backward, gradient all-reduce for N > 1, AdamW)."""
    import torch
    from dart_cuda_b200 import decoder, ops

    c = DECODER_CONFIGS["c3"]
    cfg = decoder.DecoderConfig(vocab=c["vocab"], d_model=c["d_model"], n_layers=c["n_layers"],
                                n_heads=c["n_heads"], block_size=c["block_size"])
    B, T = c["B"], c["T"]
    m = decoder.AftDecoder(cfg, device=dev, seed=0)  # the same initial weights on every rank
    g = torch.Generator(device=dev)
    g.manual_seed(2000 + rank)
    idx = torch.randint(0, cfg.vocab, (B, T), device=dev, generator=g, dtype=torch.int32)
    tgt = torch.randint(0, cfg.vocab, (B, T), device=dev, generator=g, dtype=torch.int32)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)
    stream = torch.cuda.current_stream()
    graphs = None
    # N > 1: the gradient all-reduce in buckets (the LM head with the last
    # block, then one per block, then the embeddings), each started on a comm
    # stream as soon as the backward has completed it, so the reductions
    # overlap the rest of the backward; the CUDA graph of forward + backward
    # is captured as one graph per bucket, replayed with the bucket's
    # all-reduce queued between replays
    # (opt-in: measured slower than one all-reduce after the backward at 2
    # and 8 GPUs, 3.05 / 3.17 against 3.00 / 3.09 ms — the NCCL kernels beside
    # the backward cost more than the 25.6 MB all-reduce they hide)
    overlap = dist is not None and args.c3_overlap
    buckets = m.grad_buckets()
    comm = torch.cuda.Stream(device=dev) if overlap else None

    def reduce_bucket(k):
        a, b = buckets[k]
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream())
        comm.wait_event(ev)
        with torch.cuda.stream(comm):
            dist.all_reduce(m.grad[a:b])

    def fwd_bwd(bucket_done=None):
        m.forward(idx, tgt)
        m.backward(grad_scale=1.0 / world, bucket_done=bucket_done)

    def step():
        if graphs is not None:
            for k, gr in enumerate(graphs):
                gr.replay()
                if overlap:
                    reduce_bucket(k)
        else:
            fwd_bwd(reduce_bucket if overlap else None)
        if overlap:
            torch.cuda.current_stream().wait_stream(comm)
        elif dist is not None:
            dist.all_reduce(m.grad)
        m.optimizer_step(lr=3e-4)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    if not args.no_graph:
        # forward + backward as CUDA graphs (AdamW stays eager: its step count
        # moves); with the overlapped all-reduce, one graph per bucket
        pool = torch.cuda.graph_pool_handle()
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(torch.cuda.current_stream())
        n = len(buckets) if overlap else 1
        segs = [torch.cuda.CUDAGraph() for _ in range(n)]
        with torch.cuda.stream(cap):
            segs[0].capture_begin(pool=pool)

            def boundary(k):
                if k + 1 < n:
                    segs[k].capture_end()
                    segs[k + 1].capture_begin(pool=pool)

            fwd_bwd(boundary if overlap else None)
            segs[-1].capture_end()
        torch.cuda.current_stream().wait_stream(cap)
        graphs = segs
        step()
        barrier()
    sampler = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    with sampler:
        soak(step, barrier)
        barrier()
        total_ms = _timed(torch, step, args.steps, flush, stream)
        barrier()
    total_ms = _max_over_ranks(torch, dist, dev, total_ms)
    ms = total_ms / args.steps
    value = B * T * world / (ms / 1e3)

    # per-kernel pass (eager, events around every library launch; all on one
    # stream so that no kernel's events also span another stream's work)
    ops.profile_enable(True)
    m.concurrent = False
    for _ in range(args.steps):
        flush.zero_()
        fwd_bwd()
        if dist is not None:
            dist.all_reduce(m.grad)
        m.optimizer_step(lr=3e-4)
    torch.cuda.synchronize()
    m.concurrent = True
    prof = ops.profile_read()
    ops.profile_enable(False)
    d, F, V, M, L = cfg.d_model, 4 * cfg.d_model, cfg.vocab, B * T, cfg.n_layers
    fwd_gemm = L * 2 * M * d * (3 * d + d + d + d + 2 * F) + 2 * M * d * V
    gemm_flops = 3 * fwd_gemm  # forward, input gradients, weight gradients
    aft_flops = L * cfg.n_heads * 3 * 2 * B * cfg.head * T * (T + 1)
    P = peaks()
    kern = _kernel_table(prof, args.steps, flops_per={"gemm_tc": gemm_flops}, P=P)
    dom = max(prof, key=lambda k: prof[k][0]) if prof else None
    roof = None
    if dom == "gemm_tc":
        # the decoder's GEMMs run tf32 operands: their ceiling is the dense
        # tf32 rate, half the bf16 rate on this part (1.1 against 2.25
        # PFLOP/s nominal), taken as half the measured bf16 burst peak
        k = kern[dom]
        tf32 = P["bf16_tflops"] / 2
        roof = {"bound": "tensor", "achieved": k["TFLOP/s"], "peak": tf32, "unit": "TFLOP/s",
                "frac": k["TFLOP/s"] / tf32, "traffic": None, "kernel": dom,
                "peak_source": P["source"] + " bf16 burst / 2 (tf32 operands)"}
        kern[dom]["tensor_frac"] = k["TFLOP/s"] / tf32

    # end to end: token ids and targets from pinned host memory, the loss back
    h_idx, h_tgt = idx.cpu().pin_memory(), tgt.cpu().pin_memory()
    h_loss = torch.empty(1).pin_memory()

    def e2e_step():
        idx.copy_(h_idx, non_blocking=True)
        tgt.copy_(h_tgt, non_blocking=True)
        step()
        h_loss.copy_(m._bufs["loss"], non_blocking=True)

    e2e_ms = _max_over_ranks(torch, dist, dev, _timed(torch, e2e_step, args.steps, flush, stream))
    line = {
        "metric": c["metric"], "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": c["desc"], "B_per_gpu": B, "seq_len": T, "global_batch": B * world,
                   "parallelism": f"dp{world}", "l2": "flushed between steps (256 MiB write)",
                   "cuda_graph": not args.no_graph,
                   "grad_allreduce": ("none" if dist is None else
                                      f"{len(buckets)} buckets overlapped with the backward" if overlap
                                      else "one all-reduce after the backward")},
        "tflops": (gemm_flops + aft_flops) * world / (ms / 1e3) / 1e12,
        "e2e": {"value": B * T * world / (e2e_ms / args.steps / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * B * T * 4, "d2h_bytes_per_step": 4},
        "roofline": roof, "kernels": kern,
        "gpu_launches": sum(cnt for _, cnt in prof.values()),
        "clocks": sampler.summary(),
        "cpu_baseline": None,
    }
    return line


def bench_decode(args, dev, rank, world, dist):
    """C5: one bench step = prefill of the prompt plus new-1 cached decode
    steps (each a CUDA-graph replay) for B sequences per GPU; N GPUs run
    independent replicas."""
    import torch
    from dart_cuda_b200 import decoder, ops

    c = DECODER_CONFIGS["c5"]
    cfg = decoder.DecoderConfig(vocab=c["vocab"], d_model=c["d_model"], n_layers=c["n_layers"],
                                n_heads=c["n_heads"], block_size=c["block_size"])
    B, T0, new = c["B"], c["T"], c["new"]
    m = decoder.AftDecoder(cfg, device=dev, seed=0)
    g = torch.Generator(device=dev)
    g.manual_seed(3000 + rank)
    prompt = torch.randint(0, cfg.vocab, (B, T0), device=dev, generator=g, dtype=torch.int32)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)
    stream = torch.cuda.current_stream()
    m.prefill(prompt)
    m.decode_step()
    torch.cuda.synchronize()
    pre_g, dec_g = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(pre_g):
        m.prefill(prompt)
    dec_g = m.capture_decode_step()

    def generation():
        pre_g.replay()
        for _ in range(new - 1):
            dec_g.replay()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        generation()
    barrier()
    steps = max(1, args.steps)
    sampler = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    with sampler:
        barrier()
        total_ms = _timed(torch, generation, steps, flush, stream)
        barrier()
    total_ms = _max_over_ranks(torch, dist, dev, total_ms)
    ms = total_ms / steps
    value = B * new * world / (ms / 1e3)
    # decode-only rate: time the replays without the prefill
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pre_g.replay()
    e0.record(stream)
    for _ in range(new - 1):
        dec_g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    dec_ms = e0.elapsed_time(e1)

    # per-kernel pass: one eager generation
    ops.profile_enable(True)
    m.prefill(prompt)
    for _ in range(new - 1):
        m.decode_step()
    torch.cuda.synchronize()
    prof = ops.profile_read()
    ops.profile_enable(False)
    d, L, H = cfg.d_model, cfg.n_layers, cfg.n_heads
    # algorithmic bytes of the decode kernel over one generation: the k/v
    # history of positions <= t, the bias row, q|k|v in, Z out, per layer
    dec_bytes = sum(L * ((t + 1) * B * d * 8 + H * (t + 1) * 4 + B * 3 * d * 4 + B * d * 4)
                    for t in range(T0, T0 + new - 1))
    P = peaks()
    kern = _kernel_table(prof, 1, bytes_per={"aft_decode": dec_bytes}, P=P)
    roof = None
    if "aft_decode" in kern:
        k = kern["aft_decode"]
        algo = dec_bytes / max(prof["aft_decode"][1], 1)
        # measured DRAM traffic at one position, scaled to the mean launch by
        # the algorithmic bytes (both grow with the history length t)
        traffic = None
        tf = ROOT / "profiles" / "decoder_c5_traffic.json"
        if tf.exists():
            t = json.loads(tf.read_text())
            traffic = algo * t["dram_bytes_per_launch_at_t"] / t["algorithmic_bytes_per_launch_at_t"]
        roof = {"bound": "hbm", "achieved": k["GB/s"], "peak": P["hbm_gbs"], "unit": "GB/s",
                "frac": k["hbm_frac"], "traffic": traffic, "kernel": "aft_decode", "peak_source": P["source"],
                "algorithmic_bytes": algo}
        # the whole decode step: every weight the step's GEMMs read once (fp32;
        # the cross key/value weights are not read, the encoder row being
        # constant) plus the decode kernel's history and activations, per
        # generated token, against the step's measured time
        Fd = cfg.ffn_mult * d
        w_layer = (d * 3 * d + 3 * d) + (d * d + d) * 3 + (d * Fd + Fd) + (Fd * d + d) + 6 * d + d
        w_bytes = 4 * (L * w_layer + d * cfg.vocab + cfg.vocab + 2 * d)
        step_bytes = w_bytes + dec_bytes / (new - 1)
        step_ms = dec_ms / (new - 1)
        roof["step"] = {"bytes_per_token_step": step_bytes, "weights_bytes": w_bytes,
                        "history_bytes_mean": dec_bytes / (new - 1), "ms_per_token_step": step_ms,
                        "GB/s": step_bytes / (step_ms / 1e3) / 1e9,
                        "frac": step_bytes / (step_ms / 1e3) / 1e9 / P["hbm_gbs"],
                        "launches_per_token_step": sum(cnt for _, cnt in prof.values()) / max(new - 1, 1)}
    toks = m._dec["tokens"]
    h_prompt = prompt.cpu().pin_memory()
    h_toks = torch.empty(B, T0 + new, dtype=torch.int32).pin_memory()

    def e2e_gen():
        prompt.copy_(h_prompt, non_blocking=True)
        generation()
        h_toks.copy_(toks[:, : T0 + new], non_blocking=True)

    e2e_ms = _max_over_ranks(torch, dist, dev, _timed(torch, e2e_gen, steps, flush, stream))
    line = {
        "metric": c["metric"], "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": c["desc"], "B_per_gpu": B, "prompt": T0, "new_tokens": new,
                   "global_batch": B * world, "parallelism": f"replicas x{world}",
                   "l2": "flushed between generations (256 MiB write); the k/v history exceeds L2",
                   "cuda_graph": True},
        "decode_only_tokens_per_s": B * (new - 1) * world / (dec_ms / 1e3),
        "e2e": {"value": B * new * world / (e2e_ms / steps / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": B * T0 * 4, "d2h_bytes_per_step": B * (T0 + new) * 4},
        "roofline": roof, "kernels": kern,
        "gpu_launches": sum(cnt for _, cnt in prof.values()),
        "clocks": sampler.summary(),
        "cpu_baseline": None,
    }
    return line


def main_decoder(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    c = DECODER_CONFIGS[args.config]
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "metric": c["metric"],
                              "unavailable": "the reference has no host-side decoder path to time; its "
                                             "CPU restatement here covers the AFT operator and row ops only"}),
                  flush=True)
        return
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        line = (bench_train if args.config == "c3" else bench_decode)(args, dev, rank, world, dist)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c4", choices=sorted(CONFIGS) + sorted(DECODER_CONFIGS))
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="weak: every rank runs the configuration's B sequences; strong: the B "
                         "sequences are split over the ranks (B divisible by N)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of a CUDA graph")
    ap.add_argument("--backward", default="auto", choices=["auto", "stats", "recompute"],
                    help="stats: the forward keeps r, 1/den for the backward; recompute: the backward "
                         "repeats the forward contraction; auto: stats from T >= 256, where the "
                         "contraction costs more than the saved statistics' bytes")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-overlap", action="store_true",
                    help="N>1: all-reduce dW after the whole backward instead of beside dK/dV")
    ap.add_argument("--spare-sms", type=int, default=-1,
                    help="N>1: SMs the dK/dV kernel leaves free for the overlapped all-reduce "
                         "(default: 32 at N=2, 48 from N=4, where NCCL's all-reduce runs more CTAs; "
                         "measured at C2: N=8 6.6x with 16-32, 7.4x with 48)")
    ap.add_argument("--c3-overlap", action="store_true",
                    help="c3, N>1: all-reduce the gradients bucket by bucket beside the backward "
                         "(one CUDA graph per bucket) instead of once after it")
    ap.add_argument("--no-dw-pack", action="store_true",
                    help="N>1: all-reduce the full T x T dW instead of its block-packed causal part")
    ap.add_argument("--nccl-max-ctas", type=int, default=0,
                    help="N>1: cap NCCL's CTAs per collective (communicator config max_ctas); the "
                         "dK/dV kernel then leaves that many SMs free unless --spare-sms is given")
    ap.add_argument("--no-rows", action="store_true", help="skip the LayerNorm/bias/CE bandwidth pass")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the configuration's sequences per GPU (small profiling cases)")
    args = ap.parse_args()

    if args.config in DECODER_CONFIGS:
        return main_decoder(args)
    B, T, d, dt, desc = CONFIGS[args.config]
    if args.batch:
        B = args.batch
        desc = desc.replace(f"B={CONFIGS[args.config][0]}", f"B={B}")
    stats = args.backward == "stats" or (args.backward == "auto" and T >= 256)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.scaling == "strong":
        if B % world:
            raise SystemExit(f"--scaling strong needs B ({B}) divisible by the rank count ({world})")
        B //= world  # this rank's share of the configuration's sequences
    config = {"workload": desc, "B_per_gpu": B, "T": T, "d": d, "causal": True,
              "global_batch": B * world, "seq_len": T, "parallelism": f"batch-shard x{world}",
              "scaling": args.scaling,
              "l2": "flushed between steps (256 MiB write); inputs larger than L2 at T=4096",
              "cuda_graph": not args.no_graph,
              "backward": "reads the forward's r, 1/den" if stats else "recomputes num/den"}

    if args.impl == "reference":
        # The reference's CPU path (the oracle port) on the host cores: W
        # untimed and K timed steps, each one bounded sample of this
        # workload; ms_per_step is the measured time of a sample, so
        # steps x ms_per_step is the arm's own timed wall time.
        if rank != 0:
            return
        K = max(1, args.steps)
        W_ = max(0, args.warmup)
        per_step = max(0.2, min(args.cpu_budget, 100.0 / (K + W_)))
        cs = CpuSample(B * world, T, d, per_step)
        for _ in range(W_):
            cs.step()
        secs, rates = [], []
        for _ in range(K):
            t, r = cs.step()
            secs.append(t)
            rates.append(r)
        tok_s = len(secs) * cs.nseq * T * (cs.dsub / d) / sum(secs)
        line = {"metric": METRIC, "value": tok_s, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
                "steps": K, "warmup": W_, "higher_is_better": True, "scaling": config["scaling"],
                "dtype": "f32", "data": "synthetic", "config": config, "vs_baseline": None,
                "ms_per_step": 1e3 * sum(secs) / K,
                "step": "one bounded sample of the workload: " + cs.describe(),
                "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cs.cores, "kind": "port",
                                 "sample": cs.describe()},
                "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        opts = dist.ProcessGroupNCCL.Options()
        if args.nccl_max_ctas > 0:
            # cap the SMs NCCL's kernels take, so the dK/dV kernel running
            # beside the dW all-reduce can leave exactly that many free
            opts.config.max_ctas = args.nccl_max_ctas
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev, pg_options=opts)

    from dart_cuda_b200 import ops

    tdt = torch.bfloat16 if dt == "bf16" else torch.float32
    esz = 2 if dt == "bf16" else 4
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    Q, K_, V, dZ = (torch.randn(B, T, d, device=dev, generator=g).to(tdt) for _ in range(4))
    g0 = torch.Generator(device=dev)
    g0.manual_seed(999)  # w is shared: the same on every rank
    w = 0.02 * torch.randn(T, T, device=dev, generator=g0)
    Z = torch.empty_like(Q)
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K_), torch.empty_like(V)
    dW = torch.empty(T, T, device=dev)
    ws = ops.AftWorkspace(B, T, T, d, tdt, flags=1, device=dev, save_stats=stats)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)

    grads = (dQ, dK, dV, dW)
    overlap = dist is not None and not args.no_overlap
    # N > 1: dW in the block-packed causal layout for the all-reduce (the
    # upper triangle, zero on every rank, is not moved), expanded after it
    # (from T = 2048: below, the unpack costs more than the bytes it saves)
    pack = dist is not None and not args.no_dw_pack and T >= 2048
    dWp = torch.empty(ops.aft_dw_packed_size(T, T), device=dev) if pack else None
    red = dWp if pack else dW
    if args.spare_sms < 0:
        # measured: with the packed dW (T >= 2048) 32 free SMs beat 48 at 8
        # GPUs (C4: 7.38x against 7.21x one GPU) and 16 at 2 (1.072 against
        # 1.106 ms); the full 1 MiB dW of T = 512 ran best with 48 from N = 4
        if args.nccl_max_ctas > 0:
            args.spare_sms = args.nccl_max_ctas
        else:
            args.spare_sms = 32 if world <= 2 or T >= 2048 else 48
    config["dw_allreduce"] = ("none" if dist is None else ("serial" if not overlap
                              else f"beside dK/dV ({args.spare_sms} SMs left free)")
                              + (", block-packed causal dW (53% of T^2 at T=4096), expanded after"
                                 if pack else ", full T x T"))

    def compute():
        ops.aft_fwd(Q, K_, V, w, causal=True, out=Z, workspace=ws)
        ops.aft_bwd(Q, K_, V, w, dZ, causal=True, grads=(dQ, dK, dV, red), workspace=ws, ws_valid=True,
                    dw_packed=pack)

    # N > 1: forward, dQ and dW; then dW's all-reduce on a side stream while
    # the dK/dV contraction runs with a few SMs left to the collective
    def part_a():
        ops.aft_fwd(Q, K_, V, w, causal=True, out=Z, workspace=ws)
        ops.aft_bwd(Q, K_, V, w, dZ, causal=True, grads=(dQ, None, None, red), workspace=ws, ws_valid=True,
                    part="dw", dw_packed=pack)

    def part_b():
        ops.aft_bwd(Q, K_, V, w, dZ, causal=True, grads=grads, workspace=ws, ws_valid=True,
                    part="dkdv", spare_sms=args.spare_sms)

    graphs = None
    comm = torch.cuda.Stream(device=dev)
    dw_ready = torch.cuda.Event()

    def run(i, fn):
        if graphs is not None:
            graphs[i].replay()
        else:
            fn()

    def step():
        if not overlap:
            run(0, compute)
            if dist is not None:
                dist.all_reduce(red)
        else:
            run(0, part_a)
            dw_ready.record()
            with torch.cuda.stream(comm):
                comm.wait_event(dw_ready)
                dist.all_reduce(red)
            run(1, part_b)
            torch.cuda.current_stream().wait_stream(comm)
        if pack:
            ops.aft_dw_unpack(dWp, dW)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    if not args.no_graph:
        # the library's launches of one fwd+bwd replayed as CUDA graphs (two
        # when the all-reduce runs between them)
        parts = (part_a, part_b) if overlap else (compute,)
        captured = []
        for fn in parts:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                fn()
            captured.append(gr)
        graphs = captured
        for _ in range(2):
            step()
        barrier()
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(local)
    with sampler:
        # untimed steps for half a second first, so the 200 ms clock samples
        # see the GPU under this load when the timed region itself is short
        soak(step, barrier)
        barrier()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    if dist is not None:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t)
    ms_per_step = total_ms / args.steps
    value = B * T * world / (ms_per_step / 1e3)

    # ---- per-kernel timing pass (same steps, events around every launch)
    ops.profile_enable(True)  # eager launches: the events bracket each kernel
    saved, graphs = graphs, None
    for i in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    graphs = saved
    prof = ops.profile_read()
    ops.profile_enable(False)
    launches = sum(c for _, c in prof.values()) / args.steps

    # ---- end to end through the C ABI with pinned host buffers.  Every step
    # uploads its four inputs and reads back Z, dQ, dK, dV and dW; two device
    # buffer sets let step i's read-back (D2H stream) and step i+1's upload
    # (H2D stream) run on the two copy directions at once while the compute
    # stream runs the library calls in between.
    hQ, hK, hV, hdZ = (x.cpu().pin_memory() for x in (Q, K_, V, dZ))

    class BufSet:
        def __init__(self, dev_in, dev_out):
            self.inp, self.out = dev_in, dev_out
            self.host = [torch.empty(x.shape, dtype=x.dtype).pin_memory() for x in dev_out]
            self.in_ready, self.done, self.out_free = (torch.cuda.Event() for _ in range(3))

    sets = [BufSet((Q, K_, V, dZ), (Z, dQ, dK, dV, dW)),
            BufSet(tuple(torch.empty_like(x) for x in (Q, K_, V, dZ)),
                   tuple(torch.empty_like(x) for x in (Z, dQ, dK, dV, dW)))]
    for bs in sets:
        bs.done.record(stream)
        bs.out_free.record(stream)
    h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def e2e_step(i):
        bs = sets[i % 2]
        with torch.cuda.stream(h2d_s):
            h2d_s.wait_event(bs.done)  # the set's previous step no longer reads its inputs
            for dst, src in zip(bs.inp, (hQ, hK, hV, hdZ)):
                dst.copy_(src, non_blocking=True)
            bs.in_ready.record(h2d_s)
        stream.wait_event(bs.in_ready)
        stream.wait_event(bs.out_free)  # its previous outputs have been read back
        q, k, v, g = bs.inp
        ops.aft_fwd(q, k, v, w, causal=True, out=bs.out[0], workspace=ws)
        ops.aft_bwd(q, k, v, w, g, causal=True, grads=bs.out[1:4] + (red,), workspace=ws, ws_valid=True,
                    dw_packed=pack)
        if dist is not None:
            dist.all_reduce(red)
        if pack:
            ops.aft_dw_unpack(dWp, bs.out[4])
        bs.done.record(stream)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(bs.done)
            for dst, src in zip(bs.host, bs.out):
                dst.copy_(src, non_blocking=True)
            bs.out_free.record(d2h_s)

    def e2e_run(n):
        h2d_s.wait_stream(stream)
        d2h_s.wait_stream(stream)
        for i in range(n):
            e2e_step(i)
        stream.wait_stream(h2d_s)
        stream.wait_stream(d2h_s)

    e2e_run(2)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(args.steps)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t)
    e2e_val = B * T * world / (e2e_ms / args.steps / 1e3)
    h2d = 4 * B * T * d * esz
    d2h = 4 * B * T * d * esz + T * T * 4
    link = host_link(torch, dist, dev, sets[0], (hQ, hK, hV, hdZ), h2d, d2h, e2e_ms / args.steps, world)

    # ---- roofline.  Algorithmic work of one fwd+bwd step (per rank):
    # F = 6 B d T(T+1) tensor-core FLOPs (three causal [num|den]-shaped
    # contractions) and the user tensors' bytes: Q, K, V, dZ read and Z, dQ,
    # dK, dV written (esz each), w read and dW written (fp32).
    P = peaks()
    capped = "sw_power_cap" in sampler.summary()["reasons"]
    p_tc = P["bf16_tflops_sustained"] if capped else P["bf16_tflops"]
    io = B * T * d * esz            # one user tensor
    wbytes = T * T * 4
    step_flops = causal_flops(B, T, d)
    step_bytes = 8 * io + 2 * wbytes
    t_tc = step_flops / (p_tc * 1e12)
    t_tc_burst = step_flops / (P["bf16_tflops"] * 1e12)
    t_hbm = step_bytes / (P["hbm_gbs"] * 1e9)
    t_roof = max(t_tc, t_hbm)
    # per kernel: the user-tensor bytes each kernel must move (intermediate
    # panels are not credited) and the FLOPs of its contraction
    user_bytes = {
        "aft_prep": wbytes + 2 * io,          # w, K, V (one-launch prep)
        "aft_prep_w_colmax": wbytes + io,     # w, K
        "aft_prep_p": 2 * io,                 # K, V
        "aft_tc_fwd": 2 * io,                 # Q in, Z out
        "aft_tc_bwd_recompute": 3 * io,       # Q, dZ in, dQ out
        "aft_bwd_from_stats": 3 * io + wbytes,  # Q, dZ in, dQ out; clears dW
        "aft_tc_dkdv": 4 * io,                # K, V in, dK, dV out
        "aft_tc_dw": 2 * wbytes,              # w in, dW out
        "aft_dw_unpack": wbytes,              # dW out (N > 1)
    }
    gemm = 2.0 * B * d * T * (T + 1)  # one [num|den] contraction, causal half
    flops_per = {"aft_tc_fwd": gemm, "aft_tc_bwd_recompute": gemm, "aft_tc_dkdv": gemm, "aft_tc_dw": gemm}
    tot_ms = max(sum(m for m, _ in prof.values()), 1e-9)
    kern = {}
    for name, (ms, cnt) in prof.items():
        per_ms = ms / max(cnt, 1)
        gbs = user_bytes.get(name, 0) / (per_ms / 1e3) / 1e9
        tfs = flops_per.get(name, 0) / (per_ms / 1e3) / 1e12
        kern[name] = {"ms_per_launch": per_ms, "launches": cnt, "share": ms / tot_ms,
                      "user_GB/s": gbs, "TFLOP/s": tfs,
                      "hbm_frac": gbs / P["hbm_gbs"], "tensor_frac": tfs / p_tc}
    dom = max(prof, key=lambda k: prof[k][0]) if prof else None
    # measured DRAM traffic per launch (ncu summaries under profiles/)
    traffic = None
    traffic_step = None
    tf = ROOT / "profiles" / f"aft_{args.config}_traffic.json"
    if tf.exists():
        tj = json.loads(tf.read_text())
        per = tj["dram_bytes_per_launch"]
        if dom:
            traffic = per.get(dom)
        if tj.get("B") == B and all(k in per for k in prof):
            traffic_step = sum(per[k] * cnt for k, (_, cnt) in prof.items()) / max(args.steps, 1)
    roof = None
    if dom:
        k = kern[dom]
        step = {"t_roof_ms": t_roof * 1e3, "t_measured_ms": ms_per_step, "frac": t_roof * 1e3 / ms_per_step,
                "frac_vs_burst": max(t_tc_burst, t_hbm) * 1e3 / ms_per_step,
                "bound": "tensor" if t_tc >= t_hbm else "hbm",
                "flops": step_flops, "user_bytes": step_bytes,
                "t_tensor_ms": t_tc * 1e3, "t_hbm_ms": t_hbm * 1e3,
                "dram_traffic_bytes": traffic_step,
                "traffic_over_user_bytes": traffic_step / step_bytes if traffic_step else None}
        if dom in flops_per:
            roof = {"bound": "tensor", "achieved": k["TFLOP/s"], "peak": p_tc, "unit": "TFLOP/s",
                    "frac": k["TFLOP/s"] / p_tc, "traffic": traffic, "kernel": dom,
                    "algorithmic_flops_per_launch": flops_per[dom],
                    "peak_source": P["source"] + (" bf16 sustained (sw_power_cap seen)" if capped
                                                  else " bf16 burst")}
        else:
            roof = {"bound": "hbm", "achieved": k["user_GB/s"], "peak": P["hbm_gbs"], "unit": "GB/s",
                    "frac": k["hbm_frac"], "traffic": traffic, "kernel": dom, "peak_source": P["source"],
                    "algorithmic_bytes_per_launch": user_bytes.get(dom)}
        roof["step"] = step

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": dt, "data": "synthetic", "config": config,
        "tflops": causal_flops(B, T, d) * world / (ms_per_step / 1e3) / 1e12,
        "e2e": {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "copies": "pinned host buffers; uploads, library calls and read-backs on three "
                          "streams over two device buffer sets", "host_link": link},
        "roofline": roof, "kernels": kern, "gpu_launches": launches * args.steps,
        "clocks": sampler.summary(),
    }
    rg = ROOT / "profiles" / "reference_gpu_kernels.json"
    if rg.exists():
        # the reference's own GPU kernels on this workload (a committed,
        # separately measured bounded sample: profiles/reference_gpu_kernels.md)
        ref_gpu = json.loads(rg.read_text()).get(args.config)
        if ref_gpu:
            line["reference_gpu_kernels"] = {"value": ref_gpu["tokens_per_s"], "unit": "tokens/s",
                                             "sample": ref_gpu["sample"], "source": "profiles/reference_gpu_kernels.md"}
    if rank == 0 and world == 1 and not args.no_rows:
        line["row_kernels"] = row_kernels(dev, P)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tok_s, cores, sample = cpu_baseline(B, T, d, dt, budget_s=args.cpu_budget)
        line["cpu_baseline"] = {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": "port",
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del ws
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
