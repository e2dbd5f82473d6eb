"""Time the reference engine's own GPU AFT kernels — TEST INFRASTRUCTURE.

Runs ``oracle/_ref/libmat_mul_ref.so`` (the reference's ``native/src/engine.cu``
built from its own sources by ``make -C oracle ref``) through its own C ABI,
exactly as its front end calls it: one ``aft_forward`` per sequence (the ABI
has no batch dimension) and ``backward`` from ``sum(Z * dZ)``.  The sample is
bounded: ``--nseq`` of the workload's sequences and ``--dsub`` of its channels
(channels are independent in the reference algorithm, so the rate scales to
the whole workload by d / dsub).  Device time per sequence is taken with CUDA
events around the forward + backward calls (the reference synchronises inside
some of them).  Needs a GPU:

    python oracle/time_ref_gpu.py --T 4096 --d 1024 --dsub 128 --nseq 2 --out ref_gpu.json
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import oracle  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--T", type=int, default=4096)
    ap.add_argument("--d", type=int, default=1024)
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--dsub", type=int, default=128)
    ap.add_argument("--nseq", type=int, default=2)
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--out", default="")
    a = ap.parse_args()
    import torch

    E = oracle.RefEngine()
    rng = np.random.default_rng(0)
    T, D = a.T, a.dsub
    W = (0.02 * rng.standard_normal((T, T))).astype(np.float32)
    seqs = [tuple(rng.standard_normal((T, D)).astype(np.float32) for _ in range(4)) for _ in range(a.nseq)]
    E.aft(*seqs[0][:3], W, seqs[0][3], True)  # warm-up (module load, first allocations)
    torch.cuda.synchronize()
    times = []
    for _ in range(a.reps):
        for Q, K, V, dZ in seqs:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            e0.record()
            E.aft(Q, K, V, W, dZ, True)
            e1.record()
            torch.cuda.synchronize()
            times.append((e0.elapsed_time(e1) / 1e3, time.perf_counter() - t0))
    dev_s = float(np.median([t[0] for t in times]))
    wall_s = float(np.median([t[1] for t in times]))
    rate = T * (D / a.d) / wall_s
    out = {"what": "reference engine's GPU aft_forward + backward (native/src/engine.cu), one call per "
                   "sequence, through its own C ABI; includes its host copies of the sample",
           "T": T, "d": a.d, "dsub": D, "nseq": a.nseq, "reps": a.reps,
           "seconds_per_sequence_sample": {"device_events": dev_s, "wall": wall_s},
           "tokens_per_s_whole_workload": rate,
           "tflops": 6.0 * D * T * (T + 1) / wall_s / 1e12,
           "gpu": torch.cuda.get_device_name(0)}
    print(json.dumps(out))
    if a.out:
        Path(a.out).write_text(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
