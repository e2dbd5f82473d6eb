"""bench.py's reference arm on the CPU (the oracle port on the host cores):
one JSON line with the contract's keys, timing only what it reports (steps x
ms_per_step is the arm's timed wall time), and rank 0 alone printing under
torchrun.  The small fp32 workload keeps it to about a second."""
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(args, env=None):
    t0 = time.perf_counter()
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                       timeout=300, env={**os.environ, **(env or {})}, cwd=str(ROOT))
    return r, time.perf_counter() - t0


def test_reference_arm_line():
    r, wall = _run(["--impl", "reference", "--config", "c1", "--steps", "3", "--warmup", "1", "--cpu-budget", "0.5"])
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "dtype", "config", "cpu_baseline", "e2e", "impl"):
        assert k in d, k
    assert d["impl"] == "reference" and d["steps"] == 3 and d["warmup"] == 1
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    # the timed steps fit inside the process's own wall time
    assert d["steps"] * d["ms_per_step"] / 1e3 <= wall


def test_reference_arm_other_ranks_silent():
    r, _ = _run(["--impl", "reference", "--config", "c1", "--steps", "1", "--warmup", "0"],
                env={"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


def test_decoder_reference_arm_unavailable():
    r, _ = _run(["--impl", "reference", "--config", "c3"])
    assert r.returncode == 0, r.stderr
    d = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert d["impl"] == "reference" and "unavailable" in d
