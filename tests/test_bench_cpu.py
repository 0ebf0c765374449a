"""bench.py's host-side contract on CPU: every warm-up and timed step gets fresh prompt token ids
with the same lengths (no step can hit another step's prefix cache), and the reference arm's
unavailable paths print one JSON line and exit 0."""
import json
import os
import subprocess
import sys

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_steps_share_lengths_but_not_token_ids():
    seeds = [bench.step_seed("warmup", i) for i in range(3)] + [bench.step_seed("timed", i) for i in range(5)]
    assert len(set(seeds)) == len(seeds)
    runs = [bench.workload(64, 151936, token_seed=s) for s in seeds]
    for prompts, outs in runs:
        assert [len(p) for p in prompts] == [len(p) for p in runs[0][0]] and outs == runs[0][1]
        assert all(100 <= len(p) <= 1024 for p in prompts) and all(100 <= o <= 1024 for o in outs)
    firsts = {tuple(r[0][0][:16]) for r in runs}
    assert len(firsts) == len(runs)  # every step's first prompt differs
    assert bench.workload(8, 1000, token_seed=7) == bench.workload(8, 1000, token_seed=7)


def test_reference_arm_unavailable_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--kv", "fp8", "--steps", "1",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unavailable"]


def test_reference_arm_without_a_gpu_prints_unavailable():
    import torch
    if torch.cuda.is_available():
        return
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                         cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    assert json.loads(out.stdout.strip().splitlines()[-1])["impl"] == "reference"
