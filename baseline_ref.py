"""Reference arm of bench.py: runs the unmodified reference engine (installed under
``baseline/_ref``) through its own public API on the same workload as ``bench.py``."""
from __future__ import annotations

import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def unavailable(reason: str) -> None:
    print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


def run_reference_arm(args, workload, ClockSampler, dist_info, reduce_max, metric, model_names):
    if not os.path.isdir(os.path.join(REF_DIR, "nanovllm")):
        unavailable("reference not installed under baseline/_ref")
        return
    unavailable("reference arm harness not wired yet")
