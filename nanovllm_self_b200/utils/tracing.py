"""Step tracing: NVTX ranges and per-phase timings of the serve loop.

The reference's profiling (``nanovllm/layers/attention.py:39-61``, ``llm_engine.py:193-222``)
synchronises the device around each attention sub-step and prints ``[PROFILE]`` lines.  Here
nothing synchronises: host phases are timed with ``perf_counter`` and the device part of each
step comes from the CUDA events the model runner already records.  With ``nvtx=True`` every
phase is also an NVTX range, so an external timeline profiler shows the same structure.
"""
from __future__ import annotations

import os
import time
from contextlib import contextmanager

import torch


class StepTracer:
    PHASES = ("schedule", "run", "postprocess")

    def __init__(self, enabled: bool = False, nvtx: bool | None = None):
        self.enabled = enabled
        if nvtx is None:
            nvtx = os.environ.get("NVB_NVTX", "0") not in ("", "0")
        self.nvtx = bool(nvtx) and torch.cuda.is_available()
        self.reset()

    def reset(self) -> None:
        self.host_s = {p: 0.0 for p in self.PHASES}
        self.device_ms = 0.0
        self.steps = 0
        self.prefill_steps = 0
        self.decode_steps = 0

    @contextmanager
    def phase(self, name: str):
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        t0 = time.perf_counter() if self.enabled else 0.0
        try:
            yield
        finally:
            if self.enabled:
                self.host_s[name] = self.host_s.get(name, 0.0) + time.perf_counter() - t0
            if self.nvtx:
                torch.cuda.nvtx.range_pop()

    def record_step(self, seqs, dev_ms: float) -> None:
        if not self.enabled:
            return
        self.steps += 1
        self.device_ms += dev_ms
        if seqs and all(s.num_new_tokens == 1 and s.is_prefill_done for s in seqs):
            self.decode_steps += 1
        else:
            self.prefill_steps += 1

    def summary(self) -> dict:
        return {"steps": self.steps, "prefill_steps": self.prefill_steps, "decode_steps": self.decode_steps,
                "device_ms": round(self.device_ms, 3),
                **{f"host_{k}_ms": round(v * 1e3, 3) for k, v in self.host_s.items()}}

    def print_summary(self) -> None:
        s = self.summary()
        print("[PROFILE] " + " ".join(f"{k}={v}" for k, v in s.items()), flush=True)
