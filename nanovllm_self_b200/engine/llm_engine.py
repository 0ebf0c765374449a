"""Offline engine: ``generate`` loops schedule -> run -> postprocess until all requests finish.

Reference counterpart: ``llm_engine_self`` (``nanovllm/engine/llm_engine.py:98-320``).
Same public behaviour:

* ``generate(inputs, sampling_params=None, return_metrics=False, request_metadata=None)``
  accepts token-id sequences (lists or 1-D tensors) and, when a tokenizer is present,
  strings; returns ``[prompt + completion token ids]`` per input, or
  ``{"outputs": ..., "metrics": ...}`` with ``return_metrics=True``;
* ``request_metadata["session_id" | "program_id"]`` turns on the session prefix cache;
* ``metrics["throughput_tok_s"]`` = generated tokens / summed model-runner time.

Differences: per-engine config (no shared global), optional tokenizer (random-weight
models have none), device-side step timing with CUDA events (the reference uses
``synchronize`` + ``perf_counter``), TTFT/TPOT percentiles in the metrics, and the
step loop never busy-spins on an empty schedule (the reference loops forever when
``schedule()`` returns nothing, ``llm_engine.py:164-170``).
"""
from __future__ import annotations

import os
import time

import numpy as np
import torch

from ..config import EngineConfig
from ..models.loader import has_checkpoint
from ..parallel.state import init_tensor_parallel
from ..sampling_params import SamplingParams
from ..utils.tracing import StepTracer
from .model_runner import ModelRunner
from .scheduler import Scheduler
from .sequence import Sequence, SequenceStatus


def _percentile(xs, q):
    return float(np.percentile(np.asarray(xs, dtype=np.float64), q)) if len(xs) else 0.0


class LLMEngine:
    def __init__(self, model_path: str | None = None, tensor_parallel_size: int = 1, enable_profile: bool = False,
                 config: EngineConfig | None = None, **kwargs):
        if config is None:
            config = EngineConfig(model_path=model_path, tensor_parallel_size=tensor_parallel_size, **kwargs)
        else:
            config = config.replace(**kwargs) if kwargs else config
        self.config = config
        self.enable_profile = enable_profile
        self.tracer = StepTracer(enabled=enable_profile)
        self.tp = init_tensor_parallel(config.tensor_parallel_size, config.device, timeout_s=config.dist_timeout_s)
        self.comm = None
        if self.tp.size > 1:
            from ..parallel.comm import TPComm
            self.comm = TPComm(self.tp, backend=config.comm_backend, config=config)
        self.tokenizer = None
        if config.model_path and os.path.isdir(config.model_path):
            try:
                from transformers import AutoTokenizer
                self.tokenizer = AutoTokenizer.from_pretrained(config.model_path)
            except Exception:
                self.tokenizer = None
        self.model_runner = ModelRunner(config, self.tp, self.comm)
        self.block_manager = self.model_runner.block_manager
        self.scheduler = Scheduler(config, self.block_manager)
        arch = self.model_runner.arch
        if config.eos >= 0:
            self.eos_token_id = config.eos
        elif self.tokenizer is not None and self.tokenizer.eos_token_id is not None:
            self.eos_token_id = self.tokenizer.eos_token_id
        elif has_checkpoint(config.model_path):
            self.eos_token_id = arch.eos_token_id
        else:
            self.eos_token_id = -1
        self.scheduler.eos = self.eos_token_id
        self._next_seq_idx = 0
        self._dev_events = None

    # ----------------------------------------------------------------- text
    def encoder(self, text):
        if self.tokenizer is None:
            raise RuntimeError("this engine has no tokenizer (random-weight model)")
        return self.tokenizer(text)

    encode = encoder

    def decode(self, token_ids):
        if self.tokenizer is None:
            raise RuntimeError("this engine has no tokenizer (random-weight model)")
        return self.tokenizer.decode(token_ids, skip_special_tokens=True)

    def _to_ids(self, x):
        if isinstance(x, str):
            return self.encoder(x)["input_ids"]
        if isinstance(x, torch.Tensor):
            return x.reshape(-1).tolist()
        return list(x)

    # ------------------------------------------------------------- requests
    def add_request(self, prompt, sampling_params: SamplingParams | None = None, session_id=None) -> Sequence:
        ids = self._to_ids(prompt)
        sp = sampling_params or SamplingParams()
        if len(ids) + sp.max_tokens > self.config.max_model_len:
            raise ValueError(f"prompt ({len(ids)}) + max_tokens ({sp.max_tokens}) exceeds "
                             f"max_model_len={self.config.max_model_len}")
        seq = Sequence(self._next_seq_idx, ids, sp, self.config.block_size, session_id=session_id)
        self._next_seq_idx += 1
        self.scheduler.add(seq)
        return seq

    def step(self):
        """One schedule -> run -> postprocess iteration. Returns (scheduled, finished, dev_ms)."""
        tr = self.tracer
        with tr.phase("schedule"):
            seqs = self.scheduler.schedule()
        if not seqs:
            return [], [], 0.0
        # decode-only step (every sequence adds one token after its prefill): timed per batch size
        self.last_step_decode = all(s.num_new_tokens == 1 and s.is_prefill_done for s in seqs)
        with tr.phase("run"):
            token_ids, need = self.model_runner.run(seqs)
        dev_ms = self.model_runner.last_dev_ms
        tr.record_step(seqs, dev_ms)
        with tr.phase("postprocess"):
            finished = self.scheduler.postprocess(seqs, token_ids, need)
        return seqs, finished, dev_ms

    def is_finished(self) -> bool:
        return self.scheduler.is_finished()

    # -------------------------------------------------------------- generate
    def generate(self, inputs, sampling_params=None, return_metrics: bool = False,
                 request_metadata: dict | None = None, use_tqdm: bool = False):
        inputs = list(inputs)
        if sampling_params is None:
            sampling_params = [SamplingParams()] * len(inputs)
        elif isinstance(sampling_params, SamplingParams):
            sampling_params = [sampling_params] * len(inputs)
        if len(sampling_params) != len(inputs):
            raise ValueError("one SamplingParams per input")
        session_id = None
        if request_metadata is not None:
            session_id = request_metadata.get("session_id") or request_metadata.get("program_id")
        seqs = [self.add_request(x, sp, session_id) for x, sp in zip(inputs, sampling_params)]
        pbar = None
        if use_tqdm:
            from tqdm import tqdm
            pbar = tqdm(total=sum(s.max_tokens for s in seqs), desc="Generating", dynamic_ncols=True)
        dev_ms_total = 0.0
        steps = 0
        stalls = 0
        decode_steps = {}  # batch size -> [decode-only steps, their summed device ms]
        t_start = time.perf_counter()
        with torch.inference_mode():
            while not self.scheduler.is_finished():
                prev = sum(s.num_completion_tokens for s in seqs) if pbar else 0
                scheduled, _, dev_ms = self.step()
                if not scheduled:
                    stalls += 1
                    if stalls > 3:
                        raise RuntimeError(f"scheduler made no progress: {self.scheduler.last_schedule_info.reason}"
                                           f" (KV blocks free={self.block_manager.num_free_blocks()})")
                    continue
                stalls = 0
                dev_ms_total += dev_ms
                steps += 1
                if self.last_step_decode:
                    d = decode_steps.setdefault(len(scheduled), [0, 0.0])
                    d[0] += 1
                    d[1] += dev_ms
                if pbar:
                    pbar.update(sum(s.num_completion_tokens for s in seqs) - prev)
        wall = time.perf_counter() - t_start
        if pbar:
            pbar.close()
        if self.enable_profile:
            self.tracer.print_summary()
        outputs = [s.token_ids for s in seqs]
        if not return_metrics and not self.config.metrics_path:
            return outputs
        gen = sum(s.num_completion_tokens for s in seqs)
        total_s = dev_ms_total / 1e3 if self.model_runner.is_cuda else wall
        ttft = [(s.first_token_time - s.arrival_time) * 1e3 for s in seqs if s.first_token_time]
        tpot = [((s.finish_time - s.first_token_time) * 1e3 / (s.num_completion_tokens - 1))
                for s in seqs if s.finish_time and s.num_completion_tokens > 1]
        metrics = {
            "prefill_backend": self.model_runner.ops.name,
            "decode_backend": self.model_runner.ops.name,
            "num_seqs": len(seqs),
            "prompt_tokens": sum(s.num_prompt_tokens for s in seqs),
            "generated_tokens": gen,
            "total_time_s": total_s,
            "wall_time_s": wall,
            "schedule_steps": steps,
            "avg_step_ms": (total_s * 1e3 / steps) if steps else 0.0,
            "throughput_tok_s": gen / total_s if total_s > 0 else 0.0,
            "e2e_throughput_tok_s": gen / wall if wall > 0 else 0.0,
            "ttft_ms_p50": _percentile(ttft, 50), "ttft_ms_p99": _percentile(ttft, 99),
            "tpot_ms_p50": _percentile(tpot, 50), "tpot_ms_p99": _percentile(tpot, 99),
            "num_preemptions": self.scheduler.num_preemptions,
            # decode-only steps by batch size: {batch: [steps, mean device ms per step]}
            "decode_steps": {b: [n, ms / n] for b, (n, ms) in sorted(decode_steps.items())},
            "block_usage": self.block_manager.get_block_usage_snapshot(),
        }
        if self.enable_profile:
            metrics["profile"] = self.tracer.summary()
        if self.config.metrics_path and self.tp.rank == 0:
            import json
            row = {k: v for k, v in metrics.items() if k != "block_usage"}
            row["decode_steps"] = {str(b): v for b, v in row["decode_steps"].items()}
            with open(self.config.metrics_path, "a") as f:
                f.write(json.dumps(dict(row, time=time.time()), default=str) + "\n")
        if not return_metrics:
            return outputs
        return {"outputs": outputs, "metrics": metrics}

    def shutdown(self):
        self.model_runner.release_graphs()
        if self.comm is not None:
            self.comm.close()


# Name kept for users of the reference.
llm_engine_self = LLMEngine
