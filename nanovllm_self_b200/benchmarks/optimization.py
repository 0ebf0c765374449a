"""Engine-configuration search loop.

The reference's ``optimization/`` package is an empty scaffold (abstract
``OptimizationCandidate`` / ``BenchmarkRunner`` / ``TrafficGenerator`` /
``OptimizationLoop``; its CLI only exits, ``optimization/main.py:17-23``).  Here the same
four roles do work: candidates are engine-config overrides, the traffic generator is a
seeded workload, the runner measures device-timed tok/s, and the loop keeps the best.
"""
from __future__ import annotations

from dataclasses import dataclass, field

from .. import LLM, SamplingParams
from . import datasets


@dataclass
class OptimizationCandidate:
    name: str
    overrides: dict = field(default_factory=dict)


@dataclass
class TrafficGenerator:
    n: int = 32
    in_range: tuple = (100, 512)
    out_range: tuple = (32, 128)
    seed: int = 0

    def rows(self, vocab: int) -> list:
        return datasets.uniform_serving(self.n, vocab, self.in_range, self.out_range, self.seed)


@dataclass
class BenchmarkRunner:
    model: str = "tiny"
    base: dict = field(default_factory=dict)

    def run(self, cand: OptimizationCandidate, traffic: TrafficGenerator) -> dict:
        kw = dict(self.base)
        kw.update(cand.overrides)
        llm = LLM(self.model, **kw)
        rows = traffic.rows(llm.model_runner.arch.vocab_size)
        sps = [SamplingParams(temperature=0.0, max_tokens=r["max_tokens"], ignore_eos=True) for r in rows]
        llm.generate([r["prompt_ids"] for r in rows], sps)
        m = llm.generate([r["prompt_ids"] for r in rows], sps, return_metrics=True)["metrics"]
        llm.shutdown()
        return {"candidate": cand.name, "tok_s": m["throughput_tok_s"], "e2e_tok_s": m["e2e_throughput_tok_s"]}


@dataclass
class OptimizationLoop:
    runner: BenchmarkRunner
    traffic: TrafficGenerator
    candidates: list

    def run(self) -> dict:
        results = [self.runner.run(c, self.traffic) for c in self.candidates]
        best = max(results, key=lambda r: r["e2e_tok_s"])
        return {"best": best, "results": results}
