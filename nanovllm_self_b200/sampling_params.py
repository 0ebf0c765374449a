"""Per-request sampling parameters.

Same fields and defaults as the reference (``nanovllm/sampling_params.py:4-8``):
``temperature=0.7``, ``max_tokens=256``, ``ignore_eos=False``.  ``top_p`` (nucleus
sampling, 1.0 = off) and ``seed`` are additions that the fused sampler supports.
"""
from dataclasses import dataclass


@dataclass
class SamplingParams:
    temperature: float = 0.7
    max_tokens: int = 256
    ignore_eos: bool = False
    top_p: float = 1.0
    seed: int | None = None

    def __post_init__(self):
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if not (0.0 < self.top_p <= 1.0):
            raise ValueError("top_p must be in (0, 1]")
