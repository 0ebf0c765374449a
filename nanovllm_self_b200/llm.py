"""Public API: ``LLM(model, ...).generate(prompts, SamplingParams)``.

``LLM`` and ``LLM_self`` are the same class here; the reference has ``LLM_self`` (its
own engine, ``nanovllm/llm.py:9-21``) and ``LLM`` (a plain HuggingFace ``generate``
wrapper used as a comparison, ``nanovllm/llm.py:3-7``).  The HF wrapper is kept as
:class:`HFLLM` for the same purpose.
"""
from __future__ import annotations

import torch

from .engine.llm_engine import LLMEngine
from .sampling_params import SamplingParams


class LLM(LLMEngine):
    def __init__(self, model: str | None = None, tensor_parallel_size: int = 1, enable_profile: bool = False,
                 **kwargs):
        # ``model`` may be a checkpoint directory or an architecture preset name.
        import os
        from .models.configs import PRESETS
        if model is not None and not os.path.isdir(model) and model.lower().replace("-random", "") in PRESETS:
            kwargs.setdefault("model", model.lower().replace("-random", ""))
            model_path = None
        else:
            model_path = model
        super().__init__(model_path=model_path, tensor_parallel_size=tensor_parallel_size,
                         enable_profile=enable_profile, **kwargs)


LLM_self = LLM


class HFLLM:
    """Naive HuggingFace ``generate`` loop (reference ``llm_engine``, ``llm_engine.py:27-96``)."""

    def __init__(self, model_path: str, device: str = "cuda", dtype=torch.bfloat16, eos_token_id: int | None = None):
        """``eos_token_id``: stop token (default: the directory's tokenizer's; -1 never stops, for
        checkpoints without a tokenizer)."""
        from transformers import AutoModelForCausalLM
        self.model = AutoModelForCausalLM.from_pretrained(model_path, dtype=dtype).to(device)
        self.device = device
        self.tokenizer = None
        if eos_token_id is None:
            from transformers import AutoTokenizer
            self.tokenizer = AutoTokenizer.from_pretrained(model_path)
            eos_token_id = self.tokenizer.eos_token_id
        self.eos_token_id = eos_token_id

    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_token: int = 20, temperature: float = 0.8):
        ids = input_ids.to(self.device)
        finished = torch.zeros(ids.shape[0], dtype=torch.bool, device=self.device)
        past = None
        for _ in range(max_token):
            if bool(finished.all()):
                break
            cur = ids if past is None else ids[:, -1:]
            out = self.model(cur, past_key_values=past, use_cache=True)
            past = out.past_key_values
            logits = out.logits[:, -1, :].float()
            if temperature > 0:
                nxt = torch.multinomial(torch.softmax(logits / temperature, -1), 1)
            else:
                nxt = logits.argmax(-1, keepdim=True)
            finished |= nxt.squeeze(-1) == self.eos_token_id
            nxt = torch.where(finished[:, None], torch.full_like(nxt, self.eos_token_id), nxt)
            ids = torch.cat([ids, nxt], 1)
        return ids


__all__ = ["LLM", "LLM_self", "HFLLM", "SamplingParams"]
