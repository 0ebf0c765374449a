"""Qwen3 dense architecture descriptions and presets.

The reference supports exactly one model family, the Qwen3 dense decoder
(``nanovllm/models/qwen3.py``): GQA, per-head q/k RMSNorm, NeoX RoPE, SwiGLU MLP, an
optionally tied lm_head.  ``Qwen3Arch`` carries the HF ``config.json`` fields the model
needs; presets match the published Qwen3 shapes used by the benchmarks.
"""
from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, fields


@dataclass
class Qwen3Arch:
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = True
    bos_token_id: int = 151643
    eos_token_id: int = 151645
    name: str = "qwen3"

    @classmethod
    def from_hf_dict(cls, d: dict) -> "Qwen3Arch":
        kw = {f.name: d[f.name] for f in fields(cls) if f.name in d and d[f.name] is not None}
        if "head_dim" not in d or d.get("head_dim") is None:
            kw["head_dim"] = d["hidden_size"] // d["num_attention_heads"]
        if isinstance(kw.get("eos_token_id"), list):
            kw["eos_token_id"] = kw["eos_token_id"][0]
        return cls(**kw)

    @classmethod
    def from_pretrained(cls, path: str) -> "Qwen3Arch":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_hf_dict(json.load(f))

    def to_hf_dict(self) -> dict:
        d = asdict(self)
        d.pop("name")
        d.update({
            "architectures": ["Qwen3ForCausalLM"],
            "model_type": "qwen3",
            "hidden_act": "silu",
            "attention_bias": False,
            "attention_dropout": 0.0,
            "initializer_range": 0.02,
            "use_cache": True,
            "use_sliding_window": False,
            "sliding_window": None,
            "max_window_layers": self.num_hidden_layers,
            "torch_dtype": "bfloat16",
            "rope_scaling": None,
        })
        return d

    def num_params(self) -> int:
        h, i, d = self.hidden_size, self.intermediate_size, self.head_dim
        attn = h * d * (self.num_attention_heads * 2 + self.num_key_value_heads * 2)
        mlp = 3 * h * i
        per_layer = attn + mlp + 2 * h + 2 * d
        emb = self.vocab_size * h * (1 if self.tie_word_embeddings else 2)
        return self.num_hidden_layers * per_layer + emb + h


PRESETS = {
    # Config 1 of the benchmark plan: CPU fp32 oracle model.
    "tiny": Qwen3Arch(vocab_size=1024, hidden_size=128, intermediate_size=384, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=4096,
                      tie_word_embeddings=True, bos_token_id=1, eos_token_id=2, name="tiny"),
    # Qwen3-8B's head ratio (32 query / 8 KV heads, here 16 / 8) at tiny size: shards down to TP8, where
    # every rank keeps one KV head, as Qwen3-8B does at TP8.
    "tiny-tp8": Qwen3Arch(vocab_size=1024, hidden_size=128, intermediate_size=512, num_hidden_layers=2,
                          num_attention_heads=16, num_key_value_heads=8, head_dim=32, max_position_embeddings=4096,
                          tie_word_embeddings=False, bos_token_id=1, eos_token_id=2, name="tiny-tp8"),
    # Same topology as tiny but with head_dim 128 so the GPU kernels (head_dim 128 only) run it.
    "tiny-gpu": Qwen3Arch(vocab_size=2048, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                          num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=8192,
                          tie_word_embeddings=True, bos_token_id=1, eos_token_id=2, name="tiny-gpu"),
    "qwen3-0.6b": Qwen3Arch(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                            num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                            tie_word_embeddings=True, name="qwen3-0.6b"),
    "qwen3-8b": Qwen3Arch(vocab_size=151936, hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                          num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                          tie_word_embeddings=False, name="qwen3-8b"),
    "qwen3-32b": Qwen3Arch(vocab_size=151936, hidden_size=5120, intermediate_size=25600, num_hidden_layers=64,
                           num_attention_heads=64, num_key_value_heads=8, head_dim=128,
                           tie_word_embeddings=False, name="qwen3-32b"),
}


def resolve_arch(model=None, model_path: str | None = None) -> Qwen3Arch:
    """Architecture from (in order) an explicit preset/dict, or ``model_path/config.json``."""
    if isinstance(model, Qwen3Arch):
        return model
    if isinstance(model, dict):
        return Qwen3Arch.from_hf_dict(model)
    if isinstance(model, str):
        key = model.lower()
        if key in PRESETS:
            return PRESETS[key]
        raise ValueError(f"unknown model preset {model!r}; known: {sorted(PRESETS)}")
    if model_path is not None:
        if os.path.isfile(os.path.join(model_path, "config.json")):
            return Qwen3Arch.from_pretrained(model_path)
        key = os.path.basename(os.path.normpath(model_path)).lower().replace("-random", "")
        if key in PRESETS:
            return PRESETS[key]
    raise ValueError("no model architecture: pass model=<preset> or a model_path with config.json")
