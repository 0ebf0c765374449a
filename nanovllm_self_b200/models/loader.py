"""Weight sources for :class:`Qwen3ForCausalLM`: HF safetensors (TP-sharded) or seeded random init.

* ``load_safetensors``: reads ``*.safetensors`` shards of an HF Qwen3 checkpoint with
  ``safe_open`` and slices each tensor for this TP rank while reading
  (``get_slice``), so no rank ever materialises the full model.  The reference instead
  instantiates the whole HF model in fp16 on every rank and then slices
  (``nanovllm/models/qwen3.py:291-428``).  Slicing rules match the reference: q/k/v and
  gate/up by output rows, o/down by input columns; embedding and lm_head are split by
  vocab rows here (vocab-parallel).
* ``random_init``: every tensor drawn from N(0, std) with a generator seeded from
  ``(seed, tensor name)`` on the target device; norm weights are 1.  The full tensor is
  drawn and then sliced, so the weights are the same at every TP degree.
* ``save_hf_checkpoint``: writes the same random weights as an HF directory
  (``config.json`` + safetensors) so another engine can load identical weights.
"""
from __future__ import annotations

import glob
import json
import os
import zlib

import torch

from .configs import Qwen3Arch
from ..ops.torch_ref import interleave_gate_up
from .qwen3 import Qwen3ForCausalLM

_HF = "model.layers.{i}."


def _seed_for(seed: int, name: str) -> int:
    return (seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFF


def _randn(name: str, shape, seed: int, std: float, device, dtype) -> torch.Tensor:
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(_seed_for(seed, name))
    t = torch.randn(*shape, generator=g, device=dev, dtype=torch.float32)
    return t.mul_(std).to(dtype)


def hf_tensor_shapes(arch: Qwen3Arch) -> dict:
    a = arch
    h, d, i = a.hidden_size, a.head_dim, a.intermediate_size
    shapes = {"model.embed_tokens.weight": (a.vocab_size, h), "model.norm.weight": (h,)}
    if not a.tie_word_embeddings:
        shapes["lm_head.weight"] = (a.vocab_size, h)
    for li in range(a.num_hidden_layers):
        p = _HF.format(i=li)
        shapes.update({
            p + "self_attn.q_proj.weight": (a.num_attention_heads * d, h),
            p + "self_attn.k_proj.weight": (a.num_key_value_heads * d, h),
            p + "self_attn.v_proj.weight": (a.num_key_value_heads * d, h),
            p + "self_attn.o_proj.weight": (h, a.num_attention_heads * d),
            p + "self_attn.q_norm.weight": (d,),
            p + "self_attn.k_norm.weight": (d,),
            p + "mlp.gate_proj.weight": (i, h),
            p + "mlp.up_proj.weight": (i, h),
            p + "mlp.down_proj.weight": (h, i),
            p + "input_layernorm.weight": (h,),
            p + "post_attention_layernorm.weight": (h,),
        })
    return shapes


class _RandomSource:
    """Serves full HF-named tensors drawn from the seeded generator."""

    def __init__(self, arch, seed, std, device):
        self.arch, self.seed, self.std, self.device = arch, seed, std, device
        self.shapes = hf_tensor_shapes(arch)

    def get(self, name, dtype, rows=None, cols=None):
        shape = self.shapes[name]
        if len(shape) == 1:
            t = torch.ones(shape, device=self.device, dtype=dtype)
        else:
            t = _randn(name, shape, self.seed, self.std, self.device, dtype)
        if rows is not None:
            t = t[rows[0]:rows[1]]
        if cols is not None:
            t = t[:, cols[0]:cols[1]]
        return t.contiguous()

    def has(self, name):
        return name in self.shapes


class _SafetensorsSource:
    def __init__(self, path, device):
        from safetensors import safe_open
        files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no *.safetensors under {path}")
        self.handles = [safe_open(f, framework="pt", device="cpu") for f in files]
        self.index = {}
        for h in self.handles:
            for k in h.keys():
                self.index[k] = h
        self.device = device

    def has(self, name):
        return name in self.index

    def get(self, name, dtype, rows=None, cols=None):
        sl = self.index[name].get_slice(name)
        shape = sl.get_shape()
        if len(shape) == 1:
            t = sl[:]
        else:
            r0, r1 = rows if rows is not None else (0, shape[0])
            c0, c1 = cols if cols is not None else (0, shape[1])
            t = sl[r0:r1, c0:c1]
        return t.to(device=self.device, dtype=dtype).contiguous()


def _fill(model: Qwen3ForCausalLM, src) -> Qwen3ForCausalLM:
    a, r, tp = model.arch, model.tp_rank, model.tp_size
    dt = model.dtype
    d = a.head_dim
    nq, nkv, ni = model.num_heads, model.num_kv_heads, model.intermediate
    vs, ve = model.vocab_start, model.vocab_end
    model.embed = src.get("model.embed_tokens.weight", dt, rows=(vs, ve))
    if a.tie_word_embeddings or not src.has("lm_head.weight"):
        model.lm_head = model.embed
    else:
        model.lm_head = src.get("lm_head.weight", dt, rows=(vs, ve))
    model.norm = src.get("model.norm.weight", dt)
    for li, L in enumerate(model.layers):
        p = _HF.format(i=li)
        q = src.get(p + "self_attn.q_proj.weight", dt, rows=(r * nq * d, (r + 1) * nq * d))
        k = src.get(p + "self_attn.k_proj.weight", dt, rows=(r * nkv * d, (r + 1) * nkv * d))
        v = src.get(p + "self_attn.v_proj.weight", dt, rows=(r * nkv * d, (r + 1) * nkv * d))
        L.qkv = torch.cat([q, k, v], 0).contiguous()
        del q, k, v
        L.o = src.get(p + "self_attn.o_proj.weight", dt, cols=(r * nq * d, (r + 1) * nq * d))
        L.q_norm = src.get(p + "self_attn.q_norm.weight", dt)
        L.k_norm = src.get(p + "self_attn.k_norm.weight", dt)
        g = src.get(p + "mlp.gate_proj.weight", dt, rows=(r * ni, (r + 1) * ni))
        u = src.get(p + "mlp.up_proj.weight", dt, rows=(r * ni, (r + 1) * ni))
        # gate/up rows interleaved in groups of 16: the GEMM applies SiLU-and-mul in its epilogue
        L.gate_up = interleave_gate_up(g, u).contiguous()
        del g, u
        L.down = src.get(p + "mlp.down_proj.weight", dt, cols=(r * ni, (r + 1) * ni))
        L.ln1 = src.get(p + "input_layernorm.weight", dt)
        L.ln2 = src.get(p + "post_attention_layernorm.weight", dt)
    return model


def random_init(model: Qwen3ForCausalLM, seed: int = 0, std: float = 0.02) -> Qwen3ForCausalLM:
    return _fill(model, _RandomSource(model.arch, seed, std, model.device))


def load_safetensors(model: Qwen3ForCausalLM, path: str) -> Qwen3ForCausalLM:
    return _fill(model, _SafetensorsSource(path, model.device))


def has_checkpoint(path: str | None) -> bool:
    return bool(path) and os.path.isdir(path) and bool(glob.glob(os.path.join(path, "*.safetensors")))


def save_hf_checkpoint(arch: Qwen3Arch, path: str, seed: int = 0, std: float = 0.02,
                       dtype=torch.bfloat16, device="cpu", max_shard_bytes: int = 4 << 30) -> None:
    """Write the seeded random weights as an HF Qwen3 checkpoint directory."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    src = _RandomSource(arch, seed, std, device)
    shard, shard_bytes, n_shard, index = {}, 0, 0, {}

    def flush():
        nonlocal shard, shard_bytes, n_shard
        if not shard:
            return
        fname = f"model-{n_shard:05d}.safetensors"
        save_file(shard, os.path.join(path, fname), metadata={"format": "pt"})
        for k in shard:
            index[k] = fname
        shard, shard_bytes = {}, 0
        n_shard += 1

    for name in src.shapes:
        t = src.get(name, dtype).cpu()
        shard[name] = t
        shard_bytes += t.numel() * t.element_size()
        if shard_bytes >= max_shard_bytes:
            flush()
    flush()
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": index}, f)
    cfg = arch.to_hf_dict()
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    with open(os.path.join(path, "generation_config.json"), "w") as f:
        json.dump({"bos_token_id": arch.bos_token_id, "eos_token_id": arch.eos_token_id}, f)
