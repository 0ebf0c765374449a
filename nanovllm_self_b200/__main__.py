"""Command-line generation: ``python -m nanovllm_self_b200 [options]``.

The reference's entry scripts (``main.py``: two prompts through ``LLM_self`` with the profile
summary, or through the HuggingFace loop; ``pd_self/pd_flow.py``: the same prompt through the
in-process prefill/decode coordinator) as one command:

    python -m nanovllm_self_b200 --model /path/to/Qwen3-8B --prompt "What is a large language model?"
    python -m nanovllm_self_b200 --model qwen3-8b --prompt-ids 1,2,3 --max-tokens 32 --profile
    python -m nanovllm_self_b200 --model qwen3-0.6b --prompt-ids 1,2,3 --pd      # P/D coordinator
    python -m nanovllm_self_b200 --model /path/to/ckpt --prompt "..." --hf        # HuggingFace loop
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m nanovllm_self_b200 --model qwen3-8b --tp 2 ...

``--model`` is a checkpoint directory (its tokenizer encodes ``--prompt``) or an architecture preset
with random weights (give ``--prompt-ids``).  Prints one JSON line per prompt (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import time


def _parse(argv):
    ap = argparse.ArgumentParser(prog="python -m nanovllm_self_b200", description="generate with the B200 engine")
    ap.add_argument("--model", required=True, help="checkpoint directory or preset (tiny, qwen3-0.6b, qwen3-8b, ...)")
    ap.add_argument("--prompt", action="append", default=[], help="text prompt (repeatable; needs a tokenizer)")
    ap.add_argument("--prompt-ids", action="append", default=[], help="comma-separated token ids (repeatable)")
    ap.add_argument("--max-tokens", type=int, default=64)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--top-p", type=float, default=1.0)
    ap.add_argument("--stop-at-eos", action="store_true", help="finish a sequence at EOS (default: ignore EOS)")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--dtype", default="bf16")
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel size (launch with torchrun)")
    ap.add_argument("--kv", default="none", help="kv_cache_quant_mode: none, fp8, int8_mock")
    ap.add_argument("--max-model-len", type=int, default=4096)
    ap.add_argument("--block-size", type=int, default=256)
    ap.add_argument("--num-blocks", type=int, default=-1, help="-1 sizes the KV pool from free memory")
    ap.add_argument("--eager", action="store_true", help="no CUDA graphs")
    ap.add_argument("--profile", action="store_true", help="per-phase host / device time summary")
    mode = ap.add_mutually_exclusive_group()
    mode.add_argument("--pd", action="store_true", help="in-process prefill/decode coordinator")
    mode.add_argument("--hf", action="store_true", help="HuggingFace generate loop (checkpoint directory only)")
    return ap.parse_args(argv)


def main(argv=None) -> list:
    a = _parse(argv)
    ids = [[int(x) for x in s.split(",") if x.strip()] for s in a.prompt_ids]
    if not ids and not a.prompt:
        raise SystemExit("give --prompt or --prompt-ids")
    kw = dict(device=a.device, dtype=a.dtype, max_model_len=a.max_model_len, block_size=a.block_size,
              num_blocks=a.num_blocks, kv_cache_quant_mode=a.kv, enforce_eager=a.eager)
    results = []
    t0 = time.perf_counter()
    if a.hf:
        import torch

        from .llm import HFLLM
        if not os.path.isdir(a.model):
            raise SystemExit("--hf needs a checkpoint directory")
        import glob
        has_tok = bool(glob.glob(os.path.join(a.model, "tokenizer*")))
        if a.prompt and not has_tok:
            raise SystemExit("text prompts need a tokenizer in the checkpoint directory; give --prompt-ids")
        dt = {"fp32": torch.float32, "fp16": torch.float16}.get(a.dtype, torch.bfloat16)
        # without a tokenizer there is no EOS id: -1 never stops
        hf = HFLLM(a.model, device=a.device, dtype=dt, eos_token_id=None if has_tok else -1)
        prompts = ids + [list(hf.tokenizer(p)["input_ids"]) for p in a.prompt]
        for p in prompts:
            out = hf.generate(torch.tensor([p], device=a.device), max_token=a.max_tokens,
                              temperature=a.temperature)
            results.append({"prompt_ids": p, "output_ids": out[0].tolist()[len(p):]})
        tok = hf.tokenizer
    elif a.pd:
        from .config import EngineConfig
        from .pd.coordinator import PDCoordinator
        tok = None
        if os.path.isdir(a.model):
            model_kw = {"model_path": a.model}
            if a.prompt:
                from transformers import AutoTokenizer
                tok = AutoTokenizer.from_pretrained(a.model)
        elif a.prompt:
            raise SystemExit("text prompts need a checkpoint directory with a tokenizer; give --prompt-ids")
        else:
            model_kw = {"model": a.model}
        pd = PDCoordinator(EngineConfig(**model_kw, **kw), tokenizer=tok)
        prompts = ids + [list(tok(p)["input_ids"]) for p in a.prompt]
        outs = pd.generate(prompts, max_tokens=a.max_tokens, temperature=a.temperature,
                           ignore_eos=not a.stop_at_eos)
        results = [{"prompt_ids": p, "output_ids": o[len(p):]} for p, o in zip(prompts, outs)]
    else:
        from . import LLM, SamplingParams
        llm = LLM(a.model, tensor_parallel_size=a.tp, enable_profile=a.profile, **kw)
        prompts = ids + [list(llm.encoder(p)["input_ids"]) for p in a.prompt]
        sp = SamplingParams(temperature=a.temperature, top_p=a.top_p, max_tokens=a.max_tokens,
                            ignore_eos=not a.stop_at_eos)
        outs = llm.generate(prompts, sp)
        results = [{"prompt_ids": p, "output_ids": o[len(p):]} for p, o in zip(prompts, outs)]
        tok = llm.tokenizer
    wall = time.perf_counter() - t0
    if int(os.environ.get("RANK", "0")) == 0:
        for r in results:
            if tok is not None:
                r["text"] = tok.decode(r["output_ids"])
            r["wall_s"] = wall
            print(json.dumps(r), flush=True)
    return results


if __name__ == "__main__":
    main()
