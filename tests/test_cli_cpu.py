"""``python -m nanovllm_self_b200``: token-id prompts through the engine and through the in-process
P/D coordinator give the engine's greedy tokens (tiny random-init model on CPU)."""
import json
import os
import subprocess
import sys

from nanovllm_self_b200 import LLM, SamplingParams
from nanovllm_self_b200.__main__ import main

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASE = ["--model", "tiny", "--device", "cpu", "--dtype", "fp32", "--block-size", "16", "--num-blocks", "64",
        "--max-model-len", "256", "--max-tokens", "6"]
PROMPTS = [[5, 17, 300, 9, 44], [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17]]


def _want():
    llm = LLM("tiny", device="cpu", dtype="fp32", block_size=16, num_blocks=64, max_model_len=256)
    outs = llm.generate(PROMPTS, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    return [o[len(p):] for o, p in zip(outs, PROMPTS)]


def test_engine_and_pd_paths_agree(capsys):
    args = BASE + sum((["--prompt-ids", ",".join(map(str, p))] for p in PROMPTS), [])
    want = _want()
    assert [r["output_ids"] for r in main(args)] == want
    lines = [json.loads(x) for x in capsys.readouterr().out.strip().splitlines()]
    assert [x["output_ids"] for x in lines] == want and [x["prompt_ids"] for x in lines] == PROMPTS
    assert [r["output_ids"] for r in main(args + ["--pd"])] == want


def test_module_entry_point_runs():
    out = subprocess.run([sys.executable, "-m", "nanovllm_self_b200", *BASE, "--prompt-ids", "5,17,300,9,44"],
                         cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    assert json.loads(out.stdout.strip().splitlines()[-1])["output_ids"] == _want()[0]
    bad = subprocess.run([sys.executable, "-m", "nanovllm_self_b200", *BASE], cwd=ROOT, capture_output=True,
                         text=True, timeout=300)
    assert bad.returncode != 0 and "--prompt" in bad.stderr


def test_hf_loop_on_a_checkpoint_without_tokenizer(tmp_path):
    import torch

    from nanovllm_self_b200.models.configs import PRESETS
    from nanovllm_self_b200.models.loader import save_hf_checkpoint
    path = str(tmp_path / "ckpt")
    save_hf_checkpoint(PRESETS["tiny"], path, seed=0, dtype=torch.float32)
    res = main(["--model", path, "--device", "cpu", "--dtype", "fp32", "--max-tokens", "4", "--hf",
                "--prompt-ids", "5,17,300,9,44"])
    assert len(res) == 1 and len(res[0]["output_ids"]) == 4 and all(0 <= t < 1024 for t in res[0]["output_ids"])
