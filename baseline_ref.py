"""Reference arm of ``bench.py``: the unmodified reference engine on the same workload.

The reference (Xhkkji/nanovllm_self) ships no packaging metadata, so ``pip install`` of
its source tree fails ("neither setup.py nor pyproject.toml").  ``install_reference()``
(run by ``__graft_entry__.build()``) first tries exactly that install into
``baseline/_ref``; when it fails it copies the tree's ``nanovllm`` and ``pd_self``
packages, unmodified, to a temporary directory, adds a ``pyproject.toml`` that only names
those two packages, and runs the same offline ``pip install --target baseline/_ref`` on
the copy.  The arm then imports the reference from ``baseline/_ref``.

What the harness does around the reference (none of it changes the reference's code):

* writes a random-init Qwen3 HF checkpoint (``config.json`` + safetensors, the same seeded
  weights this repository's engine draws) plus a word-level tokenizer, because the
  reference always loads weights and a tokenizer from a directory
  (``nanovllm/engine/llm_engine.py:107``, ``nanovllm/models/qwen3.py:291``); cached under
  ``/tmp`` so the runs of one box share it;
* wraps ``transformers.AutoModelForCausalLM.from_pretrained`` to drop ``device_map="cpu"``:
  the reference loads its weights with that argument (``nanovllm/models/qwen3.py:295-300``),
  and transformers 5.5 refuses any ``device_map`` unless the ``accelerate`` package is
  installed, which this image does not have (nor its offline wheelhouse).  Loading on the
  CPU is what transformers does without a ``device_map``, so the reference's own loading
  code runs unchanged;
* raises the reference's module-level ``config.num_blocks`` so its fixed KV pool holds the
  whole workload (the reference never preempts and otherwise stalls,
  ``nanovllm/engine/scheduler.py:211-218``);
* passes list-of-tensor inputs with greedy ``SamplingParams`` and ``ignore_eos=True``;
* times each engine step on the device with CUDA events recorded by forward hooks on the
  reference's model (start) and sampler (end), and the whole ``generate`` for e2e.
"""
from __future__ import annotations

import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
CKPT_ROOT = "/tmp/nvb_ref_ckpt"
_PYPROJECT = """[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "nanovllm-self-reference"
version = "0.0.0"

[tool.setuptools.packages.find]
where = ["."]
include = ["nanovllm*", "pd_self*"]
namespaces = true
"""


def reference_source() -> str | None:
    """The reference's source tree: $NVB_REFERENCE_SRC, else BASELINE.json's reference_path."""
    src = os.environ.get("NVB_REFERENCE_SRC")
    if not src:
        try:
            with open(os.path.join(ROOT, "BASELINE.json")) as f:
                src = json.load(f).get("reference_path")
        except (OSError, ValueError):
            src = None
    return src if src and os.path.isdir(os.path.join(src, "nanovllm")) else None


def install_reference(quiet: bool = True) -> str:
    """Install the unmodified reference into baseline/_ref (offline); returns what happened.

    Never raises: a machine without the reference tree simply leaves the arm unavailable.
    """
    import shutil
    import subprocess
    import tempfile
    if os.path.isdir(os.path.join(REF_DIR, "nanovllm")):
        return "already installed"
    src = reference_source()
    if src is None:
        return "reference source tree not found"
    pip = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
           "/opt/wheelhouse", "--target", REF_DIR]
    out = subprocess.DEVNULL if quiet else None
    try:
        if subprocess.call(pip + [src], stdout=out, stderr=out, timeout=600) == 0:
            return f"pip install of {src}"
        tmp = tempfile.mkdtemp(prefix="nvb_ref_src_")
        for pkg in ("nanovllm", "pd_self"):
            shutil.copytree(os.path.join(src, pkg), os.path.join(tmp, pkg),
                            ignore=shutil.ignore_patterns("__pycache__"))
        with open(os.path.join(tmp, "pyproject.toml"), "w") as f:
            f.write(_PYPROJECT)
        rc = subprocess.call(pip + ["--no-deps", tmp], stdout=out, stderr=out, timeout=600)
        shutil.rmtree(tmp, ignore_errors=True)
        return f"pip install of a packaged copy of {src}" if rc == 0 else f"pip install failed (rc={rc})"
    except (OSError, subprocess.SubprocessError) as e:
        return f"install failed: {e!r}"


def unavailable(reason: str) -> None:
    print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


def write_tokenizer(path: str, vocab_size: int, eos_id: int) -> None:
    from tokenizers import Tokenizer, models, pre_tokenizers
    vocab = {f"t{i}": i for i in range(vocab_size)}
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="t0"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": f"t{eos_id}", "unk_token": "t0",
                   "model_max_length": 1 << 20}, f)
    with open(os.path.join(path, "special_tokens_map.json"), "w") as f:
        json.dump({"eos_token": f"t{eos_id}", "unk_token": "t0"}, f)


def ensure_checkpoint(model: str, seed: int, rank: int, device: str, timeout_s: float = 1800.0) -> str:
    from nanovllm_self_b200.models.configs import PRESETS
    from nanovllm_self_b200.models.loader import save_hf_checkpoint
    arch = PRESETS[model]
    path = os.path.join(CKPT_ROOT, f"{model}-seed{seed}")
    marker = os.path.join(path, ".complete")
    if os.path.exists(marker):
        return path
    if rank == 0:
        os.makedirs(path, exist_ok=True)
        save_hf_checkpoint(arch, path, seed=seed, device=device)
        write_tokenizer(path, arch.vocab_size, arch.eos_token_id)
        with open(marker, "w") as f:
            f.write("ok")
    else:
        deadline = time.time() + timeout_s
        while not os.path.exists(marker):
            if time.time() > deadline:
                raise TimeoutError("rank 0 did not finish writing the checkpoint")
            time.sleep(1.0)
    return path


def _allow_cpu_device_map() -> None:
    import transformers
    cls = transformers.AutoModelForCausalLM
    if getattr(cls, "_nvb_cpu_map_ok", False):
        return
    orig = cls.from_pretrained

    def from_pretrained(*a, **kw):
        if kw.get("device_map") == "cpu":
            kw.pop("device_map")
        return orig(*a, **kw)

    cls.from_pretrained = from_pretrained
    cls._nvb_cpu_map_ok = True


class StepTimer:
    """CUDA events from a forward pre-hook on the model to a forward hook on the sampler."""

    def __init__(self, model, sampler):
        import torch
        self.torch = torch
        self.pairs = []
        model.register_forward_pre_hook(self._start)
        model.register_forward_hook(self._end)
        sampler.register_forward_hook(self._end)

    def _start(self, *a):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        self.pairs.append([e, None])

    def _end(self, *a):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        if self.pairs:
            self.pairs[-1][1] = e

    def take_ms(self) -> float:
        self.torch.cuda.synchronize()
        ms = sum(s.elapsed_time(e) for s, e in self.pairs if e is not None)
        self.pairs = []
        return ms


def run_reference_arm(args, workload, step_seed, ClockSampler, dist_info, reduce_max, metric, model_names):
    if not os.path.isdir(os.path.join(REF_DIR, "nanovllm")):
        unavailable("reference not installed under baseline/_ref (build() installs it when the reference source tree "
                    "is present)")
        return
    import torch
    import torch.distributed as dist
    rank, world, local = dist_info()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.kv == "fp8":
        if rank == 0:
            unavailable("the reference has no fp8 KV cache (only int8_mock)")
        return
    if not torch.cuda.is_available():
        if rank == 0:
            unavailable("no CUDA device on this machine (the reference runs on GPUs only)")
        return
    torch.cuda.set_device(local)
    try:
        path = ensure_checkpoint(args.model, 0, rank, f"cuda:{local}")
    except Exception as e:  # pragma: no cover - box dependent
        if rank == 0:
            unavailable(f"could not write the random checkpoint: {e!r}"[:300])
        return
    sys.path.insert(0, REF_DIR)
    try:
        import importlib
        from nanovllm.llm import LLM_self
        # the package re-exports a class under the module's name: fetch the module itself
        ref_engine = importlib.import_module("nanovllm.engine.llm_engine")
        from nanovllm.sampling_params import SamplingParams as RefSP
    except Exception as e:  # pragma: no cover
        if rank == 0:
            unavailable(f"reference import failed: {e!r}"[:300])
        return
    from nanovllm_self_b200.models.configs import PRESETS
    arch = PRESETS[args.model]
    prompts, outs = workload(args.num_requests, arch.vocab_size)
    bs = ref_engine.config.block_size
    blocks_needed = sum((len(p) + o + bs - 1) // bs for p, o in zip(prompts, outs)) + 8
    ref_engine.config.num_blocks = max(ref_engine.config.num_blocks, blocks_needed)
    _allow_cpu_device_map()
    try:
        llm = LLM_self(model_path=path, tensor_parallel_size=args.gpus)
    except Exception as e:
        if rank == 0:
            unavailable(f"reference engine failed to start: {e!r}"[:300])
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()
        return
    timer = StepTimer(llm.model_runner.model, llm.model_runner.sampler)
    sps = [RefSP(temperature=0.0, max_tokens=o, ignore_eos=True) for o in outs]

    def step_inputs(phase, i):
        ps = workload(args.num_requests, arch.vocab_size, token_seed=step_seed(phase, i))[0]
        return ps, [torch.tensor(p, dtype=torch.long) for p in ps]

    try:
        for i in range(args.warmup):
            llm.generate(step_inputs("warmup", i)[1], sps)
    except Exception as e:
        if rank == 0:
            unavailable(f"reference generate failed: {e!r}"[:300])
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()
        return
    timed = [step_inputs("timed", i) for i in range(args.steps)]
    timer.take_ms()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    gen = 0
    for step_prompts, inputs in timed:
        # return_metrics=True raises in this reference snapshot (it reads a
        # ``prefill_backend`` attribute its PagedAttention no longer has), so count here
        outs_ids = llm.generate(inputs, sps)
        gen += sum(len(o) - len(p) for o, p in zip(outs_ids, step_prompts))
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    wall_ms = ev0.elapsed_time(ev1)
    dev_ms = timer.take_ms()
    clk = clocks.stop()
    dev_max, wall_max = reduce_max([dev_ms, wall_ms], world, f"cuda:{local}")
    if rank == 0:
        name = model_names.get(args.model, args.model)
        h2d = sum(len(p) for p in prompts) * 8  # the reference moves int64 ids; lower bound
        print(json.dumps({
            "metric": metric, "value": round(gen / (dev_max / 1e3), 2), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall_max / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: uniform-random prompt token ids, random-init weights N(0, 0.02), seed 0",
            "config": {"model": name, "global_batch": args.num_requests,
                       "seq_len": "prompt U[100,1024], output U[100,1024]", "parallelism": f"tp{args.gpus}",
                       "kv_cache": "bf16", "num_blocks": ref_engine.config.num_blocks,
                       "attention_backend": "flash_attn (reference default)",
                       "l2": "no flush: each step streams the full weights (>> 126 MB L2)",
                       "prompts": "fresh token ids every warm-up and timed step (same lengths)",
                       "reference_dir": REF_DIR,
                       "step": "one LLM_self.generate over all requests"},
            "generated_tokens_per_step": gen // max(args.steps, 1), "clocks": clk,
            "e2e": {"value": round(gen / (wall_max / 1e3), 2), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": gen * 8 // max(args.steps, 1)},
            "gpu_launches": None, "impl": "reference"}), flush=True)
    if world > 1 and dist.is_initialized():
        dist.destroy_process_group()
