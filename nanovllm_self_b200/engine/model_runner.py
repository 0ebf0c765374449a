"""Model runner: owns the model, the paged KV pool, input packing, CUDA graphs, sampling.

Reference counterpart: ``nanovllm/engine/model_runner.py:14-579``.  Same contract:
``run(seqs) -> (token_ids, seq_need_compute_logits)`` where the second list holds the
batch indices of the sequences that sampled this step.

B200-first differences:

* KV pool layout ``[2, L, num_blocks, kv_heads, block_size, head_dim]`` (one block of
  one head is a contiguous ``block_size x head_dim`` tile that a kernel can stream);
  ``num_blocks`` is sized from free HBM when the config says ``-1``;
* the whole step's integer metadata is packed on the host (numpy, no per-token Python
  loops) into one pinned buffer and moved with ONE host-to-device copy;
* decode-only steps replay a CUDA graph captured per batch-size bucket
  (``[1, 2, 4, 8] + 16k`` up to ``cuda_graph_max_bs``, reference :80) that contains the
  whole forward *and* the sampler; mixed prefill steps run eagerly;
* sampled ids come back through one pinned device-to-host copy.
"""
from __future__ import annotations

import math
import os

import numpy as np
import torch

from ..models.configs import resolve_arch
from ..models.loader import has_checkpoint, load_safetensors, random_init
from ..models.qwen3 import Qwen3ForCausalLM
from ..ops import get_ops
from ..parallel.state import TPState
from ..utils.context import Context
from .block_manager import BlockManager
from .sequence import Sequence


def graph_buckets(max_bs: int) -> list[int]:
    b = [x for x in (1, 2, 4, 8) if x <= max_bs]
    b += list(range(16, max_bs + 1, 16))
    if b[-1] != max_bs:
        b.append(max_bs)
    return b


class _Packed:
    """Host-side packed step inputs (int32 segments in one pinned buffer)."""
    __slots__ = ("T", "B", "W", "S", "n_decode", "offsets", "host", "temps", "top_p", "q_lens", "k_lens",
                 "need", "max_q", "max_k")


class ModelRunner:
    def __init__(self, config, tp: TPState | None = None, comm=None):
        self.config = config
        self.tp = tp or TPState()
        self.device = torch.device(config.device) if not config.is_cuda else (
            self.tp.device if self.tp.device.type == "cuda" else torch.device("cuda", torch.cuda.current_device()))
        self.is_cuda = self.device.type == "cuda"
        self.arch = resolve_arch(config.model, config.model_path)
        dtype = config.dtype
        self.model = Qwen3ForCausalLM(self.arch, self.tp.rank, self.tp.size, dtype=dtype, device=self.device)
        with torch.inference_mode():
            if has_checkpoint(config.model_path):
                load_safetensors(self.model, config.model_path)
            else:
                random_init(self.model, seed=config.seed, std=config.init_std)
        self.ops = get_ops(self.device, config.use_custom_kernels)
        if hasattr(self.ops, "prefill_tc"):
            self.ops.prefill_tc = config.prefill_attention == "tcgen05"
        if config.deterministic and hasattr(self.ops, "C"):
            self.ops.C.gemm_set_deterministic(True)
        self.comm = comm
        max_pos = max(config.max_model_len + 1, 16)
        self.model.finalize(self.ops, comm, max_position=max(max_pos, self.arch.max_position_embeddings))
        self.block_size = config.block_size
        self.max_blocks_per_seq = (config.max_model_len + self.block_size - 1) // self.block_size
        self.num_blocks = self._decide_num_blocks()
        self._allocate_kv_cache()
        self.block_manager = BlockManager(self.num_blocks, self.block_size, config.enable_prefix_cache)
        self.sample_step = 0
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.last_dev_ms = 0.0
        # NVTX ranges around each step (NVB_NVTX=1): visible in an external timeline profiler
        self.nvtx = self.is_cuda and os.environ.get("NVB_NVTX", "0") not in ("", "0")
        self.graph_launches: dict = {}
        self._use_top_p = False
        self._gen = torch.Generator(device=self.device)
        self._gen.manual_seed(config.seed)
        self.graphs: dict = {}
        self.graph_pool = None
        self.enable_cuda_graph = bool(self.is_cuda and config.enable_cuda_graph and not config.enforce_eager)
        self._staging_dev = None
        self._pinned = None
        self._out_pinned = None
        if comm is not None:
            comm.bind(self)
        if self.is_cuda:
            self._alloc_staging()
        if self.enable_cuda_graph:
            self.capture_cuda_graphs()

    # ---------------------------------------------------------------- memory
    def kv_block_bytes(self) -> int:
        m = self.model
        elem = torch.empty(0, dtype=self.config.kv_cache_dtype).element_size()
        per = 2 * m.num_layers * m.num_kv_heads * self.block_size * m.head_dim * elem
        if self.config.kv_cache_quant_mode == "fp8":
            per += 2 * m.num_layers * m.num_kv_heads * 4
        elif self.config.kv_cache_quant_mode == "int8_mock":
            per += 2 * m.num_layers * m.num_kv_heads * self.block_size * 4
        return per

    def _activation_reserve(self) -> int:
        m, c = self.model, self.config
        t = c.max_num_batched_tokens
        per_tok = (m.q_size + 2 * m.kv_size) + 2 * m.intermediate + m.intermediate + 4 * m.hidden_size + m.q_size
        acts = t * per_tok * 2 * 2
        logits = max(c.max_num_seqs, c.cuda_graph_max_bs) * (m.vocab_end - m.vocab_start) * 4 * 2
        return acts + logits + (2 << 30)

    def _decide_num_blocks(self) -> int:
        c = self.config
        if c.num_blocks > 0:
            return c.num_blocks
        if not self.is_cuda:
            need = c.max_num_seqs * self.max_blocks_per_seq
            return max(8, min(need, 4096))
        free, total = torch.cuda.mem_get_info(self.device)
        used = total - free
        budget = int(total * c.gpu_memory_utilization) - used - self._activation_reserve()
        n = max(budget // self.kv_block_bytes(), 0)
        if self.tp.size > 1:
            t = torch.tensor([n], dtype=torch.int64, device=self.device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
            n = int(t.item())
        if n < 2:
            raise RuntimeError("not enough device memory for the KV cache")
        return int(n)

    def _allocate_kv_cache(self):
        m, c = self.model, self.config
        shape = (2, m.num_layers, self.num_blocks, m.num_kv_heads, self.block_size, m.head_dim)
        self._kv_ipc = None
        scale_shape = (2, m.num_layers, self.num_blocks, m.num_kv_heads)
        self._scale_off = 0
        self._flag_off = 0
        self.push_flags = None
        if c.kv_pool_ipc and self.is_cuda:
            # one IPC allocation: the pool, then (fp8) its per-block scales, then the push
            # completion flags (one 32-bit word per sending worker), each at a 256-byte offset,
            # so a peer's push kernels and its completion signal reach all of it through one handle
            from ..ops._ext import load
            from ..parallel.symm import _DevPtr
            C = load()
            nbytes = int(np.prod(shape)) * torch.empty(0, dtype=c.kv_cache_dtype).element_size()
            self._scale_off = (nbytes + 255) // 256 * 256
            scale_end = self._scale_off + (int(np.prod(scale_shape)) * 4 if c.kv_cache_quant_mode == "fp8" else 0)
            self._flag_off = (scale_end + 255) // 256 * 256
            total = self._flag_off + int(C.PUSH_FLAG_SLOTS) * 4
            ptr, handle = C.symm_alloc(total)
            self._kv_ipc = (C, ptr, handle)
            raw = torch.as_tensor(_DevPtr(ptr, total), device=self.device)
            self.kv_cache = raw[:nbytes].view(c.kv_cache_dtype).view(shape)
            if c.kv_cache_quant_mode == "fp8":
                self.kv_scale_cache = raw[self._scale_off:scale_end].view(torch.float32).view(scale_shape)
                self.kv_scale_cache.fill_(1.0)
            self.push_flags = raw[self._flag_off:total].view(torch.int32)
            self.push_flags.zero_()
        else:
            self.kv_cache = torch.zeros(shape, dtype=c.kv_cache_dtype, device=self.device)
        if not (c.kv_pool_ipc and self.is_cuda and c.kv_cache_quant_mode == "fp8"):
            self.kv_scale_cache = None
        if c.kv_cache_quant_mode == "fp8" and self.kv_scale_cache is None:
            self.kv_scale_cache = torch.ones(scale_shape, dtype=torch.float32, device=self.device)
        elif c.kv_cache_quant_mode == "int8_mock":
            self.kv_scale_cache = torch.ones(2, m.num_layers, self.num_blocks, m.num_kv_heads, self.block_size,
                                             dtype=torch.float32, device=self.device)
        self.kv_layers = [(self.kv_cache[0, i], self.kv_cache[1, i]) for i in range(m.num_layers)]
        self.kv_scale_layers = None
        if self.kv_scale_cache is not None:
            self.kv_scale_layers = [(self.kv_scale_cache[0, i], self.kv_scale_cache[1, i])
                                    for i in range(m.num_layers)]

    def export_kv_pool(self) -> bytes:
        """CUDA IPC handle (64 bytes) + byte offset (8 bytes) of the KV pool, for a peer's push kernel.

        Needs ``kv_pool_ipc=True``: the pool is then its own cudaMalloc allocation."""
        if self._kv_ipc is None:
            raise RuntimeError("the KV pool was not allocated for IPC (set kv_pool_ipc=True)")
        return bytes(self._kv_ipc[2]) + (0).to_bytes(8, "little")

    @property
    def kv_scale_offset(self) -> int:
        """Byte offset of the fp8 scales inside the exported allocation (0: no scales)."""
        return self._scale_off if self.kv_scale_cache is not None and self._kv_ipc is not None else 0

    @property
    def push_flag_offset(self) -> int:
        """Byte offset of the push completion flags inside the exported allocation (0: none)."""
        return self._flag_off if self._kv_ipc is not None else 0

    def wait_push(self, slot: int, epoch: int, timeout_s: float = 10.0) -> torch.Tensor:
        """Make this runner's stream wait until sender `slot` has signalled push `epoch`.

        Bounded: on expiry the stream goes on.  Returns a device int32 status, 1 once the flag
        arrived and 2 if the wait gave up (the pushed blocks are then not usable)."""
        C = self._kv_ipc[0]
        flag = self.push_flags[slot]
        status = torch.zeros(1, dtype=torch.int32, device=self.device)
        C.kv_push_wait(int(flag.data_ptr()), int(epoch), int(timeout_s * 1e9), status)
        return status

    def _alloc_staging(self):
        c = self.config
        maxT = c.max_num_batched_tokens + max(c.max_num_seqs, c.cuda_graph_max_bs)
        maxB = max(c.max_num_seqs, c.cuda_graph_max_bs)
        n = 3 * maxT + 2 * (maxB + 1) + maxB + maxB * self.max_blocks_per_seq + 2 * maxB + 64
        self._staging_n = n
        self._staging_dev = torch.zeros(n, dtype=torch.int32, device=self.device)
        self._pinned = torch.zeros(n, dtype=torch.int32, pin_memory=True)
        self._out_pinned = torch.zeros(maxB, dtype=torch.int32, pin_memory=True)
        self._out_event = torch.cuda.Event()
        self._ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))

    # --------------------------------------------------------------- packing
    def _pack(self, seqs: list[Sequence], pad_to: int | None = None) -> _Packed:
        """Pack the step: ids, positions, slots, cu_q, ctx_lens, logits idx, block tables, temps."""
        bs = self.block_size
        B = len(seqs)
        Bp = pad_to or B
        W = self.max_blocks_per_seq if pad_to else max(1, max(len(s.block_table) for s in seqs))
        q_lens = [s.num_new_tokens for s in seqs]
        starts = [s.num_cached_tokens for s in seqs]
        k_lens = [a + b for a, b in zip(starts, q_lens)]
        T = sum(q_lens)
        Tp = T + (Bp - B)
        need = [i for i, s in enumerate(seqs) if s.is_need_logits]
        S = len(need) if pad_to is None else Bp
        n_decode = 0
        if pad_to is not None:
            n_decode = B  # graph buckets only ever serve pure decode steps
        else:
            for s in seqs:
                if s.num_new_tokens == 1 and s.is_prefill_done:
                    n_decode += 1
                else:
                    break
        # segments
        offs = {}
        o = 0
        for name, n in (("ids", Tp), ("pos", Tp), ("slot", Tp), ("cuq", Bp + 1), ("ctx", Bp), ("lidx", S),
                        ("bt", Bp * W), ("temp", S), ("topp", S)):
            offs[name] = (o, n)
            o += n
        host = self._pinned.numpy()[:o] if self._pinned is not None else np.zeros(o, dtype=np.int32)
        ids = host[offs["ids"][0]:offs["ids"][0] + Tp]
        pos = host[offs["pos"][0]:offs["pos"][0] + Tp]
        slot = host[offs["slot"][0]:offs["slot"][0] + Tp]
        if n_decode == B:
            ids[:B] = [s.token_ids[-1] for s in seqs]
            p = np.asarray(starts, dtype=np.int64)
            pos[:B] = p
            tbl_last = np.asarray([s.block_table[st // bs] for s, st in zip(seqs, starts)], dtype=np.int64)
            slot[:B] = tbl_last * bs + (p % bs)
        else:
            t0 = 0
            for s, st, ql in zip(seqs, starts, q_lens):
                ids[t0:t0 + ql] = s.token_ids[st:st + ql]
                pp = np.arange(st, st + ql, dtype=np.int64)
                pos[t0:t0 + ql] = pp
                tbl = np.asarray(s.block_table, dtype=np.int64)
                slot[t0:t0 + ql] = tbl[pp // bs] * bs + (pp % bs)
                t0 += ql
        if Tp > T:
            ids[T:Tp] = 0
            pos[T:Tp] = 0
            slot[T:Tp] = -1
        cuq = host[offs["cuq"][0]:offs["cuq"][0] + Bp + 1]
        cuq[0] = 0
        cuq[1:B + 1] = np.cumsum(q_lens)
        if Bp > B:
            cuq[B + 1:] = T + np.arange(1, Bp - B + 1)
        ctx = host[offs["ctx"][0]:offs["ctx"][0] + Bp]
        ctx[:B] = k_lens
        ctx[B:] = 0
        lidx = host[offs["lidx"][0]:offs["lidx"][0] + S]
        if pad_to is None:
            lidx[:] = [int(cuq[i + 1]) - 1 for i in need]
        else:
            lidx[:] = np.arange(Bp)
        bt = host[offs["bt"][0]:offs["bt"][0] + Bp * W].reshape(Bp, W)
        bt.fill(0)
        for i, s in enumerate(seqs):
            bt[i, :len(s.block_table)] = s.block_table
        tview = host[offs["temp"][0]:offs["temp"][0] + S].view(np.float32)
        pview = host[offs["topp"][0]:offs["topp"][0] + S].view(np.float32)
        if pad_to is None:
            tview[:] = [seqs[i].temperature for i in need]
            pview[:] = [seqs[i].top_p for i in need]
        else:
            tview[:B] = [s.temperature for s in seqs]
            tview[B:] = 0.0
            pview[:B] = [s.top_p for s in seqs]
            pview[B:] = 1.0
        pk = _Packed()
        pk.T, pk.B, pk.W, pk.S, pk.n_decode = Tp, Bp, W, S, n_decode if n_decode < B else Bp
        pk.offsets, pk.host, pk.need = offs, host, need
        pk.q_lens, pk.k_lens = q_lens + [1] * (Bp - B), k_lens + [0] * (Bp - B)
        pk.max_q = max(q_lens)
        # The split-KV decode partition depends only on the batch size and max_model_len,
        # so a captured graph and an eager step of the same batch compute identically.
        pk.max_k = self.config.max_model_len
        return pk

    def _to_device(self, pk: _Packed, dev_buf: torch.Tensor | None = None):
        total = sum(n for _, n in pk.offsets.values())
        if self.is_cuda:
            dst = dev_buf if dev_buf is not None else self._staging_dev
            dst[:total].copy_(self._pinned[:total], non_blocking=True)
            self.h2d_bytes += total * 4
        else:
            dst = torch.from_numpy(pk.host[:total].copy())
        v = {k: dst[o:o + n] for k, (o, n) in pk.offsets.items()}
        ctx = Context(
            cu_seqlens_q=v["cuq"], context_lens=v["ctx"], slot_mapping=v["slot"],
            block_tables=v["bt"].view(pk.B, pk.W), logits_indices=v["lidx"],
            seq_need_compute_logits=None, max_seqlen_q=pk.max_q, max_seqlen_k=pk.max_k,
            num_decode_seqs=pk.n_decode, num_seqs=pk.B, num_tokens=pk.T,
            host_q_lens=pk.q_lens, host_k_lens=pk.k_lens)
        temps = v["temp"].view(torch.float32)
        topp = v["topp"].view(torch.float32)
        return v["ids"], v["pos"], ctx, temps, topp

    # ------------------------------------------------------------- execution
    def _forward_and_sample(self, ids, pos, ctx, temps, topp):
        if self._fused_sampler_ok(ctx):
            # one rank, no top-p rows: the sampler runs in the lm_head GEMM's epilogue
            h, residual, normed = self.model.forward_hidden(ids, pos, ctx, self.kv_layers, self.kv_scale_layers)
            if ctx.logits_indices.numel() == 0:
                return torch.empty(0, dtype=torch.int32, device=ids.device)
            x = self.model.final_rows(h, residual, ctx.logits_indices, normed)
            return self.ops.lm_head_sample(x, self.model.lm_head, temps, self._step_tensor(), self.model.vocab_start)
        logits = self.model.forward(ids, pos, ctx, self.kv_layers, self.kv_scale_layers)
        if logits.shape[0] == 0:
            return torch.empty(0, dtype=torch.int32, device=ids.device)
        return self.sample(logits, temps, topp)

    @torch.inference_mode()
    def logits(self, seqs: list[Sequence]) -> torch.Tensor:
        """One eager step's logits, ``[rows that need logits, vocab shard]``, without sampling:
        the KV cache is written as in :meth:`run`, the sequences' state is left unchanged."""
        pk = self._pack(seqs)
        ids, pos, ctx, _, _ = self._to_device(pk)
        return self.model.forward(ids, pos, ctx, self.kv_layers, self.kv_scale_layers)

    def _fused_sampler_ok(self, ctx) -> bool:
        return (self.is_cuda and self.config.fused_sampler and self.tp.size == 1 and not self._use_top_p
                and hasattr(self.ops, "lm_head_sample")
                and ctx.logits_indices.numel() <= getattr(self.ops, "sample_keys_cap", 0))

    def sample(self, logits, temps, topp):
        if self.tp.size > 1 and self.comm is not None:
            return self.comm.vocab_parallel_sample(logits, temps, topp, self.model, self)
        return self.ops.sample(logits, temps, topp, seeds=None, step=self._step_tensor(),
                               batch_greedy_compat=self.config.batch_greedy_compat, generator=self._gen,
                               use_top_p=self._use_top_p)

    def _step_tensor(self):
        if not self.is_cuda:
            return self.sample_step
        if not hasattr(self, "_step_dev"):
            self._step_dev = torch.zeros(2, dtype=torch.int64, device=self.device)
            self._step_dev[0] = self.config.seed
        return self._step_dev

    @torch.inference_mode()
    def run(self, seqs: list[Sequence]):
        if not seqs:
            return [], []
        need = [i for i, s in enumerate(seqs) if s.is_need_logits]
        all_decode = all(s.num_new_tokens == 1 and s.is_prefill_done for s in seqs)
        self._use_top_p = any(seqs[i].top_p < 1.0 and seqs[i].temperature > 0 for i in need)
        if self.config.batch_greedy_compat and any(seqs[i].temperature <= 0 for i in need):
            for i in need:  # reference quirk: one greedy row makes the whole batch greedy
                seqs[i].temperature = 0.0
        graph_bs = None
        if self.enable_cuda_graph and all_decode and not self._use_top_p and len(seqs) <= self.graph_max_bs:
            graph_bs = next(b for b in self.graph_bs_list if b >= len(seqs))
        nvtx = self.nvtx
        if nvtx:
            torch.cuda.nvtx.range_push(f"step bs={len(seqs)} {'graph' if graph_bs else 'eager'}")
        if graph_bs is not None:
            toks = self._run_graph(seqs, graph_bs)
        else:
            pk = self._pack(seqs)
            ids, pos, ctx, temps, topp = self._to_device(pk)
            self._mark(0)
            toks = self._forward_and_sample(ids, pos, ctx, temps, topp)
            self._mark(1)
            toks = self._fetch(toks, len(need))
        if nvtx:
            torch.cuda.nvtx.range_pop()
        self.last_dev_ms = self._ev[0].elapsed_time(self._ev[1]) if self.is_cuda else 0.0
        self.sample_step += 1
        if self.is_cuda:
            self._step_dev[1] += 1
        return toks[:len(need)], need

    def _mark(self, i: int) -> None:
        """Device timestamps around the forward + sampler (excludes host packing and copies)."""
        if self.is_cuda:
            self._ev[i].record()

    def _fetch(self, toks: torch.Tensor, n: int) -> list[int]:
        if n == 0:
            return []
        if not self.is_cuda:
            return [int(x) for x in toks.tolist()]
        self._out_pinned[:n].copy_(toks[:n], non_blocking=True)
        self.d2h_bytes += n * 4
        self._out_event.record()
        self._out_event.synchronize()
        return self._out_pinned[:n].tolist()

    # ----------------------------------------------------------- cuda graphs
    @property
    def graph_max_bs(self) -> int:
        return min(self.config.cuda_graph_max_bs, self.config.max_num_seqs)

    @torch.inference_mode()
    def capture_cuda_graphs(self):
        self.graph_bs_list = graph_buckets(self.graph_max_bs)
        self._step_tensor()
        self._graph_buf = torch.zeros(self._staging_n, dtype=torch.int32, device=self.device)
        dummy_block = 0
        for bs in reversed(self.graph_bs_list):
            fake = []
            for i in range(bs):
                s = Sequence(-1, [0], None, self.block_size)
                s.block_table = [dummy_block]
                s.num_cached_tokens = 0
                s.num_new_tokens = 1
                fake.append(s)
            pk = self._pack(fake, pad_to=bs)
            # Padding-style dummy rows: write nowhere, attend to nothing.
            o, n = pk.offsets["slot"]
            pk.host[o:o + n] = -1
            o, n = pk.offsets["ctx"]
            pk.host[o:o + n] = 0
            ids, pos, ctx, temps, topp = self._to_device(pk, self._graph_buf)
            for _ in range(2):
                self._forward_and_sample(ids, pos, ctx, temps, topp)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            l0 = self._launch_count()
            with torch.cuda.graph(g, pool=self.graph_pool):
                out = self._forward_and_sample(ids, pos, ctx, temps, topp)
            self.graph_launches[bs] = self._launch_count() - l0
            if self.graph_pool is None:
                self.graph_pool = g.pool()
            self.graphs[bs] = (g, out, pk.offsets)
            torch.cuda.synchronize(self.device)

    def _run_graph(self, seqs, bs) -> list[int]:
        g, out, offsets = self.graphs[bs]
        pk = self._pack(seqs, pad_to=bs)
        assert pk.offsets == offsets
        total = sum(n for _, n in offsets.values())
        self._graph_buf[:total].copy_(self._pinned[:total], non_blocking=True)
        self.h2d_bytes += total * 4
        self._mark(0)
        g.replay()
        self._mark(1)
        self._add_launches(self.graph_launches.get(bs, 0))
        return self._fetch(out, len(seqs))

    def _launch_count(self) -> int:
        n = getattr(self.ops, "launches", 0)
        if self.comm is not None:
            n += getattr(self.comm, "launches", 0)
        return n

    def _add_launches(self, n: int) -> None:
        # graph replays launch the captured kernels; attribute them to the op set
        if hasattr(self.ops, "launches"):
            self.ops.launches += n

    def release_graphs(self):
        self.graphs.clear()
        self.graph_pool = None
