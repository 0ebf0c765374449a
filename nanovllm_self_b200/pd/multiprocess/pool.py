"""P/D pool driver: N prefill workers + M decode workers, routed by the agent-aware router.

Reference: ``pd_self/multiprocess/evaluation/benchmark_agent_pd_pool.py`` (N P + M D workers
in one NCCL world, two-stage routing of P and D with session affinity, closed-loop
concurrency, metrics and summary) and ``benchmark_agent_pd_multi_pair.py`` (fixed pairs).
Arrivals are closed-loop (``concurrency``) or open-loop Poisson (``rate``).  Worker load
feedback comes from each worker's ``worker_state.json``.

``python -m nanovllm_self_b200.pd.multiprocess.pool --help`` runs it from the shell.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

from .agent_scheduler import Router, RouterConfig, estimate
from .control_plane import WorkDir


def _pct(xs, q):
    return float(np.percentile(np.asarray(xs, dtype=np.float64), q)) if xs else 0.0


class PDPool:
    def __init__(self, work_root, num_prefill=1, num_decode=1, backend="shared_memory", model="tiny",
                 prefill_devices=None, decode_devices=None, policy="load_aware", worker_args=None,
                 handshake_timeout_s=120.0, nccl_port=29650, python=sys.executable, tp=1, device_kind="cuda",
                 gpu_base=0):
        self.root = Path(work_root)
        self.root.mkdir(parents=True, exist_ok=True)
        self.P, self.D = num_prefill, num_decode
        self.backend = backend
        self.model = model
        # tp > 1: every worker is a tensor-parallel group of tp processes on consecutive GPUs
        # (prefill group i on GPUs [i tp, (i+1) tp), decode group j after all prefill groups)
        self.tp = tp
        self.device_kind = device_kind
        self.gpu_base = gpu_base  # tp > 1: first GPU of this pool's groups
        if tp > 1 and backend == "sync_gpu":
            raise ValueError("sync_gpu P/D workers are TP=1; use ipc_push or shared_memory with tp > 1")
        if tp > 1:
            self.pdev = [f"{device_kind}:{i * tp}" if device_kind == "cuda" else "cpu" for i in range(num_prefill)]
            self.ddev = [f"{device_kind}:{(num_prefill + i) * tp}" if device_kind == "cuda" else "cpu"
                         for i in range(num_decode)]
        else:
            self.pdev = prefill_devices or [f"cuda:{i}" for i in range(num_prefill)]
            self.ddev = decode_devices or [f"cuda:{num_prefill + i}" for i in range(num_decode)]
        self.p_router = Router(num_prefill, policy)
        self.d_router = Router(num_decode, policy)
        self.worker_args = list(worker_args or [])
        self.timeout = handshake_timeout_s
        self.nccl_port = nccl_port
        self.python = python
        self.procs = []
        self.pwd = [WorkDir(self.root / f"prefill_{i}") for i in range(num_prefill)]
        self.dwd = [WorkDir(self.root / f"decode_{i}") for i in range(num_decode)]
        self.submitted = {}
        self.results = {}
        self.warmup_bases = set()
        self._seq = 0

    # ------------------------------------------------------------- lifecycle
    def _launch(self, role, idx, device, wd, rank):
        args = [role, "--work-dir", str(wd.path), "--model", self.model, "--device", device, "--backend", self.backend,
                "--global-rank", str(rank), "--world-size", str(self.P + self.D), "--nccl-port", str(self.nccl_port),
                "--handshake-timeout-s", str(self.timeout)] + self.worker_args
        if self.tp > 1:
            # one torchrun per group; its ranks form the group's TP world
            offset = self.gpu_base + rank * self.tp if self.device_kind == "cuda" else 0
            cmd = [self.python, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={self.tp}",
                   "--master-addr=127.0.0.1", f"--master-port={self.nccl_port + 1 + rank}",
                   "-m", "nanovllm_self_b200.pd.multiprocess.workers"] + args + \
                  ["--tp", str(self.tp), "--gpu-offset", str(offset)]
        else:
            cmd = [self.python, "-m", "nanovllm_self_b200.pd.multiprocess.workers"] + args
        log = open(wd.f(f"{role}.log"), "w")
        env = dict(os.environ)
        env.setdefault("NCCL_NVLS_ENABLE", "0")
        root = str(Path(__file__).resolve().parents[3])
        env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
        self.procs.append(subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, env=env))

    def start(self, ready_timeout_s: float = 600.0) -> None:
        for wd in self.pwd + self.dwd:
            for stale in ("shutdown", "worker_ready.json", "kv_pool.json"):
                wd.remove(stale)
        for i, wd in enumerate(self.pwd):
            self._launch("prefill", i, self.pdev[i], wd, i)
        for i, wd in enumerate(self.dwd):
            self._launch("decode", i, self.ddev[i], wd, self.P + i)
        deadline = time.time() + ready_timeout_s
        for wd in self.pwd + self.dwd:
            while not wd.exists("worker_ready.json"):
                if time.time() > deadline or any(p.poll() not in (None, 0) for p in self.procs):
                    self.shutdown(force=True)
                    raise RuntimeError(f"worker in {wd.path} failed to start (see its log)")
                time.sleep(0.05)

    def shutdown(self, force: bool = False, timeout_s: float = 120.0) -> None:
        for wd in self.pwd + self.dwd:
            wd.touch("shutdown")
        deadline = time.time() + timeout_s
        codes = []
        for p in self.procs:
            try:
                p.wait(timeout=max(0.1, deadline - time.time()) if not force else 5)
            except subprocess.TimeoutExpired:
                p.kill()
                p.wait(timeout=10)
            codes.append(p.returncode)
        # exit status of every worker process (torchrun's for a TP group): 0 = a clean shutdown
        self.exit_codes = codes
        self.procs = []

    # --------------------------------------------------------------- routing
    def _feedback(self) -> None:
        for router, wds in ((self.p_router, self.pwd), (self.d_router, self.dwd)):
            for i, wd in enumerate(wds):
                try:
                    st = wd.read_json("worker_state.json")
                except (FileNotFoundError, json.JSONDecodeError):
                    continue
                load = st.get("queue_depth", 0) * 0.05 + st.get("active", 0) * 0.01 + (0.02 if st.get("busy") else 0)
                router.update_feedback(i, load, st)

    def submit(self, row: dict, index: int, now_s: float) -> str:
        self._feedback()
        est = estimate(row, index, int(row["max_tokens"]), RouterConfig())
        pm = self.p_router.route(est, now_s)
        dm = self.d_router.route(est, now_s)
        base = f"r{self._seq:06d}"  # unique over the pool's lifetime (several runs may share it)
        self._seq += 1
        req = {"request_id": row.get("id", base), "prompt_ids": row["prompt_ids"], "max_tokens": row["max_tokens"],
               "temperature": row.get("temperature", 0.0), "ignore_eos": row.get("ignore_eos", True),
               "session_id": est.session_id, "decode_work_dir": str(self.dwd[dm["worker_id"]].path),
               "dst_rank": self.P + dm["worker_id"]}
        self.pwd[pm["worker_id"]].write_json(f"{base}.request.json", req)
        self.submitted[base] = {"submit_time": time.time(), "p": pm, "d": dm, "row": row}
        return base

    def _collect(self) -> list:
        done = []
        for base, info in list(self.submitted.items()):
            if base in self.results:
                continue
            dwd = self.dwd[info["d"]["worker_id"]]
            for stage in ("prefill", "decode"):
                if dwd.exists(f"{base}.{stage}_error.json"):
                    self.results[base] = {"error": dwd.read_json(f"{base}.{stage}_error.json")["error"]}
                    done.append(base)
                    break
            else:
                if dwd.exists(f"{base}.decode_done"):
                    dm = dwd.read_json(f"{base}.decode_metrics.json")
                    pm = dwd.read_json(f"{base}.prefill_metrics.json") if dwd.exists(f"{base}.prefill_metrics.json") else {}
                    t_sub = info["submit_time"]
                    first = pm.get("prefill_start_time", t_sub) + pm.get("prefill_time_s", 0.0)
                    n_out = len(dm.get("output_ids", []))
                    end = dm.get("finish_time", time.time())
                    self.results[base] = {"output_ids": dm.get("output_ids", []), "ttft_s": first - t_sub,
                                          "tpot_s": (end - first) / max(1, n_out - 1), "e2e_s": end - t_sub,
                                          "prefill": pm, "decode": dm}
                    done.append(base)
        return done

    def request_rows(self) -> list:
        """One row per finished request in the fields every P/D and single-engine driver
        writes (``request_id``, token counts, ``ttft_s``/``tpot_s``/``e2e_s``, ``output_ids``,
        or ``error``)."""
        rows = []
        for base, res in self.results.items():
            row = self.submitted[base]["row"]
            out = {"request_id": row.get("id", base), "session_id": row.get("session_id"),
                   "input_tokens": len(row["prompt_ids"]), "max_tokens": row["max_tokens"]}
            if base in self.warmup_bases:
                out["warmup"] = True
            if "error" in res:
                out["error"] = res["error"]
            else:
                out.update(output_tokens=len(res["output_ids"]), ttft_s=res["ttft_s"], tpot_s=res["tpot_s"],
                           e2e_s=res["e2e_s"], output_ids=res["output_ids"])
            rows.append(out)
        return rows

    def dead_workers(self) -> list:
        """(role, index, exit code) of every worker process that has exited."""
        dead = []
        roles = [("prefill", i) for i in range(self.P)] + [("decode", i) for i in range(self.D)]
        for (role, idx), p in zip(roles, self.procs):
            rc = p.poll()
            if rc is not None:
                dead.append((role, idx, rc))
        return dead

    def _fail_stuck(self, inflight: set, request_timeout_s: float | None) -> list:
        """Mark in-flight requests routed to an exited worker, or older than the request
        timeout (a lost control message), as failed; returns their bases."""
        failed = []
        dead = self.dead_workers() if self.procs else []
        dead_p = {i for role, i, _ in dead if role == "prefill"}
        dead_d = {i for role, i, _ in dead if role == "decode"}
        now = time.time()
        for base in list(inflight):
            info = self.submitted[base]
            why = None
            if info["p"]["worker_id"] in dead_p:
                why = f"prefill worker {info['p']['worker_id']} exited"
            elif info["d"]["worker_id"] in dead_d:
                why = f"decode worker {info['d']['worker_id']} exited"
            elif request_timeout_s is not None and now - info["submit_time"] > request_timeout_s:
                why = f"no completion within {request_timeout_s} s"
            if why is not None and base not in self.results:
                self.results[base] = {"error": why}
                failed.append(base)
        return failed

    def run(self, rows: list, concurrency: int | None = 4, rate: float | None = None, timeout_s: float = 3600.0,
            seed: int = 0, request_timeout_s: float | None = None) -> dict:
        """Drive `rows` through the pool.  A request whose worker exits, or (with
        `request_timeout_s`) that does not complete in time, is recorded as an error instead of
        stalling the run; `timeout_s` bounds the whole run."""
        rng = random.Random(seed)
        t0 = time.time()
        next_arrival = 0.0
        i = 0
        inflight = set()
        mine = []  # this run's requests: the summary covers them only
        while i < len(rows) or inflight:
            now = time.time() - t0
            if i < len(rows):
                if rate:
                    if now >= next_arrival:
                        mine.append(self.submit(rows[i], i, now))
                        inflight.add(mine[-1])
                        i += 1
                        next_arrival += rng.expovariate(rate)
                elif len(inflight) < (concurrency or 1):
                    mine.append(self.submit(rows[i], i, now))
                    inflight.add(mine[-1])
                    i += 1
            for b in self._collect():
                inflight.discard(b)
            for b in self._fail_stuck(inflight, request_timeout_s):
                inflight.discard(b)
            if time.time() - t0 > timeout_s:
                raise TimeoutError("P/D pool run timed out")
            time.sleep(0.001)
        wall = time.time() - t0
        ok = [self.results[b] for b in mine if "error" not in self.results[b]]
        gen = sum(len(r["output_ids"]) for r in ok)
        return {"policy": self.p_router.policy, "num_requests": len(rows), "num_errors": len(mine) - len(ok),
                "wall_s": wall,
                "output_tok_s": gen / wall if wall > 0 else 0.0,
                "ttft_ms_p50": _pct([r["ttft_s"] * 1e3 for r in ok], 50),
                "ttft_ms_p99": _pct([r["ttft_s"] * 1e3 for r in ok], 99),
                "tpot_ms_p50": _pct([r["tpot_s"] * 1e3 for r in ok], 50),
                "tpot_ms_p99": _pct([r["tpot_s"] * 1e3 for r in ok], 99),
                "e2e_s_p90": _pct([r["e2e_s"] for r in ok], 90),
                "prefill_router": self.p_router.summary(), "decode_router": self.d_router.summary()}

    def warmup(self, rows: list, concurrency: int = 1, timeout_s: float = 3600.0) -> None:
        """Serve `rows` unmeasured; their rows carry ``warmup: true`` (the correctness check skips them)."""
        before = set(self.submitted)
        self.run(rows, concurrency=concurrency, timeout_s=timeout_s)
        self.warmup_bases |= set(self.submitted) - before


def main(argv=None):
    ap = argparse.ArgumentParser(description="P/D pool benchmark driver")
    ap.add_argument("--work-root", required=True)
    ap.add_argument("--num-prefill", type=int, default=1)
    ap.add_argument("--num-decode", type=int, default=1)
    ap.add_argument("--backend", default="ipc_push")
    ap.add_argument("--model", default="qwen3-0.6b")
    ap.add_argument("--policy", default="affinity_load_aware")
    ap.add_argument("--num-requests", type=int, default=32)
    ap.add_argument("--rate", type=float, default=None)
    ap.add_argument("--concurrency", type=int, default=4)
    ap.add_argument("--input-mean", type=float, default=2048)
    ap.add_argument("--output-mean", type=float, default=256)
    ap.add_argument("--out", default=None, help="JSON summary path; per-request rows go to <out>.jsonl")
    ap.add_argument("--tp", type=int, default=1, help="each worker is a TP group of this many GPUs")
    ap.add_argument("--prefill-gpus", default=None, help="TP = 1: GPU index of each prefill worker, e.g. 0,2")
    ap.add_argument("--decode-gpus", default=None, help="TP = 1: GPU index of each decode worker, e.g. 1,3")
    ap.add_argument("--load-mode", choices=["closed_loop", "batch"], default="closed_loop",
                    help="closed_loop: --concurrency in flight (or Poisson at --rate); batch: every request at once")
    ap.add_argument("--warmup", type=int, default=0, help="unmeasured requests served first")
    ap.add_argument("--dataset", default=None, help="JSON-lines rows (benchmarks.datasets); default synthetic")
    args, rest = ap.parse_known_args(argv)
    from .pairs import load_rows, synthetic_rows
    if args.dataset:
        rows = load_rows(args.dataset, args.num_requests + args.warmup)
    else:
        rows = synthetic_rows(args.num_requests + args.warmup, args.input_mean, args.output_mean,
                              sessions=max(1, args.num_requests // 4), max_output=1024)
    kw = {}
    if args.prefill_gpus:
        kw["prefill_devices"] = [f"cuda:{g}" for g in args.prefill_gpus.split(",")]
        args.num_prefill = len(kw["prefill_devices"])
    if args.decode_gpus:
        kw["decode_devices"] = [f"cuda:{g}" for g in args.decode_gpus.split(",")]
        args.num_decode = len(kw["decode_devices"])
    pool = PDPool(args.work_root, args.num_prefill, args.num_decode, args.backend, args.model, policy=args.policy,
                  worker_args=rest, tp=args.tp, **kw)
    pool.start()
    try:
        if args.warmup:
            pool.warmup(rows[:args.warmup])
        measured = rows[args.warmup:]
        conc = len(measured) if args.load_mode == "batch" else args.concurrency
        summary = pool.run(measured, concurrency=conc, rate=None if args.load_mode == "batch" else args.rate)
        summary.update(load_mode=args.load_mode, warmup=args.warmup)
    finally:
        pool.shutdown()
    print(json.dumps(summary))
    if args.out:
        with open(args.out, "w") as f:
            json.dump(summary, f, indent=1)
        with open(args.out + ".jsonl", "w") as f:
            for r in pool.request_rows():
                f.write(json.dumps(r) + "\n")


if __name__ == "__main__":
    main()
