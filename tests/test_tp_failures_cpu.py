"""A tensor-parallel rank that fails between steps, on CPU ranks (gloo): the surviving rank's next
collective ends with an error instead of waiting for ever.

Two forms, both made on the host: the peer process exits (its connection closes), and the peer
stays alive but never joins the collective (the process group's timeout, ``dist_timeout_s``,
ends the wait).  The surviving rank records the exception and how long its step took.
"""
import json
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from nanovllm_self_b200 import LLM, SamplingParams

TIMEOUT_S = 3.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, mode, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    llm = LLM("tiny", tensor_parallel_size=2, device="cpu", dtype="fp32", block_size=16, max_model_len=256,
              num_blocks=32, comm_backend="nccl", dist_timeout_s=TIMEOUT_S)
    prompt = torch.randint(0, 1024, (12,), generator=torch.Generator().manual_seed(1)).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True)
    llm.generate([prompt], sp)  # one healthy request on both ranks
    if rank == 1:
        if mode == "exit":
            os._exit(3)  # the peer dies between steps
        time.sleep(60)   # the peer stalls and never joins the next collective
        os._exit(0)
    t0 = time.time()
    rec = {"error": None}
    try:
        llm.generate([prompt], sp)
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome; hanging is the failure
        rec = {"error": type(e).__name__, "message": str(e)[:300]}
    rec["elapsed_s"] = time.time() - t0
    with open(out_path, "w") as f:
        json.dump(rec, f)
    os._exit(0)  # no gloo teardown with a dead or stalled peer


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_surviving_rank_errors_instead_of_hanging(tmp_path, mode):
    ctx = mp.get_context("spawn")
    port, out = _free_port(), str(tmp_path / "rank0.json")
    procs = [ctx.Process(target=_rank, args=(r, port, mode, out)) for r in (0, 1)]
    for p in procs:
        p.start()
    try:
        procs[0].join(timeout=120)
        assert procs[0].exitcode == 0, "the surviving rank did not finish its step"
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()  # the exact child process this test started
            p.join(timeout=30)
    rec = json.load(open(out))
    assert rec["error"] is not None, rec
    assert rec["elapsed_s"] < TIMEOUT_S + 30, rec
    if mode == "exit":
        assert procs[1].exitcode == 3
    else:  # ended by the process group's timeout, not by anything else
        assert rec["elapsed_s"] >= 0.9 * TIMEOUT_S, rec
