"""TP consistency / memory matrix on CPU ranks (gloo): TP = 1, 2 and 4 generate the same greedy
tokens, and every rank holds 1/TP of the weights and of each KV block (the replicated norms
excepted)."""
import json
import os
import socket

import torch.multiprocessing as mp

from nanovllm_self_b200.benchmarks import tp_matrix

KW = dict(device="cpu", dtype="fp32", block_size=16, max_model_len=256, num_blocks=64, comm_backend="nccl")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    tp_matrix.run_case(result_dir, "tiny-tp8", max_tokens=10, **KW)
    import torch.distributed as dist
    dist.barrier()
    os._exit(0)  # no gloo teardown at interpreter exit (its destructor can race its own threads)


def test_tp_matrix_tokens_and_shards(tmp_path, capsys):
    d = str(tmp_path)
    for k in ("RANK", "WORLD_SIZE"):
        assert k not in os.environ
    tp_matrix.run_case(d, "tiny-tp8", max_tokens=10, **KW)
    for world in (2, 4):
        mp.spawn(_rank, args=(world, _free_port(), d), nprocs=world, join=True)
    tp_matrix.main(["summary", "--result-dir", d, "--tps", "1,2,4"])
    printed = json.loads(capsys.readouterr().out)
    assert set(printed) == {"1", "2", "4"}
    s = json.loads((tmp_path / "summary.json").read_text())
    assert s["all_match"]
    for tp, c in s["cases"].items():
        assert c["ranks"] == int(tp)
        assert len(c["generated_token_ids"]) == 10
        assert 1.0 <= c["weight_shard_ratio"] < 1.1, c["weight_shard_ratio"]
        assert abs(c["kv_block_shard_ratio"] - 1.0) < 1e-9
        assert len(set(c["weight_mb_per_rank"])) == 1  # every rank holds the same share
        assert [m["rank"] for m in c["rank_memory"]] == list(range(int(tp)))


def test_matrix_command_runs_each_size_as_its_own_job(tmp_path, capsys):
    """The one-command form: TP 1 in-process and TP 2 under torch.distributed.run (gloo on CPU)."""
    tp_matrix.main(["matrix", "--result-dir", str(tmp_path), "--tps", "1,2", "--model", "tiny-tp8", "--device",
                    "cpu", "--dtype", "fp32", "--max-tokens", "6", "--max-model-len", "256", "--block-size", "16",
                    "--num-blocks", "32"])
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["1"]["matches_tp1"] and out["2"]["matches_tp1"]
    assert abs(out["2"]["kv_block_shard_ratio"] - 1.0) < 1e-9
