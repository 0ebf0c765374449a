"""P/D disaggregation on CPU (tiny fp32 model): handoff contract, P/D == monolithic, online
coordinator streaming/abort/metrics, stores (dict / shared memory), restore failure cleanup."""
import pytest
import torch

from nanovllm_self_b200 import LLM, SamplingParams
from nanovllm_self_b200.config import EngineConfig
from nanovllm_self_b200.pd.coordinator import PDCoordinator
from nanovllm_self_b200.pd.kv_store import KVStoreItem, SharedMemoryKVStoreBackend
from nanovllm_self_b200.pd.online_coordinator import OnlinePDCoordinator
from nanovllm_self_b200.pd.request_state import RequestStatus


def _cfg(**kw):
    base = dict(model="tiny", device="cpu", dtype="fp32", block_size=16, max_model_len=256, num_blocks=64)
    base.update(kw)
    return EngineConfig(**base)


def _prompts():
    g = torch.Generator().manual_seed(11)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (5, 16, 33, 47)]


@pytest.mark.parametrize("backend", ["dict", "shared_memory"])
def test_pd_equals_monolithic(backend):
    ref = LLM("tiny", **{k: v for k, v in _cfg().__dict__.items() if k in ("device", "dtype", "block_size",
                                                                               "max_model_len", "num_blocks")})
    want = ref.generate(_prompts(), SamplingParams(temperature=0, max_tokens=10, ignore_eos=True))
    pd = PDCoordinator(_cfg(), kv_backend=backend)
    got = pd.generate(_prompts(), max_tokens=10, temperature=0.0)
    assert got == want


def test_handoff_payload_contract():
    pd = PDCoordinator(_cfg())
    p = _prompts()[2]
    payloads = pd.prefill_engine.run_prefill([p], max_tokens=5)
    (pl,) = payloads
    assert pl.token_ids[:len(p)] == p and len(pl.token_ids) == len(p) + 1
    assert pl.num_cached_tokens == len(p) and pl.num_prompt_tokens == len(p)
    assert not pl.finished and pl.transfer_meta.num_kv_blocks == (len(p) + 15) // 16
    assert pl.transfer_meta.last_block_num_tokens == len(p) % 16 or 16
    assert pd.prefill_runner.block_manager.num_used_blocks() == 0  # prefill blocks released
    (fin,) = pd.prefill_engine.run_prefill([p], max_tokens=1, start_seq_id=9)
    assert fin.finished and fin.transfer_meta is None


def test_online_stream_abort_and_metrics():
    oc = OnlinePDCoordinator(_cfg())
    prompts = _prompts()
    r0 = oc.submit(prompts[0], max_tokens=6)
    r1 = oc.submit(prompts[1], max_tokens=50)
    with pytest.raises(ValueError):
        oc.submit(prompts[0], request_id=r0)
    evs = list(oc.stream(r0))
    assert evs[-1].finished and sum(e.token_id is not None for e in evs) == 6
    assert oc.abort_request(r1)
    assert oc.requests[r1].status == RequestStatus.ABORTED
    assert oc.decode_runner.block_manager.num_used_blocks() == 0
    oc.step()  # metrics are recorded per step
    m = oc.get_last_online_scheduler_metrics()
    assert m is not None and m.finished_requests == 1 and m.aborted_requests == 1
    # staggered arrivals still produce the offline tokens
    want = PDCoordinator(_cfg()).generate(prompts, max_tokens=7)
    oc2 = OnlinePDCoordinator(_cfg())
    rids = [oc2.submit(prompts[0], max_tokens=7)]
    oc2.step()
    rids += [oc2.submit(p, max_tokens=7) for p in prompts[1:]]
    while oc2.has_unfinished():
        oc2.step()
    assert [oc2.requests[r].token_ids for r in rids] == want
    assert oc2.request_metrics()["ttft_ms_p50"] > 0


def test_shared_memory_store_roundtrip_bf16_is_not_upcast():
    b = SharedMemoryKVStoreBackend()
    kv = torch.randn(2, 3, 4, 2, 16, 8).bfloat16()
    stored = b.put("h1", KVStoreItem(kv, None, 40, 4, 8))
    assert stored.storage_ref.nbytes == kv.numel() * 2
    back = b.pop("h1")
    assert torch.equal(back.kv_blocks, kv)
    assert not b.exists("h1")


def test_decode_restore_failure_frees_blocks():
    pd = PDCoordinator(_cfg())
    (pl,) = pd.prefill_engine.run_prefill([_prompts()[3]], max_tokens=5)
    pd.consumer.kv_store_backend.delete(pl.transfer_meta.handoff_id)  # drop the KV: restore must fail
    used = pd.decode_runner.block_manager.num_used_blocks()
    with pytest.raises(KeyError):
        pd.decode_engine.restore_sequence(pl)
    assert pd.decode_runner.block_manager.num_used_blocks() == used


def test_error_marks_active_requests():
    oc = OnlinePDCoordinator(_cfg())
    rid = oc.submit(_prompts()[1], max_tokens=20)
    oc.step()

    def boom(*a, **k):
        raise RuntimeError("injected decode failure")
    oc.decode_engine.continuous_step = boom
    with pytest.raises(RuntimeError):
        oc.step()
    assert oc.requests[rid].status == RequestStatus.ERROR
    assert oc.requests[rid].stream_queue.queue[-1].error == "injected decode failure"
