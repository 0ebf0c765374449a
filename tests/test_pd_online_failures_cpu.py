"""Online P/D coordinator under host-side faults and overload, on CPU (tiny fp32 model).

Aborts in the middle of a chunked prefill and in the middle of decode free every block on both
sides and leave the other requests' tokens unchanged; an overloaded pool (more requests than KV
blocks) queues and finishes every request with the tokens it would have produced alone; an
admission check that fails rolls the request back.
"""
import pytest
import torch

from nanovllm_self_b200.config import EngineConfig
from nanovllm_self_b200.pd.coordinator import PDCoordinator
from nanovllm_self_b200.pd.online_coordinator import OnlinePDCoordinator
from nanovllm_self_b200.pd.request_state import RequestStatus


def _cfg(**kw):
    base = dict(model="tiny", device="cpu", dtype="fp32", block_size=16, max_model_len=256, num_blocks=64)
    base.update(kw)
    return EngineConfig(**base)


def _prompt(n, seed):
    return torch.randint(0, 1024, (n,), generator=torch.Generator().manual_seed(seed)).tolist()


def _alone(prompt, max_tokens, **kw):
    return PDCoordinator(_cfg(**kw)).generate([prompt], max_tokens=max_tokens)[0]


def _used(oc):
    return (oc.prefill_runner.block_manager.num_used_blocks(), oc.decode_runner.block_manager.num_used_blocks())


def test_abort_mid_prefill_frees_blocks_and_spares_others():
    kw = dict(enable_chunked_prefill=True, prefill_chunk_size=16, max_num_batched_tokens=32)
    oc = OnlinePDCoordinator(_cfg(**kw))
    long_p, short_p = _prompt(120, 1), _prompt(20, 2)
    victim = oc.submit(long_p, max_tokens=8)
    other = oc.submit(short_p, max_tokens=8)
    oc.step()
    assert oc.requests[victim].status == RequestStatus.PREFILLING and not oc.requests[victim].output_ids
    assert _used(oc)[0] > 0
    assert oc.abort_request(victim)
    assert oc.requests[victim].status == RequestStatus.ABORTED
    assert not oc.abort_request(victim)  # a second abort is a no-op
    while oc.has_unfinished():
        oc.step()
    assert oc.requests[other].status == RequestStatus.FINISHED
    assert oc.requests[other].token_ids == _alone(short_p, 8, **kw)
    assert not oc.requests[victim].output_ids
    assert _used(oc) == (0, 0)


def test_abort_mid_decode_stops_events_and_frees_blocks():
    oc = OnlinePDCoordinator(_cfg())
    a_p, b_p = _prompt(30, 3), _prompt(45, 4)
    victim = oc.submit(a_p, max_tokens=40)
    other = oc.submit(b_p, max_tokens=12)
    while len(oc.requests[victim].output_ids) < 4:
        oc.step()
    assert oc.requests[victim].status == RequestStatus.DECODING
    n_before = len(oc.requests[victim].output_ids)
    assert oc.abort_request(victim, reason="client went away")
    while oc.has_unfinished():
        oc.step()
    st = oc.requests[victim]
    assert st.status == RequestStatus.ABORTED and len(st.output_ids) == n_before
    assert st.token_ids == _alone(a_p, 40)[:len(a_p) + n_before]
    assert oc.requests[other].token_ids == _alone(b_p, 12)
    assert _used(oc) == (0, 0)
    assert oc.get_last_online_scheduler_metrics().aborted_requests == 1


def test_overload_queues_and_finishes_every_request():
    # 16 blocks of 16 tokens on each side; 10 requests of about 70 tokens need about 50 blocks
    kw = dict(num_blocks=16)
    prompts = [_prompt(40 + 3 * i, 10 + i) for i in range(10)]
    oc = OnlinePDCoordinator(_cfg(**kw))
    rids = [oc.submit(p, max_tokens=24) for p in prompts]
    steps = 0
    while oc.has_unfinished():
        oc.step()
        steps += 1
        assert steps < 5000
    assert all(oc.requests[r].status == RequestStatus.FINISHED for r in rids)
    for r, p in zip(rids, prompts):
        assert oc.requests[r].token_ids == _alone(p, 24, **kw)
    assert _used(oc) == (0, 0)
    assert max(m.waiting_prefill_requests for m in oc.metrics_history) > 0  # requests did queue


def test_admission_check_rolls_back_an_overloaded_submit():
    oc = OnlinePDCoordinator(_cfg(num_blocks=4))
    ok = oc.submit(_prompt(40, 5), max_tokens=4, check_admission=True)
    with pytest.raises(RuntimeError, match="overloaded"):
        oc.submit(_prompt(70, 6), max_tokens=4, request_id="too-big", check_admission=True)  # 5 blocks > 4
    assert "too-big" not in oc.requests and list(oc.requests) == [ok]
    while oc.has_unfinished():
        oc.step()
    assert oc.requests[ok].status == RequestStatus.FINISHED
