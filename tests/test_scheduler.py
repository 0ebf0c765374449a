"""Scheduler: decode-first, chunked prefill, FIFO admission, finish rules, abort, preemption."""
from nanovllm_self_b200.config import EngineConfig
from nanovllm_self_b200.engine.block_manager import BlockManager
from nanovllm_self_b200.engine.scheduler import Scheduler
from nanovllm_self_b200.engine.sequence import Sequence, SequenceStatus
from nanovllm_self_b200.sampling_params import SamplingParams


def _mk(**kw):
    base = dict(device="cpu", block_size=4, max_num_seqs=8, max_num_batched_tokens=64, num_blocks=32)
    base.update(kw)
    cfg = EngineConfig(**base)
    return cfg, Scheduler(cfg, BlockManager(cfg.num_blocks, cfg.block_size))


def _seq(i, n, max_tokens=4, **kw):
    return Sequence(i, list(range(100 * i, 100 * i + n)), SamplingParams(max_tokens=max_tokens, ignore_eos=True, **kw),
                    block_size=4)


def _fake_step(sch, seqs, tok=7):
    need = [i for i, s in enumerate(seqs) if s.is_need_logits]
    return sch.postprocess(seqs, [tok] * len(need), need)


def test_prefill_then_decode_first():
    cfg, sch = _mk()
    a, b = _seq(1, 6), _seq(2, 5)
    sch.add(a)
    sch.add(b)
    out = sch.schedule()
    assert out == [a, b] and a.num_new_tokens == 6
    _fake_step(sch, out)
    assert a.num_completion_tokens == 1 and a.is_prefill_done
    c = _seq(3, 3)
    sch.add(c)
    out = sch.schedule()
    assert out[:2] == [a, b] and out[2] is c  # decode first, then admission
    assert sch.last_schedule_info.num_decode_tokens == 2


def test_chunked_prefill_samples_only_on_last_chunk():
    cfg, sch = _mk(enable_chunked_prefill=True, prefill_chunk_size=4)
    a = _seq(1, 10)
    sch.add(a)
    sizes = []
    while not a.is_prefill_done:
        out = sch.schedule()
        sizes.append(a.num_new_tokens)
        need = [i for i, s in enumerate(out) if s.is_need_logits]
        if a.num_context_tokens < 10:
            assert need == []
        _fake_step(sch, out)
    assert sizes == [4, 4, 2] and a.num_completion_tokens == 1


def test_token_budget_and_fifo_admission_stops():
    cfg, sch = _mk(max_num_batched_tokens=10)
    a, b = _seq(1, 8), _seq(2, 8)
    sch.add(a)
    sch.add(b)
    out = sch.schedule()
    assert out == [a, b] and b.num_new_tokens == 2  # budget caps the second prompt
    cfg, sch = _mk(num_blocks=3)
    a, b = _seq(1, 8), _seq(2, 8)
    sch.add(a)
    sch.add(b)
    out = sch.schedule()
    assert out == [a] and sch.last_schedule_info.blocked_prefill == 1


def test_finish_on_max_tokens_and_eos():
    cfg, sch = _mk()
    a = _seq(1, 3, max_tokens=2)
    sch.add(a)
    _fake_step(sch, sch.schedule())
    fin = _fake_step(sch, sch.schedule())
    assert fin == [a] and a.status == SequenceStatus.FINISHED and a.block_table == []
    assert sch.is_finished()
    cfg, sch = _mk(eos=7)
    b = Sequence(5, [1, 2, 3], SamplingParams(max_tokens=10), block_size=4)
    sch.add(b)
    fin = _fake_step(sch, sch.schedule(), tok=7)
    assert fin == [b] and b.finish_reason == "stop"


def test_abort():
    cfg, sch = _mk()
    a, b = _seq(1, 3), _seq(2, 3)
    sch.add(a)
    sch.add(b)
    sch.schedule()
    assert sch.abort_by_seq_idx(1)
    assert a.status == SequenceStatus.FINISHED and a.block_table == []
    assert not sch.abort_by_seq_idx(99)


def test_preemption_frees_blocks_and_recomputes():
    cfg, sch = _mk(num_blocks=4, max_num_batched_tokens=64)
    a, b = _seq(1, 8, max_tokens=8), _seq(2, 7, max_tokens=8)
    sch.add(a)
    sch.add(b)
    for _ in range(20):
        if sch.is_finished():
            break
        out = sch.schedule()
        assert out, sch.last_schedule_info.reason
        _fake_step(sch, out)
    assert sch.is_finished()
    assert sch.num_preemptions >= 1
    assert a.num_completion_tokens == 8 and b.num_completion_tokens == 8


def test_no_preemption_reports_blocked():
    cfg, sch = _mk(num_blocks=4, enable_preemption=False)
    a, b = _seq(1, 8, max_tokens=8), _seq(2, 7, max_tokens=8)
    sch.add(a)
    sch.add(b)
    reasons = set()
    for _ in range(12):
        out = sch.schedule()
        reasons.add(sch.last_schedule_info.reason)
        if out:
            _fake_step(sch, out)
    assert "blocked_by_blocks" in reasons
