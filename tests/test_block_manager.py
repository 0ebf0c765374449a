"""Block manager: hash format, prefix reuse, decode growth, session cache, ref counts."""
import xxhash

from nanovllm_self_b200.engine.block_manager import BlockManager, compute_block_hash
from nanovllm_self_b200.engine.sequence import Sequence
from nanovllm_self_b200.sampling_params import SamplingParams


def _ref_hash(tokens, prev=-1):
    h = xxhash.xxh64()
    if prev != -1:
        h.update(prev.to_bytes(8, "little"))
    for t in tokens:
        h.update(int(t).to_bytes(4, "little"))
    return h.intdigest()


def test_hash_byte_format_matches_streaming_xxh64():
    toks = list(range(100, 116))
    h0 = compute_block_hash(toks)
    assert h0 == _ref_hash(toks)
    assert compute_block_hash(toks, h0) == _ref_hash(toks, h0)


def test_allocate_and_prefix_reuse():
    bm = BlockManager(16, 4)
    a = Sequence(0, list(range(10)), block_size=4)
    bm.allocate(a)
    assert len(a.block_table) == 3 and a.num_cached_tokens == 0
    b = Sequence(1, list(range(10)), block_size=4)
    bm.allocate(b)
    # two full blocks shared, last (partial) block fresh
    assert b.block_table[:2] == a.block_table[:2]
    assert b.block_table[2] != a.block_table[2]
    assert b.num_cached_tokens == 8 and b.prefix_cache_hit
    assert bm.blocks[a.block_table[0]].ref_count == 2
    # after the first miss every later block is fresh
    c = Sequence(2, [0, 1, 2, 3, 99, 5, 6, 7, 8, 9, 10], block_size=4)
    bm.allocate(c)
    assert c.block_table[0] == a.block_table[0]
    assert c.block_table[1] != a.block_table[1]
    assert c.num_cached_tokens == 4


def test_block_with_last_prompt_token_is_recomputed():
    bm = BlockManager(16, 4)
    a = Sequence(0, list(range(8)), block_size=4)
    bm.allocate(a)
    b = Sequence(1, list(range(8)), block_size=4)
    bm.allocate(b)
    assert b.num_cached_tokens == 4  # not 8: the last block must produce logits
    assert not b.is_prefill_done


def test_free_and_ref_counts_and_retained_hash():
    bm = BlockManager(8, 4)
    a = Sequence(0, list(range(9)), block_size=4)
    bm.allocate(a)
    used = list(a.block_table)
    bm.deallocate(a)
    assert bm.num_free_blocks() == 8 and a.block_table == []
    # freed-but-hashed blocks still serve a later identical prefix
    b = Sequence(1, list(range(9)), block_size=4)
    bm.allocate(b)
    assert b.block_table[:2] == used[:2] and b.num_cached_tokens == 8


def test_reference_eviction_mode():
    bm = BlockManager(8, 4, retain_freed_hashes=False)
    a = Sequence(0, list(range(9)), block_size=4)
    bm.allocate(a)
    bm.deallocate(a)
    b = Sequence(1, list(range(9)), block_size=4)
    bm.allocate(b)
    assert b.num_cached_tokens == 0


def test_decode_growth_and_sealing():
    bm = BlockManager(8, 4)
    s = Sequence(0, [1, 2, 3], block_size=4)
    bm.allocate(s)
    assert len(s.block_table) == 1
    s.append_token(4)  # len 4: fills the block -> sealed
    assert bm.can_append(s)
    bm.may_append(s)
    blk = bm.blocks[s.block_table[0]]
    assert blk.hash == compute_block_hash([1, 2, 3, 4])
    s.append_token(5)  # len 5: needs a new block
    bm.may_append(s)
    assert len(s.block_table) == 2
    assert bm.blocks[s.block_table[1]].prev_hash == blk.hash


def test_can_allocate_and_can_append_limits():
    bm = BlockManager(2, 4)
    s = Sequence(0, list(range(9)), block_size=4)
    assert not bm.can_allocate(s)
    t = Sequence(1, list(range(8)), block_size=4)
    assert bm.can_allocate(t)
    bm.allocate(t)
    t.append_token(1)
    assert not bm.can_append(t)


def test_session_prefix_cache():
    bm = BlockManager(16, 4)
    s = Sequence(0, list(range(10)), SamplingParams(max_tokens=2), block_size=4, session_id="sess")
    bm.allocate(s)
    s.num_cached_tokens, s.num_new_tokens = 0, 10
    s.append_token(50)
    bm.save_session_prefix_cache("sess", s)
    entry = bm.session_prefix_cache["sess"]
    assert entry.num_cached_tokens == 8 and entry.block_ids == s.block_table[:2]
    bm.deallocate(s)
    assert bm.blocks[entry.block_ids[0]].ref_count == 1  # pinned by the session
    nxt = Sequence(1, list(range(10)) + [50, 7, 8], block_size=4, session_id="sess")
    bm.allocate(nxt)
    assert nxt.prefix_cache_source == "session_local" and nxt.num_cached_tokens >= 8
    bm.release_session("sess")
    assert bm.blocks[entry.block_ids[0]].ref_count == 1  # still held by nxt
    bm.deallocate(nxt)
    assert bm.num_used_blocks() == 0


def test_usage_snapshot():
    bm = BlockManager(4, 4)
    snap = bm.get_block_usage_snapshot()
    assert snap["total_blocks"] == 4 and snap["free_blocks"] == 4 and snap["used_blocks"] == 0
