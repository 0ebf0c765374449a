"""Host-side paged-KV block manager with prefix-hash reuse and a session prefix cache.

It holds no tensors: it hands out physical block ids that index the KV pool owned by
the model runner.  Semantics follow the reference ``block_manager``
(``nanovllm/engine/block_manager.py:50-401``):

* **Chained block hash** over *full* blocks only: xxh64 over the 8-byte little-endian
  previous-block hash (omitted for the first block) followed by each token id as a
  4-byte little-endian integer (reference ``compute_hash`` :294-305).  The byte format
  is kept identical so a hash computed by either implementation names the same block.
* **Prefix reuse** walks the prompt block by block; a block is reused only on a hash hit
  *and* exact token equality; after the first miss every later block is fresh
  (reference :364-397).  ``num_cached_tokens`` advances by ``block_size`` per hit.
* **Decode growth**: ``can_append``/``may_append`` allocate when ``len % bs == 1`` and
  seal the hash of a block when it becomes full (``len % bs == 0``) (reference :163-196).
* **Session prefix cache**: on finish/handoff the full blocks up to
  ``min(cached + new, len - 1)`` are pinned with one extra reference under
  ``session_id``; an older entry for the same session is released (reference :93-136).
  ``allocate`` checks the session entry first, then the hash chain (reference :335-358).

One deliberate improvement: a block whose reference count drops to zero keeps its hash
and goes to the *back* of the free queue, so a later request with the same prefix can
still hit it until the block is actually reused (least-recently-freed eviction).  The
reference un-hashes a block as soon as it is freed, so its reuse needs a live holder.
Set ``retain_freed_hashes=False`` to get the reference's behaviour exactly.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass

import numpy as np

try:  # xxhash is the reference's hash; fall back to the in-repo implementation.
    import xxhash as _xxhash
except ImportError:  # pragma: no cover - exercised only on images without xxhash
    _xxhash = None

from ..utils.hashing import xxh64_bytes
from .sequence import Sequence


def compute_block_hash(token_ids, prev_hash: int = -1) -> int:
    """xxh64(prev_hash as u64 LE [if != -1] ++ tokens as u32 LE)."""
    payload = np.asarray(token_ids, dtype="<u4").tobytes()
    if prev_hash != -1:
        payload = int(prev_hash).to_bytes(8, "little") + payload
    if _xxhash is not None:
        return _xxhash.xxh64_intdigest(payload)
    return xxh64_bytes(payload)


@dataclass
class SessionPrefixCacheEntry:
    token_ids: list
    block_ids: list
    num_cached_tokens: int


class Block:
    __slots__ = ("block_id", "block_size", "ref_count", "hash", "token_ids", "prev_hash")

    def __init__(self, block_id: int, block_size: int):
        self.block_id = block_id
        self.block_size = block_size
        self.ref_count = 0
        self.hash = -1
        self.token_ids: tuple = ()
        self.prev_hash = -1

    def update(self, h: int, token_ids, prev_hash: int) -> None:
        self.hash = h
        self.token_ids = tuple(token_ids)
        self.prev_hash = prev_hash

    def reset(self) -> None:
        self.ref_count = 0
        self.hash = -1
        self.token_ids = ()
        self.prev_hash = -1


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, enable_prefix_cache: bool = True,
                 retain_freed_hashes: bool = True):
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.enable_prefix_cache = enable_prefix_cache
        self.retain_freed_hashes = retain_freed_hashes and enable_prefix_cache
        self.blocks = [Block(i, block_size) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        # Insertion-ordered free set: allocation pops the oldest entry.
        self.free_blocks_idx: OrderedDict[int, None] = OrderedDict((i, None) for i in range(num_blocks))
        self.used_blocks_idx: set[int] = set()
        self.session_prefix_cache: dict[str, SessionPrefixCacheEntry] = {}
        # Counters for observability.
        self.num_prefix_hit_blocks = 0
        self.num_prefix_query_blocks = 0

    # ------------------------------------------------------------------ hashing
    @staticmethod
    def compute_hash(token_ids, prev_hash: int = -1) -> int:
        return compute_block_hash(token_ids, prev_hash)

    # ------------------------------------------------------------- observability
    def num_free_blocks(self) -> int:
        return len(self.free_blocks_idx)

    def num_used_blocks(self) -> int:
        return len(self.used_blocks_idx)

    def get_block_usage_snapshot(self) -> dict:
        return {
            "total_blocks": self.num_blocks,
            "used_blocks": self.num_used_blocks(),
            "free_blocks": self.num_free_blocks(),
            "cached_hashes": len(self.hash_to_block_id),
            "session_entries": len(self.session_prefix_cache),
            "prefix_hit_blocks": self.num_prefix_hit_blocks,
            "prefix_query_blocks": self.num_prefix_query_blocks,
        }

    # ---------------------------------------------------------- raw allocation
    def _take_free(self, block_id: int | None = None) -> int:
        if block_id is None:
            block_id, _ = self.free_blocks_idx.popitem(last=False)
        else:
            del self.free_blocks_idx[block_id]
        blk = self.blocks[block_id]
        if blk.ref_count == 0 and blk.hash != -1:
            # Evict the stale cached content of a block that is about to be rewritten.
            if self.hash_to_block_id.get(blk.hash) == block_id:
                del self.hash_to_block_id[blk.hash]
            blk.reset()
        self.used_blocks_idx.add(block_id)
        blk.ref_count = 1
        return block_id

    def allocate_block(self, num_blocks: int) -> list[int]:
        """Allocate ``num_blocks`` fresh blocks (ref 1, no hash)."""
        if num_blocks > len(self.free_blocks_idx):
            raise RuntimeError(f"out of KV blocks: need {num_blocks}, have {len(self.free_blocks_idx)}")
        return [self._take_free() for _ in range(num_blocks)]

    def _revive(self, block_id: int) -> None:
        """Take a reference on a block found in the hash map (possibly free)."""
        blk = self.blocks[block_id]
        if blk.ref_count == 0:
            del self.free_blocks_idx[block_id]
            self.used_blocks_idx.add(block_id)
        blk.ref_count += 1

    def free_blocks(self, block_ids) -> None:
        for idx in block_ids:
            if not (0 <= idx < self.num_blocks):
                raise AssertionError(f"block id {idx} out of range")
            if idx not in self.used_blocks_idx:
                raise AssertionError(f"block {idx} is not in use")
            blk = self.blocks[idx]
            blk.ref_count -= 1
            if blk.ref_count == 0:
                self.used_blocks_idx.discard(idx)
                if self.retain_freed_hashes and blk.hash != -1:
                    self.free_blocks_idx[idx] = None  # back of the queue: evicted last
                else:
                    if blk.hash != -1 and self.hash_to_block_id.get(blk.hash) == idx:
                        del self.hash_to_block_id[blk.hash]
                    blk.reset()
                    self.free_blocks_idx[idx] = None
                    self.free_blocks_idx.move_to_end(idx, last=False)  # reused first

    # ------------------------------------------------------------- sequences
    def can_allocate(self, seq: Sequence) -> bool:
        return (len(seq) + self.block_size - 1) // self.block_size <= len(self.free_blocks_idx)

    def can_append(self, seq: Sequence) -> bool:
        if len(seq) % self.block_size == 1:
            return len(self.free_blocks_idx) >= 1
        return True

    def may_append(self, seq: Sequence) -> None:
        bs = self.block_size
        n = len(seq)
        if n % bs == 1:
            new_id = self._take_free()
            if seq.block_table:
                self.blocks[new_id].prev_hash = self.blocks[seq.block_table[-1]].hash
            seq.block_table.append(new_id)
        elif n % bs == 0 and self.enable_prefix_cache:
            last_id = seq.block_table[-1]
            toks = seq.token_ids[-bs:]
            prefix = self.blocks[seq.block_table[-2]].hash if len(seq.block_table) > 1 else -1
            h = self.compute_hash(toks, prefix)
            self.blocks[last_id].update(h, toks, prefix)
            self.hash_to_block_id.setdefault(h, last_id)

    def allocate(self, seq: Sequence) -> list[int]:
        return self.allocate_with_prefill(seq)

    def allocate_with_prefill(self, seq: Sequence) -> list[int]:
        seq.prefix_cache_hit = False
        seq.prefix_cached_tokens = 0
        seq.prefix_new_tokens = seq.num_prompt_tokens
        seq.prefix_cache_source = None
        bs = self.block_size
        token_ids = seq.token_ids
        physical: list[int] = []
        prev_hash = -1
        start = 0
        seq.num_cached_tokens = 0

        sid = seq.session_id
        if sid and self.enable_prefix_cache:
            entry = self.session_prefix_cache.get(sid)
            # Never let the cache cover the whole prompt: the last prompt token must be
            # recomputed to produce logits.
            if (entry is not None and entry.num_cached_tokens < len(token_ids)
                    and token_ids[:entry.num_cached_tokens] == entry.token_ids):
                for b in entry.block_ids:
                    self._revive(b)
                physical.extend(entry.block_ids)
                seq.num_cached_tokens = entry.num_cached_tokens
                start = entry.num_cached_tokens
                seq.prefix_cache_hit = entry.num_cached_tokens > 0
                seq.prefix_cached_tokens = entry.num_cached_tokens
                seq.prefix_new_tokens = max(0, seq.num_prompt_tokens - entry.num_cached_tokens)
                seq.prefix_cache_source = "session_local"
                if entry.block_ids:
                    prev_hash = self.blocks[entry.block_ids[-1]].hash

        cache_miss = not self.enable_prefix_cache
        n = len(token_ids)
        for i in range(start, n, bs):
            blk_tokens = token_ids[i:i + bs]
            is_full = len(blk_tokens) == bs
            # The block holding the last prompt token is always recomputed so the step
            # produces logits for it.
            reusable = is_full and i + bs < n
            h = self.compute_hash(blk_tokens, prev_hash) if is_full else -1
            if not cache_miss:
                self.num_prefix_query_blocks += 1
                bid = self.hash_to_block_id.get(h, -1) if reusable else -1
                if bid == -1 or self.blocks[bid].token_ids != tuple(blk_tokens):
                    cache_miss = True
            if cache_miss:
                nid = self._take_free()
                physical.append(nid)
                blk = self.blocks[nid]
                if is_full:
                    blk.update(h, blk_tokens, prev_hash)
                    if self.enable_prefix_cache:
                        self.hash_to_block_id.setdefault(h, nid)
                else:
                    blk.prev_hash = prev_hash
            else:
                self._revive(bid)
                physical.append(bid)
                seq.num_cached_tokens += bs
                self.num_prefix_hit_blocks += 1
                if seq.prefix_cache_source is None:
                    seq.prefix_cache_source = "hash"
                seq.prefix_cache_hit = True
            if is_full:
                prev_hash = h
        seq.prefix_cached_tokens = seq.num_cached_tokens
        seq.prefix_new_tokens = seq.num_prompt_tokens - seq.num_cached_tokens
        seq.block_table = physical
        return physical

    def deallocate(self, seq: Sequence) -> None:
        if not seq.block_table:
            return
        self.free_blocks(seq.block_table)
        seq.block_table = []
        seq.num_cached_tokens = 0

    # ------------------------------------------------------- session cache
    def _release_session_prefix_cache(self, session_id: str) -> None:
        old = self.session_prefix_cache.pop(session_id, None)
        if old is not None:
            self.free_blocks(old.block_ids)

    def release_session(self, session_id: str) -> None:
        self._release_session_prefix_cache(session_id)

    def save_session_prefix_cache(self, session_id: str, seq: Sequence) -> None:
        if not session_id or not self.enable_prefix_cache:
            return
        num_cached = min(seq.num_cached_tokens + seq.num_new_tokens, max(0, len(seq.token_ids) - 1))
        full = num_cached // self.block_size
        if full <= 0:
            return
        cached = full * self.block_size
        block_ids = list(seq.block_table[:full])
        token_ids = list(seq.token_ids[:cached])
        # Take the new references before dropping the old entry so shared blocks survive.
        for b in block_ids:
            self.blocks[b].ref_count += 1
        self._release_session_prefix_cache(session_id)
        self.session_prefix_cache[session_id] = SessionPrefixCacheEntry(token_ids, block_ids, cached)

    def register_full_blocks(self, seq: Sequence, num_tokens: int) -> None:
        """Hash-register the full blocks covering ``seq.token_ids[:num_tokens]``.

        Used after importing KV that was produced elsewhere (P/D handoff), so the
        decode side can serve later prefix hits (reference
        ``pd_self/decode_engine.py:_restore_block_manager_meta``).
        """
        if not self.enable_prefix_cache:
            return
        bs = self.block_size
        prev = -1
        for j in range(num_tokens // bs):
            toks = seq.token_ids[j * bs:(j + 1) * bs]
            h = self.compute_hash(toks, prev)
            bid = seq.block_table[j]
            self.blocks[bid].update(h, toks, prev)
            self.hash_to_block_id.setdefault(h, bid)
            prev = h


# Name kept for users of the reference (``nanovllm.engine.block_manager.block_manager``).
block_manager = BlockManager
