"""A seeded engine trace for block managers, and a minimal sequence type.

``run_trace`` drives a block manager the way the reference scheduler does
(``microinfer/engine/scheduler.py:113-253``: ``can_allocate`` then ``allocate``
and a whole-prompt prefill, ``can_append`` / ``may_append`` before every decode
step, ``hash_blocks`` after every step, ``deallocate`` on finish or when a
sequence cannot get its next page) over prompts built from a few shared prefixes,
so prefix-cache hits, LRU reuse of released pages and evictions all happen.  It
records, after every operation, what the manager returned, the sequence's block
table, a digest of the sorted free pages and ``stats()``.

``make_block_golden.py`` ran it on the reference ``BlockManager`` with the
reference ``Sequence`` (block size patched to 4) and stored the records;
``tests/test_block_manager.py`` replays it on ``CowBlockManager`` with
``TraceSequence`` and compares every record.
"""
from __future__ import annotations

import hashlib

import numpy as np


class TraceSequence:
    """The fields and methods a block manager uses, with the reference
    ``Sequence``'s meaning (``microinfer/engine/sequence.py``)."""

    block_size = 4

    def __init__(self, token_ids):
        self.token_ids = list(token_ids)
        self.num_tokens = len(self.token_ids)
        self.num_cached_tokens = 0
        self.num_scheduled_tokens = 0
        self.block_table: list[int] = []

    def __len__(self):
        return self.num_tokens

    @property
    def num_blocks(self):
        return (self.num_tokens + self.block_size - 1) // self.block_size

    def block(self, i):
        assert 0 <= i < self.num_blocks
        return self.token_ids[i * self.block_size:(i + 1) * self.block_size]

    def append_token(self, token_id: int):
        self.token_ids.append(token_id)
        self.num_tokens += 1


# the stats() entries a record keeps (num_blocks and kv_utilization follow from them)
STATS = ("used_blocks", "free_blocks", "prefix_cache_entries", "prefix_cache_hit_tokens",
         "prefix_cache_hit_blocks", "prefix_cache_evictions")


def run_trace(manager, make_seq, seed: int = 0, steps: int = 400):
    """Records ``[op, result, block table, free-page digest, stats]`` per operation."""
    rng = np.random.default_rng(seed)
    prefixes = [[int(t) for t in rng.integers(1, 50, int(n))] for n in (9, 13, 6)]
    running = []
    records = []

    def rec(op, result, seq=None):
        free = ",".join(map(str, sorted(manager.free_block_ids)))
        st = manager.stats()
        records.append([op, result, list(seq.block_table) if seq is not None else None,
                        hashlib.sha1(free.encode()).hexdigest()[:12],
                        [st[k] for k in STATS]])

    for _ in range(steps):
        r = rng.random()
        if r < 0.25 or not running:  # admit a request (whole prompt in one prefill)
            base = prefixes[int(rng.integers(0, len(prefixes)))]
            keep = int(rng.integers(len(base) // 2, len(base) + 1))
            prompt = base[:keep] + [int(t) for t in rng.integers(50, 90, int(rng.integers(0, 7)))]
            seq = make_seq(prompt)
            reused = manager.can_allocate(seq)
            rec("can_allocate", reused, seq)
            if reused < 0:
                continue
            manager.allocate(seq, reused)
            rec("allocate", seq.num_cached_tokens, seq)
            seq.num_scheduled_tokens = seq.num_tokens - seq.num_cached_tokens
            manager.hash_blocks(seq)
            seq.num_cached_tokens += seq.num_scheduled_tokens
            seq.num_scheduled_tokens = 0
            seq.append_token(int(rng.integers(1, 90)))
            rec("prefill", None, seq)
            running.append(seq)
        elif r < 0.9:  # one decode step of a running sequence
            seq = running[int(rng.integers(0, len(running)))]
            if not manager.can_append(seq):
                manager.deallocate(seq)
                running.remove(seq)
                rec("preempt", None, seq)
                continue
            seq.num_scheduled_tokens = 1
            manager.may_append(seq)
            rec("may_append", None, seq)
            manager.hash_blocks(seq)
            seq.num_cached_tokens += 1
            seq.num_scheduled_tokens = 0
            seq.append_token(int(rng.integers(1, 90)))
            rec("decode", None, seq)
        else:  # a sequence finishes
            seq = running.pop(int(rng.integers(0, len(running))))
            manager.deallocate(seq)
            rec("finish", None, seq)
    return records
