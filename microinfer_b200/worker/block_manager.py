"""Host-side page allocator: the engine's prefix-caching block manager plus copy-on-write.

``CowBlockManager`` is a drop-in for the reference ``BlockManager``
(``microinfer/engine/blockmanager.py:27-242``) as the scheduler drives it
(``can_allocate`` / ``allocate`` before a prefill, ``can_append`` /
``may_append`` before a decode step, ``hash_blocks`` after a step,
``deallocate`` / ``trim`` on finish, preemption and speculative rollback,
``stats``).  Its prefix cache follows the reference's rules:

* every full page is keyed by a chained 64-bit xxHash of its token ids and the
  key of the page before it; a lookup also compares the token ids, so a hash
  collision never maps foreign tokens into a sequence;
* ``can_allocate`` walks a new sequence's full pages (never the last one, which
  may be partial) until the first miss, returns how many are reusable (or -1 if
  the pool cannot hold the rest) and refreshes the hits' LRU time;
* released pages keep their tokens and keys until they are handed out again;
  free pages are handed out least recently used first (a lazy heap of
  ``(last_used, page)`` entries, stale entries skipped), and reusing a page that
  still held a cached prefix counts as an eviction.

On top of that, pages may be shared *including a partial last page*
(``fork``: parallel sampling or beam search); the reference never shares one, so
it never needs a copy.  A sequence about to write into a page that another
sequence still references gets a private copy first (``may_append`` for the
scheduler's convention, ``prepare_append`` for a caller that wants the next
token's slot): a fresh page is taken, ``(old, new)`` is queued, and the old
page stays pinned (neither freed nor handed out) until the queued copies are
taken by ``take_copies``.  ``apply_copies`` issues them on the device as one
``KVCache.copy_blocks`` launch (every layer, K and V) before the step's
``store_kvcache``, which is the order the pins rely on.

Sequences are the reference's ``Sequence`` objects (or anything with
``token_ids``, ``num_tokens``, ``num_blocks``, ``block(i)``, ``block_table``,
``num_cached_tokens`` and ``num_scheduled_tokens``).
"""
from __future__ import annotations

import heapq

import numpy as np
import xxhash


class _Page:
    """A view of one page's bookkeeping with the reference ``Block``'s fields
    (``block_id``, ``ref_count``, ``hash``, ``token_ids``, ``last_used``,
    ``update``, ``reset``), reading and writing the manager's arrays."""

    __slots__ = ("_m", "block_id")

    def __init__(self, manager: "CowBlockManager", block_id: int):
        self._m = manager
        self.block_id = block_id

    @property
    def ref_count(self) -> int:
        return self._m.ref_count[self.block_id]

    @ref_count.setter
    def ref_count(self, value: int):
        self._m.ref_count[self.block_id] = value

    @property
    def hash(self) -> int:
        return self._m._key[self.block_id]

    @hash.setter
    def hash(self, value: int):
        self._m._key[self.block_id] = value

    @property
    def token_ids(self) -> list[int]:
        return self._m._tokens[self.block_id]

    @token_ids.setter
    def token_ids(self, value):
        self._m._tokens[self.block_id] = value

    @property
    def last_used(self) -> int:
        return self._m._last_used[self.block_id]

    def update(self, hash: int, token_ids: list[int]):
        self.hash, self.token_ids = hash, token_ids

    def reset(self):
        self.ref_count, self.hash, self.token_ids = 1, -1, []


class CowBlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        if type(num_blocks) is not int or type(block_size) is not int or min(num_blocks, block_size) <= 0:
            raise ValueError("num_blocks and block_size must be positive integers")
        self.num_blocks = num_blocks
        self.block_size = block_size
        n = num_blocks
        self.ref_count = [0] * n      # sequences referencing each page
        self._pins = [0] * n          # queued copies still to read each page
        self._key = [-1] * n          # prefix-cache key of the page's tokens (-1: none)
        self._tokens: list[list[int]] = [[] for _ in range(n)]  # tokens the key covers
        self._last_used = [0] * n
        self._clock = 0
        self._free: set[int] = set(range(n))
        self._lru: list[tuple[int, int]] = [(0, i) for i in range(n)]
        heapq.heapify(self._lru)
        self.used_block_ids: set[int] = set()
        self.hash_to_block_id: dict[int, int] = {}
        self._keys_of: dict[int, set[int]] = {}  # every key published for a page
        self._pending: list[tuple[int, int]] = []  # (src, dst) copies not yet issued
        self.prefix_cache_hit_tokens = 0
        self.prefix_cache_hit_blocks = 0
        self.prefix_cache_evictions = 0

    # ------------------------------------------------------------------ pool
    @property
    def free_block_ids(self) -> set[int]:
        return self._free

    @property
    def blocks(self) -> list[_Page]:
        """Per-page views with the reference ``Block`` fields (diagnostics and tests)."""
        if getattr(self, "_pages", None) is None:
            self._pages = [_Page(self, i) for i in range(self.num_blocks)]
        return self._pages

    @property
    def num_free_blocks(self) -> int:
        return len(self._free)

    @staticmethod
    def compute_hash(token_ids, prefix: int = -1) -> int:
        """Chained key of one page: xxh64 over the previous page's key (8 bytes,
        little endian; none for the first page) and the token ids as int64."""
        h = xxhash.xxh64()
        if prefix != -1:
            h.update(prefix.to_bytes(8, "little"))
        h.update(np.asarray(token_ids, dtype=np.int64).tobytes())
        return h.intdigest()

    def _touch(self, page: int):
        self._clock += 1
        self._last_used[page] = self._clock
        if page in self._free:
            heapq.heappush(self._lru, (self._clock, page))
            if len(self._lru) > max(64, 4 * self.num_blocks):  # drop stale entries
                self._lru = [(self._last_used[i], i) for i in self._free]
                heapq.heapify(self._lru)

    def _forget_keys(self, page: int):
        keys = self._keys_of.pop(page, set())
        if self._key[page] != -1:
            keys.add(self._key[page])
        for k in keys:
            if self.hash_to_block_id.get(k) == page:
                del self.hash_to_block_id[k]

    def _take(self) -> int:
        """The least recently used free page, wiped and referenced once."""
        while self._lru:
            last_used, page = heapq.heappop(self._lru)
            if page in self._free and last_used == self._last_used[page]:
                break
        else:
            raise RuntimeError("KV cache has no free blocks")
        self._free.remove(page)
        self.used_block_ids.add(page)
        if self._tokens[page]:
            self.prefix_cache_evictions += 1
        self._forget_keys(page)
        self.ref_count[page] = 1
        self._key[page] = -1
        self._tokens[page] = []
        self._touch(page)
        return page

    def _drop_ref(self, page: int):
        if self.ref_count[page] <= 0:
            raise RuntimeError(f"block {page} released more often than referenced")
        self.ref_count[page] -= 1
        if self.ref_count[page] == 0:
            # A queued copy into this page is moot now: drop it and unpin its source.
            for k, (src, dst) in enumerate(self._pending):
                if dst == page:
                    del self._pending[k]
                    self._unpin(src)
                    break
            self._maybe_release(page)

    def _unpin(self, page: int):
        self._pins[page] -= 1
        self._maybe_release(page)

    def _maybe_release(self, page: int):
        # Keep the tokens and keys until the page is handed out again.
        if self.ref_count[page] == 0 and self._pins[page] == 0 and page in self.used_block_ids:
            self.used_block_ids.remove(page)
            self._free.add(page)
            self._touch(page)

    def stats(self) -> dict:
        used = len(self.used_block_ids)
        return {
            "num_blocks": self.num_blocks,
            "used_blocks": used,
            "free_blocks": len(self._free),
            "kv_utilization": used / self.num_blocks,
            "prefix_cache_entries": len(self.hash_to_block_id),
            "prefix_cache_hit_tokens": self.prefix_cache_hit_tokens,
            "prefix_cache_hit_blocks": self.prefix_cache_hit_blocks,
            "prefix_cache_evictions": self.prefix_cache_evictions,
        }

    def reset_prefix_cache(self):
        """Forget every cached prefix; only while no page is in use."""
        if self.used_block_ids:
            raise RuntimeError("cannot reset prefix cache while blocks are in use")
        self.hash_to_block_id.clear()
        self._keys_of.clear()
        self._key = [-1] * self.num_blocks
        self._tokens = [[] for _ in range(self.num_blocks)]
        self.prefix_cache_hit_tokens = 0
        self.prefix_cache_hit_blocks = 0
        self.prefix_cache_evictions = 0

    # ------------------------------------------------------------- sequences
    def can_allocate(self, seq) -> int:
        """Reusable cached pages of ``seq`` (its full pages before the first
        miss, never the last page), or -1 if the pool cannot take the rest."""
        reused = free_hits = 0
        key = -1
        for i in range(seq.num_blocks - 1):
            tokens = seq.block(i)
            key = self.compute_hash(tokens, key)
            page = self.hash_to_block_id.get(key)
            if page is None or self._tokens[page] != tokens:
                break
            reused += 1
            self._touch(page)
            if page in self._free:
                free_hits += 1
        # cached pages that sit in the free pool still take free capacity
        if seq.num_blocks - reused > len(self._free) - free_hits:
            return -1
        return reused

    def allocate(self, seq, num_cached_blocks: int):
        """Pages for a new sequence: its first ``num_cached_blocks`` from the
        prefix cache (as ``can_allocate`` found them), fresh ones for the rest.
        Keys of the new pages are published only by ``hash_blocks`` once their
        tokens are stored."""
        if seq.block_table:
            raise ValueError("sequence already holds pages")
        self.prefix_cache_hit_tokens += num_cached_blocks * self.block_size
        self.prefix_cache_hit_blocks += num_cached_blocks
        seq.num_cached_tokens = num_cached_blocks * self.block_size
        key = -1
        for i in range(num_cached_blocks):
            key = self.compute_hash(seq.block(i), key)
            page = self.hash_to_block_id[key]
            if page in self._free:
                self._free.remove(page)
                self.used_block_ids.add(page)
            self.ref_count[page] += 1
            self._touch(page)
            seq.block_table.append(page)
        for i in range(num_cached_blocks, seq.num_blocks):
            tokens = seq.block(i)
            key = self.compute_hash(tokens, key)
            page = self._take()
            self._key[page] = key
            self._tokens[page] = tokens
            seq.block_table.append(page)

    def deallocate(self, seq):
        """Release every page the sequence references."""
        seq.num_cached_tokens = 0
        for page in seq.block_table:
            self._drop_ref(page)
        seq.block_table.clear()

    def trim(self, seq):
        """Release pages past the sequence's current length (speculative rollback)."""
        while len(seq.block_table) > seq.num_blocks:
            self._drop_ref(seq.block_table.pop())

    def _write_page_shared(self, seq, pos: int) -> bool:
        index = pos // self.block_size
        return index < len(seq.block_table) and self.ref_count[seq.block_table[index]] > 1

    def can_append(self, seq) -> bool:
        """Whether ``may_append`` finds its pages: the missing ones, plus a
        private copy when the page of the token stored this step is shared."""
        need = max(0, seq.num_blocks - len(seq.block_table))
        if seq.num_tokens > 0 and self._write_page_shared(seq, seq.num_tokens - 1):
            need += 1
        return len(self._free) >= need

    def _make_private(self, seq, index: int):
        old = seq.block_table[index]
        if self.ref_count[old] <= 1:
            return
        new = self._take()
        self._pending.append((old, new))
        self._pins[old] += 1
        self.ref_count[old] -= 1
        seq.block_table[index] = new

    def may_append(self, seq):
        """Before a decode step (the token at ``num_tokens - 1`` is stored this
        step): pages up to ``num_blocks``, and a private copy of the write
        page when another sequence still references it."""
        if not self.can_append(seq):
            raise ValueError("insufficient cache blocks")
        if seq.num_tokens > 0 and self._write_page_shared(seq, seq.num_tokens - 1):
            self._make_private(seq, (seq.num_tokens - 1) // self.block_size)
        while len(seq.block_table) < seq.num_blocks:
            seq.block_table.append(self._take())

    def prepare_append(self, seq) -> int:
        """Make the page of position ``seq.num_tokens`` (the next token) private
        to ``seq`` and return its slot ``page * block_size + offset``; a new
        page when the position starts one."""
        pos = seq.num_tokens
        index, offset = divmod(pos, self.block_size)
        if index > len(seq.block_table):
            raise ValueError("block table is missing pages before the next token")
        if index == len(seq.block_table):
            seq.block_table.append(self._take())
        else:
            self._make_private(seq, index)
        return seq.block_table[index] * self.block_size + offset

    def hash_blocks(self, seq):
        """After a step: publish the keys of the pages its scheduled tokens
        completed."""
        bs = self.block_size
        start = seq.num_cached_tokens // bs
        end = (seq.num_cached_tokens + seq.num_scheduled_tokens) // bs
        key = self._key[seq.block_table[start - 1]] if start != 0 else -1
        for i in range(start, end):
            tokens = seq.block(i)
            key = self.compute_hash(tokens, key)
            page = seq.block_table[i]
            self.hash_to_block_id[key] = page
            self._keys_of.setdefault(page, set()).add(key)
            self._key[page] = key
            self._tokens[page] = tokens

    # ------------------------------------------------------ copy-on-write only
    def fork(self, parent, child):
        """``child`` shares every page of ``parent``, the partial last one
        included (the caller gives it the parent's tokens and cache state).

        Queued copies must be issued first: a page still waiting for its copy
        holds no valid data yet, so it cannot become the source of another copy
        in the same device launch.
        """
        if child.block_table:
            raise ValueError("child already holds pages")
        if self._pending:
            raise RuntimeError("issue the queued page copies (take_copies) before forking")
        for page in parent.block_table:
            self.ref_count[page] += 1
        child.block_table.extend(parent.block_table)

    def take_copies(self) -> list[tuple[int, int]]:
        """The queued ``(src, dst)`` page copies, in order; the queue is emptied.

        A source page is never a destination of the same batch (destinations are
        fresh pages) and no destination repeats, which is what ``copy_blocks``
        requires.
        """
        pairs, self._pending = self._pending, []
        for src, _ in pairs:
            self._unpin(src)
        return pairs


def apply_copies(manager: CowBlockManager, kv_cache) -> int:
    """Issue the manager's queued page copies on ``kv_cache`` (every layer, K and V)
    as one device launch; returns the number of pages copied.  Call it after the
    step's ``may_append`` / ``prepare_append`` calls and before its ``store_kvcache``."""
    pairs = manager.take_copies()
    if pairs:
        kv_cache.copy_blocks(pairs)
    return len(pairs)
