"""Host-side page allocator with reference counts and copy-on-write.

The engine's block manager (reference ``microinfer/engine/blockmanager.py:27-242``)
refcounts pages so that sequences can share a cached prefix, but it never shares
the partial last block (``can_allocate``, :144-148): a sequence writing its next
token into a shared page would overwrite the other sequences' view.  This class
keeps the same page bookkeeping (``block_table`` lists of page ids per sequence,
``ref_count`` per page, a free pool) and adds the missing piece: sequences may
share every page, the partial last one included (``fork``), and a sequence about
to write into a page that another sequence still references gets a private copy
first (``prepare_append``).  The copies are queued as ``(src, dst)`` page pairs;
the worker runs them on the device with ``KVCache.copy_blocks`` (one launch for
all layers, K and V) before the step's ``store_kvcache``, see ``apply_copies``.

Only the page allocation and the copy-on-write rule live here.  Prefix caching by
token hashes, LRU eviction and the scheduler stay with the engine.

Sequences are any objects with a ``block_table`` list and a ``num_tokens`` count
(the reference's ``Sequence`` has both).
"""
from __future__ import annotations

from collections import deque


class CowBlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        if type(num_blocks) is not int or type(block_size) is not int or min(num_blocks, block_size) <= 0:
            raise ValueError("num_blocks and block_size must be positive integers")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.ref_count = [0] * num_blocks  # sequences referencing each page
        self._pins = [0] * num_blocks  # queued copies still to read each page
        self._free = deque(range(num_blocks))
        self._pending: list[tuple[int, int]] = []  # (src, dst) copies not yet issued

    # ------------------------------------------------------------------ pool
    @property
    def num_free_blocks(self) -> int:
        return len(self._free)

    def _take(self) -> int:
        if not self._free:
            raise RuntimeError("KV cache has no free blocks")
        block_id = self._free.popleft()
        self.ref_count[block_id] = 1
        return block_id

    def _release(self, block_id: int):
        if self.ref_count[block_id] <= 0:
            raise RuntimeError(f"block {block_id} released more often than referenced")
        self.ref_count[block_id] -= 1
        if self.ref_count[block_id] == 0:
            # A queued copy into this page is moot now: drop it and unpin its source.
            for k, (src, dst) in enumerate(self._pending):
                if dst == block_id:
                    del self._pending[k]
                    self._unpin(src)
                    break
            self._maybe_free(block_id)

    def _unpin(self, block_id: int):
        self._pins[block_id] -= 1
        self._maybe_free(block_id)

    def _maybe_free(self, block_id: int):
        if self.ref_count[block_id] == 0 and self._pins[block_id] == 0:
            self._free.append(block_id)

    def blocks_needed(self, num_tokens: int) -> int:
        return (num_tokens + self.block_size - 1) // self.block_size

    # ------------------------------------------------------------- sequences
    def can_allocate(self, seq) -> bool:
        return self.blocks_needed(seq.num_tokens) <= self.num_free_blocks

    def allocate(self, seq):
        """Fresh pages for every block of a new sequence."""
        if seq.block_table:
            raise ValueError("sequence already holds pages")
        need = self.blocks_needed(seq.num_tokens)
        if need > self.num_free_blocks:
            raise RuntimeError("KV cache has no free blocks")
        seq.block_table.extend(self._take() for _ in range(need))

    def fork(self, parent, child):
        """``child`` shares every page of ``parent``, the partial last one included.

        Queued copies must be issued first: a page still waiting for its copy
        holds no valid data yet, so it cannot become the source of another copy
        in the same device launch.
        """
        if child.block_table:
            raise ValueError("child already holds pages")
        if self._pending:
            raise RuntimeError("issue the queued page copies (take_copies) before forking")
        for block_id in parent.block_table:
            self.ref_count[block_id] += 1
        child.block_table.extend(parent.block_table)

    def deallocate(self, seq):
        """Release every page the sequence references."""
        for block_id in seq.block_table:
            self._release(block_id)
        seq.block_table.clear()

    def can_append(self, seq) -> bool:
        """Whether the next token of ``seq`` finds a page (new or private copy)."""
        pos = seq.num_tokens  # position of the token about to be written
        index = pos // self.block_size
        if index >= len(seq.block_table):
            return self.num_free_blocks >= 1
        return self.ref_count[seq.block_table[index]] == 1 or self.num_free_blocks >= 1

    def prepare_append(self, seq) -> int:
        """Make the page of the next token (position ``seq.num_tokens``) private to
        ``seq`` and return its slot (``page * block_size + offset``).

        A new block gets a fresh page.  A page that other sequences still reference
        is replaced by a copy: a fresh page is taken, ``(old, new)`` is queued for
        the device copy and ``seq`` drops its reference to the old page, which the
        queued copy pins until it is handed out (``take_copies``): the old page is
        neither freed nor reused before it has been read.  The other sequences keep
        writing into the old page; a step issues its copies before its stores
        (``apply_copies``), so the copy reads the page as it was.
        """
        pos = seq.num_tokens
        index, offset = divmod(pos, self.block_size)
        if index > len(seq.block_table):
            raise ValueError("block table is missing pages before the next token")
        if index == len(seq.block_table):
            seq.block_table.append(self._take())
        else:
            old = seq.block_table[index]
            if self.ref_count[old] > 1:
                new = self._take()
                self._pending.append((old, new))
                self._pins[old] += 1
                self.ref_count[old] -= 1
                seq.block_table[index] = new
        return seq.block_table[index] * self.block_size + offset

    # ------------------------------------------------------------ copy queue
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
    step's ``prepare_append`` calls and before its ``store_kvcache``."""
    pairs = manager.take_copies()
    if pairs:
        kv_cache.copy_blocks(pairs)
    return len(pairs)
