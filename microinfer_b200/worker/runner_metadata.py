"""Per-step attention metadata built on the device from a resident page table.

The reference runner rebuilds every step's metadata on the host
(``ModelRunner.prepare_decode`` / ``_fill_decode_rows``, microinfer/runner.py:
160-188 and 348-384; ``prepare_prefill`` / ``prepare_block_tables``, :298-346):
a Python loop over the scheduled sequences fills pinned staging tensors
element by element -- the whole block table of every sequence, every step --
and five tensors are copied to the device.  For small decode batches that host
work dominates the step.

``DeviceRunnerMetadata`` keeps the block tables in HBM instead: one page-table
row per running sequence (``[max_rows, max_pages]`` int32).  A step sends only
what changed -- a 6-int record per sequence and the page-table entries written
since the last step (a new page at a block boundary, a page replaced by
copy-on-write, the whole table of a sequence new to its row) -- as one int32
buffer in one host-to-device copy, and one launch (``mi_build_decode_metadata``
/ ``mi_build_prefill_metadata``) applies the changes and writes ``input_ids``,
``positions``, ``slot_mapping``, ``context_lens`` / ``cu_seqlens_q/k`` and the
-1 padded ``block_tables``, with the values and shapes the reference's runner
produces.  ``prepare_decode`` / ``prepare_prefill`` return the reference's
``(input_ids, position_ids, metadata)`` triple.

Changes are found without walking whole tables: a step writes K/V only at
positions from its first scheduled token on, and pages before the page of that
token never change while the sequence keeps its row (full pages are immutable;
copy-on-write replaces only the page being written).  So each sequence's table
is compared with what was sent before from that page on.  ``verify=True``
compares whole tables instead and raises if an earlier page changed.

Sequences are any objects with ``block_table``, ``num_tokens`` (or ``len``),
``last_token``, ``num_cached_tokens``, ``num_scheduled_tokens``, token
indexing and a ``seq_id`` (the reference's ``Sequence``); call ``release``
when a sequence finishes or is preempted so its row can be reused.
"""
from __future__ import annotations

from collections import deque

import numpy as np
import torch

from microinfer_b200 import _lib
from microinfer_b200.layer.metadata import AttentionMetadata

RECORD = 6  # int32 per sequence: row, a, b, num_pages, update_begin, update_count


class _Updates:
    """Page-table changes of one step as (column, page) int32 pairs, kept as two
    flat lists so whole tables (sequences new to their row) join with C-level
    list operations and become one array at the end.  Single entries are range
    checked as they are added, whole tables once in ``array``."""

    __slots__ = ("cols", "pages", "unchecked")

    def __init__(self):
        self.cols: list = []
        self.pages: list = []
        self.unchecked = False

    def __len__(self) -> int:
        return len(self.cols)

    def add(self, col: int, page: int):
        self.cols.append(col)
        self.pages.append(page)

    def add_table(self, table):
        self.cols.extend(range(len(table)))
        self.pages.extend(table)
        self.unchecked = True

    def array(self, num_blocks: int) -> np.ndarray:
        if not self.cols:
            return np.empty((0, 2), dtype=np.int32)
        a = np.array((self.cols, self.pages), dtype=np.int64)
        if self.unchecked and (a[1].min() < 0 or a[1].max() >= num_blocks):
            raise ValueError("block id outside the pool")
        return np.ascontiguousarray(a.T, dtype=np.int32)


def _seq_key(seq):
    key = getattr(seq, "seq_id", None)
    return id(seq) if key is None else key


def _num_tokens(seq) -> int:
    n = getattr(seq, "num_tokens", None)
    return len(seq) if n is None else int(n)


class DeviceRunnerMetadata:
    def __init__(self, block_size: int, num_blocks: int, *, max_rows: int = 256,
                 max_pages: int | None = None, device="cuda", verify: bool = False):
        if min(block_size, num_blocks, max_rows) <= 0:
            raise ValueError("block_size, num_blocks and max_rows must be positive")
        if num_blocks * block_size > 2**31 - 1:
            raise ValueError("slots must fit int32")
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.max_rows = max_rows
        self.max_pages = int(max_pages or num_blocks)
        self.device = torch.device(device)
        self.verify = verify
        self.page_table = torch.full((max_rows, self.max_pages), -1, dtype=torch.int32,
                                     device=self.device)
        self._rows: dict = {}
        self._free_rows = deque(range(max_rows))
        self._sent: list[list[int]] = [[] for _ in range(max_rows)]  # pages already on device
        pin = self.device.type == "cuda"
        # two pinned staging buffers, each reused only after its previous copy has ended
        self._stage = [torch.empty(0, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._stage_done = [None, None]
        self._flip = 0
        self._pin = pin
        self._dev_in = torch.empty(0, dtype=torch.int32, device=self.device)
        # decode outputs persist (the reference's _DecodeBuffers): stable addresses for graphs
        self._dec_cap = 0
        self._dec = {}
        self._dec_width = 0
        self._dec_views: dict = {}
        self._status = _lib.status_buffer(self.device).data_ptr() if self._pin else 0

    # ------------------------------------------------------------------ rows
    def row_of(self, seq) -> int:
        key = _seq_key(seq)
        row = self._rows.get(key)
        if row is None:
            if not self._free_rows:
                raise RuntimeError("no free page-table row: release finished sequences")
            row = self._free_rows.popleft()
            self._rows[key] = row
            self._sent[row] = []
        return row

    def release(self, seq):
        """Give the sequence's row back (finished or preempted sequences)."""
        row = self._rows.pop(_seq_key(seq), None)
        if row is not None:
            self._sent[row] = []
            self._free_rows.append(row)

    @property
    def num_free_rows(self) -> int:
        return len(self._free_rows)

    def _changes(self, seq, row: int, first_pos: int, updates: _Updates, commits: list) -> int:
        """Append (column, page) pairs for the entries of ``seq``'s table that the
        device does not hold yet; returns the number appended.  What the device
        will hold after the launch is queued in ``commits`` and recorded only once
        the launch has been issued (``_commit``)."""
        table = seq.block_table
        if len(table) > self.max_pages:
            raise ValueError("block table longer than max_pages")
        sent = self._sent[row]
        if self.verify:
            k0 = 0
            keep = min(len(sent), first_pos // self.block_size)
            if list(table[:keep]) != sent[:keep]:
                raise ValueError("a page before the first scheduled token changed")
        else:
            k0 = min(len(sent), max(first_pos, 0) // self.block_size)
        n0 = len(updates.cols)
        if not sent:  # a row new to this sequence: the whole table (checked in array())
            updates.add_table(table)
        else:
            for col in range(k0, len(table)):
                page = table[col]
                if col >= len(sent) or sent[col] != page:
                    if not 0 <= page < self.num_blocks:
                        raise ValueError(f"block id {page} outside the pool")
                    updates.add(col, page)
        commits.append((row, k0, list(table[k0:])))
        return len(updates.cols) - n0

    def _commit(self, commits: list):
        for row, k0, tail in commits:
            sent = self._sent[row]
            del sent[k0:]
            sent.extend(tail)

    # --------------------------------------------------------------- staging
    def _upload(self, parts: list[np.ndarray]) -> list[int]:
        """Copy the int32 parts to the device in one transfer; returns their
        device addresses."""
        sizes = [p.size for p in parts]
        total = sum(sizes)
        k = self._flip
        self._flip ^= 1
        if self._stage_done[k] is not None:
            self._stage_done[k].synchronize()  # that buffer's previous copy has ended
        if self._stage[k].numel() < total:
            cap = max(total, 2 * self._stage[k].numel(), 1024)
            self._stage[k] = torch.empty(cap, dtype=torch.int32, pin_memory=self._pin)
        if self._dev_in.numel() < total:
            self._dev_in = torch.empty(max(total, 2 * self._dev_in.numel(), 1024),
                                       dtype=torch.int32, device=self.device)
        host = self._stage[k].numpy()
        views, off = [], 0
        for part, n in zip(parts, sizes):
            host[off:off + n] = part.reshape(-1)
            views.append((off, n))
            off += n
        if total:
            self._dev_in[:total].copy_(self._stage[k][:total], non_blocking=self._pin)
        if self._pin:
            if self._stage_done[k] is None:
                self._stage_done[k] = torch.cuda.Event()
            self._stage_done[k].record(torch.cuda.current_stream(self.device))
        base = self._dev_in.data_ptr()
        return [base + 4 * o for o, _ in views]

    def _decode_outputs(self, batch: int, width: int):
        """Persistent decode outputs (the reference's _DecodeBuffers: stable
        addresses for graph capture; the table width only grows, runner.py:27-48),
        with the per-batch views cached."""
        if batch > self._dec_cap or width > self._dec_width:
            cap, w = max(batch, self._dec_cap), max(width, self._dec_width)
            dev = self.device
            self._dec = {
                "input_ids": torch.empty(cap, dtype=torch.int64, device=dev),
                "positions": torch.empty(cap, dtype=torch.int64, device=dev),
                "slot_mapping": torch.empty(cap, dtype=torch.int32, device=dev),
                "context_lens": torch.empty(cap, dtype=torch.int32, device=dev),
                "block_tables": torch.empty(cap * w, dtype=torch.int32, device=dev),
            }
            self._dec_cap, self._dec_width = cap, w
            self._dec_views = {}
        views = self._dec_views.get(batch)
        if views is None:
            d, w = self._dec, self._dec_width
            views = (d["input_ids"][:batch], d["positions"][:batch], d["slot_mapping"][:batch],
                     d["context_lens"][:batch], d["block_tables"][:batch * w].view(batch, w))
            self._dec_views[batch] = views
        return views

    # ---------------------------------------------------------------- decode
    def plan_decode(self, seqs) -> dict:
        """Host half of ``prepare_decode``: rows, records and page-table changes
        (no device work; the rows of new sequences are assigned here).  Kept to
        a few dictionary and list operations per sequence: this loop is the
        whole per-step host cost."""
        batch = len(seqs)
        if batch == 0:
            raise ValueError("a scheduled batch must contain requests")
        bs, rows, sent_all, verify = self.block_size, self._rows, self._sent, self.verify
        flat: list = []
        updates = _Updates()
        commits: list = []
        seen: set = set()
        width = 0
        for seq in seqs:
            n = _num_tokens(seq)
            table = seq.block_table
            pages = len(table)
            k = (n - 1) // bs  # page of the decoded token
            if n <= 0 or k >= pages:
                raise ValueError("block table does not cover the decoded token")
            row = rows.get(_seq_key(seq))
            if row is None:
                row = self.row_of(seq)
            if row in seen:
                raise ValueError("a sequence appears twice in the batch")
            seen.add(row)
            sent = sent_all[row]
            begin = len(updates.cols)
            if verify or sent[k:] != table[k:]:  # usually one entry compared
                self._changes(seq, row, n - 1, updates, commits)
            flat += (row, n, seq.last_token, pages, begin, len(updates.cols) - begin)
            if pages > width:
                width = pages
        try:
            rec = np.array(flat, dtype=np.int32).reshape(batch, RECORD)
        except OverflowError:
            raise ValueError("token ids must be nonnegative int32 values") from None
        if rec[:, 2].min() < 0:
            raise ValueError("token ids must be nonnegative int32 values")
        return {"records": rec, "updates": updates.array(self.num_blocks), "width": width, "commits": commits}

    def prepare_decode(self, seqs):
        """``ModelRunner.prepare_decode``: last token, position ``len - 1``, its
        slot, context length and block tables ``[batch, width]``."""
        _lib.require_cuda(self.page_table)
        plan = self.plan_decode(seqs)
        batch = len(seqs)
        ids, pos, slots, ctx, bt = self._decode_outputs(batch, plan["width"])
        rec_d, upd_d = self._upload([plan["records"], plan["updates"]])
        _lib.call("mi_build_decode_metadata", self.page_table.data_ptr(), self.max_rows,
                  self.max_pages, rec_d, batch, upd_d, len(plan["updates"]), self.block_size,
                  self.num_blocks, bt.shape[1], ids.data_ptr(), pos.data_ptr(), slots.data_ptr(),
                  ctx.data_ptr(), bt.data_ptr(), self._status, _lib.stream_of(self.device))
        self._commit(plan["commits"])
        metadata = AttentionMetadata(is_prefill=False, slot_mapping=slots, context_lens=ctx,
                                     block_tables=bt, validate_cache_write=False)
        return ids, pos, metadata

    # --------------------------------------------------------------- prefill
    def plan_prefill(self, seqs) -> dict:
        """Host half of ``prepare_prefill`` (no device work)."""
        batch = len(seqs)
        if batch == 0:
            raise ValueError("a scheduled batch must contain requests")
        rec = np.empty((batch, RECORD), dtype=np.int32)
        updates = _Updates()
        commits: list = []
        tokens = []
        seen = set()
        width = max_q = max_k = 0
        any_cached = False
        for i, seq in enumerate(seqs):
            start = int(seq.num_cached_tokens)
            end = start + int(seq.num_scheduled_tokens)
            if not 0 <= start < end <= _num_tokens(seq):
                raise ValueError("invalid scheduled prefill range")
            pages = len(seq.block_table)
            if (end - 1) // self.block_size >= pages:
                raise ValueError("block table does not cover scheduled tokens")
            row = self.row_of(seq)
            if row in seen:
                raise ValueError("a sequence appears twice in the batch")
            seen.add(row)
            begin = len(updates.cols)
            count = self._changes(seq, row, start, updates, commits)
            rec[i] = (row, start, end, pages, begin, count)
            tokens.extend(seq[start:end])
            width = max(width, pages)
            max_q = max(max_q, end - start)
            max_k = max(max_k, end)
            any_cached = any_cached or start > 0
        ids = np.array(tokens, dtype=np.int64)
        if ids.size and (ids.min() < 0 or ids.max() > 2**31 - 1):
            raise ValueError("token ids must be nonnegative int32 values")
        if ids.size > 2**31 - 1:
            raise ValueError("too many scheduled tokens")
        return {"records": rec, "updates": updates.array(self.num_blocks),
                "tokens": ids.astype(np.int32), "table_width": width if any_cached else 0,
                "max_q": max_q, "max_k": max_k, "commits": commits}

    def prepare_prefill(self, seqs, *, validate_cache_write: bool = False):
        """``ModelRunner.prepare_prefill``: the scheduled range
        ``[num_cached, num_cached + num_scheduled)`` of every sequence; block
        tables only when some sequence has cached tokens (else direct prefill)."""
        _lib.require_cuda(self.page_table)
        plan = self.plan_prefill(seqs)
        batch, t, tw = len(seqs), int(plan["tokens"].size), plan["table_width"]
        rec_d, upd_d, tok_d = self._upload([plan["records"], plan["updates"], plan["tokens"]])
        dev = self.device
        input_ids = torch.empty(t, dtype=torch.int64, device=dev)
        positions = torch.empty(t, dtype=torch.int64, device=dev)
        slots = torch.empty(t, dtype=torch.int32, device=dev)
        cu = torch.empty(2, batch + 1, dtype=torch.int32, device=dev)
        bt = torch.empty(batch, tw, dtype=torch.int32, device=dev) if tw else None
        _lib.call("mi_build_prefill_metadata", self.page_table.data_ptr(), self.max_rows,
                  self.max_pages, rec_d, batch, upd_d, len(plan["updates"]), tok_d, t,
                  self.block_size, self.num_blocks,
                  tw, input_ids.data_ptr(), positions.data_ptr(), slots.data_ptr(),
                  cu[0].data_ptr(), cu[1].data_ptr(), 0 if bt is None else bt.data_ptr(),
                  _lib.status_buffer(dev).data_ptr(), _lib.stream_of(dev))
        self._commit(plan["commits"])
        metadata = AttentionMetadata.build(
            is_prefill=True, cu_seqlens_q=cu[0], cu_seqlens_k=cu[1],
            max_seqlen_q=plan["max_q"], max_seqlen_k=plan["max_k"], slot_mapping=slots,
            block_tables=bt, validate_cache_write=validate_cache_write)
        return input_ids, positions, metadata
