"""CPU oracle for the runner's per-step attention metadata -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of how the reference's ``ModelRunner`` turns scheduled
sequences into the tensors the attention backend reads.  Only ``tests/`` and
``bench.py``'s CPU-baseline leg may import it; the product path
(``microinfer_b200.worker.runner_metadata``) builds the same tensors on the
device and never calls this module.

Pinned against the reference itself: ``tests/golden/make_runner_golden.py``
ran the reference's ``prepare_prefill`` / ``prepare_decode`` over a seeded
engine scenario and committed the outputs (``tests/golden/runner_scenario.npz``);
``tests/test_runner_metadata.py`` checks this module against every step.

A sequence here is ``(tokens, block_table, num_cached, num_scheduled)``.
"""
from __future__ import annotations

import numpy as np


def slot_of(block_table, position: int, block_size: int) -> int:
    """Physical slot of a token position (runner.py:173-176, 317-321)."""
    return block_table[position // block_size] * block_size + position % block_size


def block_tables(tables) -> np.ndarray:
    """Rows padded with -1 to the longest table (runner.py:298-304, 176-184)."""
    width = max((len(t) for t in tables), default=0)
    out = np.full((len(tables), width), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        out[i, :len(t)] = t
    return out


def prefill_metadata(seqs, block_size: int) -> dict:
    """``prepare_prefill`` (runner.py:306-346): the scheduled range of every
    sequence is ``[num_cached, num_cached + num_scheduled)``; token ids and
    positions of that range in order, cumulative query lengths, cumulative
    key lengths (cached + scheduled), slots from the block table, and block
    tables only when some sequence has cached tokens."""
    ids, positions, slots, cu_q, cu_k = [], [], [], [0], [0]
    for tokens, table, cached, sched in seqs:
        start, end = cached, cached + sched
        if not 0 <= start < end <= len(tokens):
            raise ValueError("invalid scheduled prefill range")
        ids.extend(tokens[start:end])
        positions.extend(range(start, end))
        cu_q.append(cu_q[-1] + end - start)
        cu_k.append(cu_k[-1] + end)
        slots.extend(slot_of(table, p, block_size) for p in range(start, end))
    return {
        "input_ids": np.array(ids, dtype=np.int64),
        "positions": np.array(positions, dtype=np.int64),
        "slot_mapping": np.array(slots, dtype=np.int32),
        "cu_q": np.array(cu_q, dtype=np.int32),
        "cu_k": np.array(cu_k, dtype=np.int32),
        "max_q": max((s[3] for s in seqs), default=0),
        "max_k": max((s[2] + s[3] for s in seqs), default=0),
        "block_tables": (block_tables([s[1] for s in seqs]) if any(s[2] for s in seqs)
                         else None),
    }


def decode_metadata(seqs, block_size: int) -> dict:
    """``prepare_decode`` with ``_fill_decode_rows`` (runner.py:160-188, 348-384):
    per sequence the last token, position ``len - 1``, its slot, the context
    length ``len`` and the -1 padded block table."""
    ids, positions, slots, ctx = [], [], [], []
    for tokens, table, _, _ in seqs:
        pos = len(tokens) - 1
        ids.append(tokens[-1])
        positions.append(pos)
        slots.append(slot_of(table, pos, block_size))
        ctx.append(len(tokens))
    return {
        "input_ids": np.array(ids, dtype=np.int64),
        "positions": np.array(positions, dtype=np.int64),
        "slot_mapping": np.array(slots, dtype=np.int32),
        "context_lens": np.array(ctx, dtype=np.int32),
        "block_tables": block_tables([s[1] for s in seqs]),
    }


class StagedDecodeRows:
    """Timing baseline only: the reference runner's way of producing decode
    metadata (runner.py:160-188, 348-384) restated -- every step a host loop
    writes each sequence's token, position, slot, context length and whole
    block-table row into pinned staging tensors, then five tensors are copied
    to the device.  ``bench.py`` times it beside the device builder."""

    def __init__(self, block_size: int, capacity: int, width: int, device):
        import torch

        pin = torch.device(device).type == "cuda"
        self.block_size = block_size
        self.host = {
            "input_ids": torch.empty(capacity, dtype=torch.int64, pin_memory=pin),
            "positions": torch.empty(capacity, dtype=torch.int64, pin_memory=pin),
            "slot_mapping": torch.empty(capacity, dtype=torch.int32, pin_memory=pin),
            "context_lens": torch.empty(capacity, dtype=torch.int32, pin_memory=pin),
            "block_tables": torch.empty(capacity, width, dtype=torch.int32, pin_memory=pin),
        }
        self.dev = {k: torch.empty_like(v, device=device) for k, v in self.host.items()}
        self.pin = pin

    def prepare_decode(self, seqs):
        import torch

        h, bs, batch = self.host, self.block_size, len(seqs)
        h["block_tables"][:batch].fill_(-1)
        for i, seq in enumerate(seqs):
            pos = len(seq) - 1
            table = seq.block_table
            h["input_ids"][i] = seq.last_token
            h["positions"][i] = pos
            h["slot_mapping"][i] = table[pos // bs] * bs + pos % bs
            h["context_lens"][i] = len(seq)
            h["block_tables"][i, :len(table)] = torch.tensor(table, dtype=torch.int32)
        for k in ("input_ids", "positions", "slot_mapping", "context_lens", "block_tables"):
            self.dev[k][:batch].copy_(h[k][:batch], non_blocking=self.pin)
        return self.dev["input_ids"][:batch], self.dev["positions"][:batch]


def staged_prefill(seqs, block_size: int, device):
    """Timing baseline only: the reference runner's ``prepare_prefill``
    (runner.py:298-346) restated -- Python lists of every scheduled token's id,
    position and slot, cumulative lengths, the -1 padded block tables when some
    sequence has cached tokens, each built into a device tensor.  ``seqs`` are
    objects with ``token_ids``, ``block_table``, ``num_cached_tokens`` and
    ``num_scheduled_tokens``.  ``bench.py`` times it beside the device builder."""
    import torch

    ids, positions, slots, cu_q, cu_k = [], [], [], [0], [0]
    for seq in seqs:
        start = seq.num_cached_tokens
        end = start + seq.num_scheduled_tokens
        ids.extend(seq.token_ids[start:end])
        positions.extend(range(start, end))
        cu_q.append(cu_q[-1] + end - start)
        cu_k.append(cu_k[-1] + end)
        table = seq.block_table
        slots.extend(table[p // block_size] * block_size + p % block_size for p in range(start, end))
    out = {
        "cu_q": torch.tensor(cu_q, dtype=torch.int32, device=device),
        "cu_k": torch.tensor(cu_k, dtype=torch.int32, device=device),
        "slot_mapping": torch.tensor(slots, dtype=torch.int32, device=device),
        "input_ids": torch.tensor(ids, dtype=torch.int64, device=device),
        "positions": torch.tensor(positions, dtype=torch.int64, device=device),
    }
    if any(s.num_cached_tokens for s in seqs):
        width = max(len(s.block_table) for s in seqs)
        out["block_tables"] = torch.tensor(
            [list(s.block_table) + [-1] * (width - len(s.block_table)) for s in seqs],
            dtype=torch.int32, device=device)
    return out
