"""Seeded synthetic inputs at the full sizes of the BASELINE.json configs.

Shared by the full-size parity tests (``tests/test_full_configs.py``) and by
``bench.py``, so every timed workload is also a checked one.  Builders return
host (CPU) torch tensors; the caller moves them to the device.

* ``mixed_batch``         configs[2]: 24 decode sequences, context U[1, 4096],
                          plus 8 prefill sequences each adding a 512-token chunk
                          on U[0, 1536] cached tokens, one launch
* ``shared_prefix_batch`` configs[3]: 64 sequences sharing a 1024-token prefix
                          stored once (the same 64 block ids in every table),
                          each with its own 128-token suffix
* ``long_batch``          configs[4] run (a): contexts U[4096, 32768]
* ``torch_paged_attention`` a device-side fp32 restatement of the reference's
                          ``_paged_attention_reference`` (layer/paged_attention.py:22-67)
                          for sizes the numpy oracle would take minutes on
"""

from __future__ import annotations

import torch

BS = 16


def _tables(gen, contexts, nb, bs=BS):
    need = [(c + bs - 1) // bs for c in contexts]
    perm = torch.randperm(nb, generator=gen).to(torch.int32)
    table = torch.full((len(contexts), max(need)), -1, dtype=torch.int32)
    at = 0
    for r, k in enumerate(need):
        table[r, :k] = perm[at:at + k]
        at += k
    return table


def _finish(q_lens, contexts, table, nb, bs=BS):
    cu_q = torch.zeros(len(q_lens) + 1, dtype=torch.int32)
    cu_q[1:] = torch.cumsum(torch.tensor(q_lens), 0)
    cu_k = torch.zeros(len(contexts) + 1, dtype=torch.int32)
    cu_k[1:] = torch.cumsum(torch.tensor(contexts), 0)
    slots = []
    for r, (q, c) in enumerate(zip(q_lens, contexts)):
        row = table[r]
        for pos in range(c - q, c):
            slots.append(int(row[pos // bs]) * bs + pos % bs)
    return dict(q_lens=list(q_lens), contexts=list(contexts), nb=nb, table=table, cu_q=cu_q,
                cu_k=cu_k, slots=torch.tensor(slots, dtype=torch.int32),
                max_q=max(q_lens), tokens=int(sum(q_lens)))


def mixed_batch(seed: int = 3):
    """24 one-token decode rows (context U[1, 4096]) and 8
    chunks of 512 tokens on U[0, 1536] cached tokens, random block tables."""
    gen = torch.Generator().manual_seed(seed)
    dec = torch.randint(1, 4097, (24,), generator=gen)
    pre_p = torch.randint(0, 1537, (8,), generator=gen)
    q_lens = [1] * 24 + [512] * 8
    contexts = dec.tolist() + (pre_p + 512).tolist()
    nb = sum((c + BS - 1) // BS for c in contexts) + 8
    table = _tables(gen, contexts, nb)
    return _finish(q_lens, contexts, table, nb)


SHARED_PREFIX, SHARED_SUFFIX, SHARED_SEQS = 1024, 128, 64


def shared_prefix_batch(n: int = SHARED_SEQS, prefix: int = SHARED_PREFIX,
                        suffix: int = SHARED_SUFFIX):
    """``n`` sequences share one ``prefix``-token prefix
    stored once (block ids 0 .. prefix/16 - 1 in every table); each prefills its
    own ``suffix``-token chunk on top of it."""
    shared = torch.arange(prefix // BS, dtype=torch.int32)
    per = suffix // BS
    nb = prefix // BS + n * per + 8
    table = torch.empty((n, prefix // BS + per), dtype=torch.int32)
    for r in range(n):
        table[r, :prefix // BS] = shared
        table[r, prefix // BS:] = torch.arange(prefix // BS + r * per, prefix // BS + (r + 1) * per)
    return _finish([suffix] * n, [prefix + suffix] * n, table, nb)


def long_batch(n: int, seed: int = 7, lo: int = 4096, hi: int = 32768):
    """BASELINE configs[4] run (a) contexts U[lo, hi] (one decode token each)."""
    gen = torch.Generator().manual_seed(seed)
    ctx = torch.randint(lo, hi + 1, (n,), generator=gen, dtype=torch.int32)
    contexts = ctx.tolist()
    nb = sum((c + BS - 1) // BS for c in contexts) + 1
    table = _tables(gen, contexts, nb)
    return _finish([1] * n, contexts, table, nb)


def torch_paged_attention(query, key_cache, value_cache, block_tables, contexts, cu_q, scale,
                          rows=None):
    """fp32 causal GQA attention of each request's query rows over its paged cache.

    The reference's ``_paged_attention_reference`` (microinfer/layer/paged_attention.py:22-67)
    on the device: per request, the first ``ctx`` rows of its blocks in table
    order, query row i at position ``ctx - q_len + i``, keys past it masked,
    softmax in fp32, output cast to the activation dtype.  ``rows`` limits the
    work to some requests (the others stay zero).
    """
    _, hq, d = query.shape
    _, bs, hkv, _ = key_cache.shape
    g = hq // hkv
    out = torch.zeros_like(query)
    cu = [int(x) for x in cu_q]
    for r in (range(len(contexts)) if rows is None else rows):
        ctx = int(contexts[r])
        s, e = cu[r], cu[r + 1]
        if e == s:
            continue
        nblk = (ctx + bs - 1) // bs
        blocks = block_tables[r, :nblk].long()
        k = key_cache[blocks].reshape(-1, hkv, d)[:ctx].float()
        v = value_cache[blocks].reshape(-1, hkv, d)[:ctx].float()
        q = query[s:e].float().reshape(e - s, hkv, g, d)
        score = torch.einsum("qhgd,khd->hgqk", q, k) * scale
        qpos = (ctx - (e - s)) + torch.arange(e - s, device=query.device)
        vis = qpos[:, None] >= torch.arange(ctx, device=query.device)[None, :]
        score = score.masked_fill(~vis, float("-inf"))
        o = torch.einsum("hgqk,khd->qhgd", torch.softmax(score, dim=-1), v)
        out[s:e] = o.reshape(e - s, hq, d).to(query.dtype)
    return out


# ---------------------------------------------------------------------------
# Algorithmic work (the roofline numerators), e = element bytes
# ---------------------------------------------------------------------------
def decode_bytes(contexts, hq, hkv, d, e, bs):
    """K/V read once per kv head + Q read + O written + table entries + lengths."""
    kv = sum(2 * int(c) * hkv * d * e for c in contexts)
    return kv + 2 * len(contexts) * hq * d * e + 4 * sum((int(c) + bs - 1) // bs
                                                         for c in contexts) + 4 * len(contexts)


def store_bytes(tokens, hkv, d, e):
    """K/V rows read and written + one int32 slot per token."""
    return 4 * tokens * hkv * d * e + 4 * tokens


def prefill_flops(q_lens, contexts, hq, d):
    """Exact causal (query, key) pairs x 2 GEMMs x 2 flops."""
    pairs = 0
    for q, c in zip(q_lens, contexts):
        p = int(c) - int(q)
        pairs += int(q) * p + int(q) * (int(q) + 1) // 2
    return 4 * hq * d * pairs


def gather_bytes(contexts, hkv, d, e):
    """Each request's K and V rows read and written once."""
    return 2 * 2 * sum(int(c) for c in contexts) * hkv * d * e


def cow_bytes(pairs, layers, bs, hkv, d, e):
    """Every (src, dst) page copied in every layer, K and V, read and written."""
    return 2 * pairs * 2 * layers * bs * hkv * d * e
