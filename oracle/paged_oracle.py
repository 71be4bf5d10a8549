"""CPU oracle for the paged KV-cache hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference MicroInfer algorithms, used as the
checker for the sm_100a kernels.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference leg may import it; the product
path (``microinfer_b200``) never does and has no CPU fallback.

Pinned against the reference itself: ``tests/golden/make_golden.py`` runs the
reference's own functions (imported from its source tree) on seeded inputs
and commits their outputs as fixtures; ``tests/test_oracle_golden.py`` checks
this module against every fixture plus the reference tests' known answers.

Storage convention: arrays hold the raw element type -- ``float32``,
``float16``, or ``uint16`` bit patterns for bfloat16 (numpy has no bf16).
Functions take a ``dtype`` name ("f32", "f16", "bf16") where it matters.
"""

from __future__ import annotations

import numpy as np

DTYPES = ("f32", "f16", "bf16")


# ---------------------------------------------------------------------------
# bfloat16 <-> float32 (bit exact)
# ---------------------------------------------------------------------------
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Exact widening: the bf16 bits are the top half of the f32 word."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even narrowing (what torch's .to(bfloat16) does)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded[nan] = 0x7FC0
    return rounded


def to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_to_f32(a)
    return np.asarray(a).astype(np.float32)


def from_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return f32_to_bf16(a)
    if dtype == "f16":
        return np.asarray(a, dtype=np.float32).astype(np.float16)
    return np.asarray(a, dtype=np.float32)


# ---------------------------------------------------------------------------
# store_kvcache
# ---------------------------------------------------------------------------
def store_kv(key_cache, value_cache, blocks, offsets, keys, values) -> None:
    """cache[blocks[t], offsets[t]] = keys[t]; in place.

    Follows the CPU branch of LayerKVCache.write_fast
    (microinfer/worker/kv_cache.py:78-79) and the Triton scatter it replaces
    (microinfer/worker/triton_kv_store.py:17-41).
    """
    key_cache[np.asarray(blocks), np.asarray(offsets)] = keys
    value_cache[np.asarray(blocks), np.asarray(offsets)] = values


def write_checked(key_cache, value_cache, slots, keys, values) -> None:
    """Validated write: -1 skips; range/duplicate errors before any write.

    Follows LayerKVCache.write_checked (microinfer/worker/kv_cache.py:30-50).
    """
    slots = np.asarray(slots)
    if slots.ndim != 1 or slots.dtype.kind not in "iu":
        raise ValueError("slots must be a 1-D integer array")
    expected = (slots.shape[0], *key_cache.shape[2:])
    if keys.shape != expected or values.shape != expected:
        raise ValueError("K/V shape must match slots and cache heads")
    block_size = key_cache.shape[1]
    capacity = key_cache.shape[0] * block_size
    if np.any(slots < -1) or np.any(slots >= capacity):
        raise ValueError("slot outside cache")
    valid = slots >= 0
    idx = slots[valid].astype(np.int64)
    if np.unique(idx).size != idx.size:
        raise ValueError("duplicate slot")
    store_kv(key_cache, value_cache, idx // block_size, idx % block_size, keys[valid], values[valid])


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def _softmax_rows(scores: np.ndarray) -> np.ndarray:
    m = scores.max(axis=-1, keepdims=True)
    e = np.exp(scores - m)
    return e / e.sum(axis=-1, keepdims=True)


def paged_attention(query, key_cache, value_cache, block_tables, context_lens, cu_seqlens_q, *,
                    scale: float, dtype: str, accumulate=np.float32) -> np.ndarray:
    """Causal GQA attention of each request's query rows over its paged cache.

    Follows _paged_attention_reference (microinfer/layer/paged_attention.py:22-67):
    per request, read the first ``context`` rows of its blocks in table order,
    place query row i at absolute position ``context - q_len + i``, mask keys
    past it, softmax in fp32 (fp16/bf16 inputs are widened first), and cast
    the output back to the activation dtype.  Covers decode (q_len 1),
    chunked/prefix prefill and mixed batches alike.
    """
    total, num_q_heads, head_dim = query.shape
    _, block_size, num_kv_heads, _ = key_cache.shape
    group = num_q_heads // num_kv_heads
    q_all = to_f32(query, dtype).astype(accumulate)
    out = np.zeros((total, num_q_heads, head_dim), dtype=accumulate)
    for r in range(len(context_lens)):
        ctx = int(context_lens[r])
        start, end = int(cu_seqlens_q[r]), int(cu_seqlens_q[r + 1])
        q_len = end - start
        if q_len == 0:
            continue
        nblk = (ctx + block_size - 1) // block_size
        blocks = np.asarray(block_tables[r][:nblk], dtype=np.int64)
        k = to_f32(key_cache[blocks], dtype).reshape(-1, num_kv_heads, head_dim)[:ctx]
        v = to_f32(value_cache[blocks], dtype).reshape(-1, num_kv_heads, head_dim)[:ctx]
        k = k.astype(accumulate).transpose(1, 0, 2)  # [Hkv, ctx, D]
        v = v.astype(accumulate).transpose(1, 0, 2)
        q = q_all[start:end].reshape(q_len, num_kv_heads, group, head_dim).transpose(1, 2, 0, 3)
        scores = np.matmul(q, k[:, None].transpose(0, 1, 3, 2)) * accumulate(scale)  # [Hkv,g,q,ctx]
        qpos = (ctx - q_len) + np.arange(q_len)
        visible = qpos[:, None] >= np.arange(ctx)[None, :]
        scores = np.where(visible, scores, -np.inf)
        probs = _softmax_rows(scores)
        o = np.matmul(probs, v[:, None])  # [Hkv, g, q, D]
        out[start:end] = o.transpose(2, 0, 1, 3).reshape(q_len, num_q_heads, head_dim)
    return from_f32(out.astype(np.float32), dtype)


def paged_decode(query, key_cache, value_cache, block_tables, context_lens, *, scale, dtype):
    """Decode = paged_attention with one query row per request."""
    n = len(context_lens)
    return paged_attention(query, key_cache, value_cache, block_tables, context_lens,
                           np.arange(n + 1), scale=scale, dtype=dtype)


def dense_varlen_attention(query, keys, values, cu_seqlens, *, scale, dtype) -> np.ndarray:
    """Causal attention of each request on its own contiguous K/V rows.

    The no-prefix ("direct") prefill of CachedAttention
    (microinfer/layer/cached_attention.py:47-55, :87-101): request r's queries
    and keys are rows cu[r]..cu[r+1] of the packed tensors.
    """
    total, num_q_heads, head_dim = query.shape
    num_kv_heads = keys.shape[1]
    group = num_q_heads // num_kv_heads
    out = np.zeros((total, num_q_heads, head_dim), dtype=np.float32)
    q_all, k_all, v_all = to_f32(query, dtype), to_f32(keys, dtype), to_f32(values, dtype)
    for r in range(len(cu_seqlens) - 1):
        s, e = int(cu_seqlens[r]), int(cu_seqlens[r + 1])
        n = e - s
        if n == 0:
            continue
        q = q_all[s:e].reshape(n, num_kv_heads, group, head_dim).transpose(1, 2, 0, 3)
        k = k_all[s:e].transpose(1, 0, 2)
        v = v_all[s:e].transpose(1, 0, 2)
        scores = np.matmul(q, k[:, None].transpose(0, 1, 3, 2)) * np.float32(scale)
        visible = np.arange(n)[:, None] >= np.arange(n)[None, :]
        probs = _softmax_rows(np.where(visible, scores, -np.inf))
        out[s:e] = np.matmul(probs, v[:, None]).transpose(2, 0, 1, 3).reshape(n, num_q_heads,
                                                                              head_dim)
    return from_f32(out, dtype)


# ---------------------------------------------------------------------------
# gather and copy-on-write
# ---------------------------------------------------------------------------
def gather_paged_kv(key_cache, value_cache, block_tables, contexts, block_size):
    """Each request's first ``context`` rows in logical order, concatenated.

    Follows _gather_paged_kv (microinfer/layer/paged_attention.py:76-101) and
    the test helper tests/support/kv.py:8-24.
    """
    ks, vs = [], []
    tail = key_cache.shape[2:]
    for r, ctx in enumerate(contexts):
        nblk = (int(ctx) + block_size - 1) // block_size
        blocks = np.asarray(block_tables[r][:nblk], dtype=np.int64)
        ks.append(key_cache[blocks].reshape(-1, *tail)[:ctx])
        vs.append(value_cache[blocks].reshape(-1, *tail)[:ctx])
    if not ks:
        empty = np.zeros((0, *tail), dtype=key_cache.dtype)
        return empty, empty.copy()
    return np.concatenate(ks), np.concatenate(vs)


def copy_blocks(key_pool, value_pool, pairs) -> None:
    """pool[:, dst] = pool[:, src] for every pair, every layer, K and V.

    No reference counterpart: the reference shares full prefix blocks by
    refcount (microinfer/engine/blockmanager.py:144-201) and never copies.
    Semantics are those of one vectorised assignment: all sources are read
    before any destination is written.
    """
    pairs = np.asarray(pairs, dtype=np.int64).reshape(-1, 2)
    if pairs.size == 0:
        return
    src, dst = pairs[:, 0], pairs[:, 1]
    key_pool[:, dst] = key_pool[:, src].copy()
    value_pool[:, dst] = value_pool[:, src].copy()


def qk_norm_rope(qkv, q_weight, k_weight, positions, cos_table, sin_table, *, num_q_heads,
                 num_kv_heads, head_dim, eps, interleaved, dtype):
    """Attention prologue: per-head RMSNorm of q and k, then RoPE; returns (q, k, v).

    Follows Attention.forward (microinfer/layer/transformer.py:222-225): q_norm /
    k_norm are F.rms_norm (layer/norm.py: fp32 ``x * rsqrt(mean(x^2) + eps) * w``,
    one rounding to the activation dtype), then RotaryCache.apply
    (layer/rope.py:6-21, 75-84): the rounded values widened to fp32, rotated
    split-half (``cat(a*c - b*s, b*c + a*s)``) or interleaved
    (``stack(a*c - b*s, a*s + b*c)``) with separately rounded fp32 products and
    sums, rounded once more.  ``qkv`` is [T, (Hq + 2 Hkv) * D] in ``dtype``
    (raw bits for bf16), the tables fp32 [max_positions, D/2].
    """
    d = head_dim
    x = to_f32(np.asarray(qkv), dtype).reshape(len(qkv), num_q_heads + 2 * num_kv_heads, d)
    q = x[:, :num_q_heads]
    k = x[:, num_q_heads:num_q_heads + num_kv_heads]
    v = x[:, num_q_heads + num_kv_heads:]
    pos = np.asarray(positions, dtype=np.int64)
    cos = np.asarray(cos_table, np.float32)[pos][:, None, :]
    sin = np.asarray(sin_table, np.float32)[pos][:, None, :]

    def norm_rope(h, w):
        ms = np.mean(h * h, axis=-1, keepdims=True, dtype=np.float32)
        inv = (np.float32(1) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
        y = to_f32(from_f32(h * inv * to_f32(np.asarray(w), dtype), dtype), dtype)
        if interleaved:
            a, b = y[..., 0::2], y[..., 1::2]
            out = np.stack((a * cos - b * sin, a * sin + b * cos), axis=-1).reshape(y.shape)
        else:
            a, b = y[..., : d // 2], y[..., d // 2:]
            out = np.concatenate((a * cos - b * sin, b * cos + a * sin), axis=-1)
        return from_f32(out.astype(np.float32), dtype)

    return norm_rope(q, q_weight), norm_rope(k, k_weight), from_f32(v, dtype)


# ---------------------------------------------------------------------------
# roofline accounting (algorithmic bytes / flops per launch)
# ---------------------------------------------------------------------------
def decode_bytes(contexts, num_q_heads, num_kv_heads, head_dim, elem, block_size) -> int:
    """K and V read once per kv head, Q read, O written, tables and lengths."""
    contexts = [int(c) for c in contexts]
    n = len(contexts)
    kv = sum(2 * c * num_kv_heads * head_dim * elem for c in contexts)
    qo = 2 * n * num_q_heads * head_dim * elem
    tables = 4 * sum((c + block_size - 1) // block_size for c in contexts) + 4 * n
    return kv + qo + tables


def store_bytes(tokens, num_kv_heads, head_dim, elem) -> int:
    return 4 * tokens * num_kv_heads * head_dim * elem + 4 * tokens


def prefill_flops(q_lens, contexts, num_q_heads, head_dim) -> int:
    """Exact causal pairs x 2 GEMMs x 2 flops."""
    total = 0
    for q, c in zip(q_lens, contexts):
        p = int(c) - int(q)
        total += int(q) * p + int(q) * (int(q) + 1) // 2
    return 4 * num_q_heads * head_dim * total
