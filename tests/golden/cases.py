"""Seeded, platform-stable input generators for the parity cases.

Every case is rebuilt from a numpy PCG64 seed, so the committed fixtures hold
only the reference's outputs plus a SHA-256 of each input (the tests check
that regeneration reproduced the exact bytes).  Shapes follow the
BASELINE.json configs (1, 2, and reduced 3/4) and the reference's own
hot-path tests (tests/layers/test_triton_paged_attention.py,
tests/components/test_paged_attention.py, test_kv_cache.py).

Arrays use the oracle's storage convention: float32, float16, or uint16 bit
patterns for bfloat16.
"""

from __future__ import annotations

import hashlib
import math

import numpy as np

from oracle.paged_oracle import f32_to_bf16


def _cast(x: np.ndarray, dtype: str) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return f32_to_bf16(x)
    if dtype == "f16":
        return x.astype(np.float16)
    return x


def _normal(rng, shape, dtype, scale=1.0):
    return _cast(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale), dtype)


def digest(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.tobytes() + str(a.dtype).encode() + str(a.shape).encode()).hexdigest()


def _tables(rng, contexts, block_size, num_blocks, permute=True):
    """Random permutation of block ids; each request takes the next ceil(ctx/bs)."""
    ids = rng.permutation(num_blocks) if permute else np.arange(num_blocks)
    need = [(c + block_size - 1) // block_size for c in contexts]
    width = max(need) if need else 0
    table = np.full((len(contexts), max(width, 1)), -1, dtype=np.int32)
    at = 0
    for r, n in enumerate(need):
        table[r, :n] = ids[at:at + n]
        at += n
    assert at <= num_blocks
    return table


def _slot(table_row, pos, block_size):
    return int(table_row[pos // block_size]) * block_size + pos % block_size


def decode_case(seed, n, hq, hkv, d, bs, nb, ctx_lo, ctx_hi, dtype, pool_scale=1.0, contexts=None,
                table=None):
    """Store this step's token via slot_mapping, then decode over the cache."""
    rng = np.random.default_rng(seed)
    if contexts is None:
        contexts = rng.integers(ctx_lo, ctx_hi + 1, size=n).astype(np.int32)
    contexts = np.asarray(contexts, dtype=np.int32)
    if table is None:
        table = _tables(rng, contexts, bs, nb)
    key_cache = _normal(rng, (nb, bs, hkv, d), dtype, pool_scale)
    value_cache = _normal(rng, (nb, bs, hkv, d), dtype, pool_scale)
    query = _normal(rng, (n, hq, d), dtype)
    k_new = _normal(rng, (n, hkv, d), dtype)
    v_new = _normal(rng, (n, hkv, d), dtype)
    slots = np.array([_slot(table[r], int(contexts[r]) - 1, bs) for r in range(n)], dtype=np.int32)
    return dict(kind="decode", dtype=dtype, scale=1.0 / math.sqrt(d), block_size=bs,
                contexts=contexts, block_tables=table, key_cache=key_cache,
                value_cache=value_cache, query=query, k_new=k_new, v_new=v_new, slots=slots)


def prefill_case(seed, q_lens, contexts, hq, hkv, d, bs, nb, dtype, pool_scale=1.0, table=None,
                 fill="normal"):
    """Store each request's chunk at its positions, then paged causal prefill."""
    rng = np.random.default_rng(seed)
    q_lens = np.asarray(q_lens, dtype=np.int32)
    contexts = np.asarray(contexts, dtype=np.int32)
    if table is None:
        table = _tables(rng, contexts, bs, nb)
    if fill == "poison":  # unused slots hold K=1000 / V=-1000 as in the reference tests
        key_cache = _cast(np.full((nb, bs, hkv, d), 1000.0), dtype)
        value_cache = _cast(np.full((nb, bs, hkv, d), -1000.0), dtype)
        for r, c in enumerate(contexts):
            for pos in range(int(c) - int(q_lens[r])):
                b = table[r, pos // bs]
                key_cache[b, pos % bs] = _normal(rng, (hkv, d), dtype)
                value_cache[b, pos % bs] = _normal(rng, (hkv, d), dtype)
    else:
        key_cache = _normal(rng, (nb, bs, hkv, d), dtype, pool_scale)
        value_cache = _normal(rng, (nb, bs, hkv, d), dtype, pool_scale)
    total = int(q_lens.sum())
    query = _normal(rng, (total, hq, d), dtype)
    k_new = _normal(rng, (total, hkv, d), dtype)
    v_new = _normal(rng, (total, hkv, d), dtype)
    slots = []
    for r in range(len(contexts)):
        p0 = int(contexts[r]) - int(q_lens[r])
        slots.extend(_slot(table[r], p0 + i, bs) for i in range(int(q_lens[r])))
    cu_q = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(contexts)]).astype(np.int32)
    return dict(kind="prefill", dtype=dtype, scale=1.0 / math.sqrt(d), block_size=bs,
                contexts=contexts, q_lens=q_lens, cu_seqlens_q=cu_q, cu_seqlens_k=cu_k,
                block_tables=table, key_cache=key_cache, value_cache=value_cache, query=query,
                k_new=k_new, v_new=v_new, slots=np.asarray(slots, dtype=np.int32))


def direct_case(seed, lengths, hq, hkv, d, dtype):
    rng = np.random.default_rng(seed)
    lengths = np.asarray(lengths, dtype=np.int32)
    total = int(lengths.sum())
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    return dict(kind="direct", dtype=dtype, scale=1.0 / math.sqrt(d), cu_seqlens=cu,
                query=_normal(rng, (total, hq, d), dtype), keys=_normal(rng, (total, hkv, d), dtype),
                values=_normal(rng, (total, hkv, d), dtype))


def cow_case(seed, layers, nb, bs, hkv, d, dtype, pairs):
    rng = np.random.default_rng(seed)
    return dict(kind="cow", dtype=dtype, key_pool=_normal(rng, (layers, nb, bs, hkv, d), dtype),
                value_pool=_normal(rng, (layers, nb, bs, hkv, d), dtype),
                pairs=np.asarray(pairs, dtype=np.int32))


def write_checked_case(seed, dtype="f32"):
    """Padding (-1) slots interleaved with valid ones, non-contiguous blocks."""
    rng = np.random.default_rng(seed)
    nb, bs, hkv, d = 6, 4, 2, 8
    slots = np.array([9, -1, 3, 22, -1, 0, 17], dtype=np.int64)
    return dict(kind="write_checked", dtype=dtype,
                key_cache=_cast(np.full((nb, bs, hkv, d), -5.0), dtype),
                value_cache=_cast(np.full((nb, bs, hkv, d), -6.0), dtype),
                slots=slots, keys=_normal(rng, (len(slots), hkv, d), dtype),
                values=_normal(rng, (len(slots), hkv, d), dtype))


def _reversed_table(n, width):
    phys = list(range(n * width))[::-1]
    return np.array([phys[r * width:(r + 1) * width] for r in range(n)], dtype=np.int32)


def build(name: str) -> dict:
    """Rebuild case `name` (see CASES)."""
    if name == "cfg1_decode_f32":
        # batch 4, 16q/8kv, D128, bs16, nb64, ctx U[1,256], seed 0.
        return decode_case(0, 4, 16, 8, 128, 16, 64, 1, 256, "f32")
    if name == "cfg2_layer_bf16":
        # BASELINE config 2, one layer: batch 8, ctx U[128,512], nb1024, pool N(0,1)*0.5.
        return decode_case(2, 8, 16, 8, 128, 16, 1024, 128, 512, "bf16", pool_scale=0.5)
    if name == "cfg5b_slice_bf16":
        # Long single sequence with the 8B head shape (split-K path), shortened.
        return decode_case(5, 1, 32, 8, 128, 16, 512, 6000, 8000, "bf16", pool_scale=0.5)
    if name.startswith("decode_bs"):
        # tests/layers/test_triton_paged_attention.py:14-76 shapes: N=2, 4q/2kv,
        # D32, contexts [5, bs+3], reversed physical block order.
        bs, dtype = name[len("decode_bs"):].split("_")
        bs = int(bs)
        contexts = [5, bs + 3]
        width = (max(contexts) + bs - 1) // bs
        return decode_case(14, 2, 4, 2, 32, bs, 2 * width, 0, 0, dtype, contexts=contexts,
                           table=_reversed_table(2, width))
    if name.startswith("prefill_bs"):
        # tests/layers/test_triton_paged_attention.py:80-145 shapes: contexts
        # [bs+5, 2bs+9], q_lens [19, 7], 4q/2kv, D32, flipped tables.
        bs, dtype = name[len("prefill_bs"):].split("_")
        bs = int(bs)
        contexts = [bs + 5, 2 * bs + 9]
        width = max((c + bs - 1) // bs for c in contexts)
        table = np.arange(2 * width, dtype=np.int32).reshape(2, width)[:, ::-1].copy()
        return prefill_case(80, [19, 7], contexts, 4, 2, 32, bs, 2 * width, dtype, table=table)
    if name == "prefill_poison_bf16":
        # tests/components/test_paged_attention.py:106-162: bs16, 8q/2kv, D32,
        # contexts [33, 17], q_lens [16, 5], tables [[5,1,3],[0,4,2]], poison fill.
        table = np.array([[5, 1, 3], [0, 4, 2]], dtype=np.int32)
        return prefill_case(106, [16, 5], [33, 17], 8, 2, 32, 16, 6, "bf16", table=table,
                            fill="poison")
    if name == "mixed_bf16":
        # Reduced BASELINE config 3: 6 decode requests + 2 prefill chunks, one launch.
        rng = np.random.default_rng(3)
        dec = rng.integers(1, 300, size=6)
        pre_q = np.array([40, 77])
        pre_p = rng.integers(0, 200, size=2)
        q_lens = np.concatenate([np.ones(6, dtype=np.int64), pre_q])
        contexts = np.concatenate([dec, pre_q + pre_p])
        return prefill_case(33, q_lens, contexts, 16, 8, 128, 16, 128, "bf16", pool_scale=0.5)
    if name == "prefix_bf16":
        # Reduced BASELINE config 4: 4 requests whose tables share 4 prefix
        # blocks, each with a 24-token private suffix prefilled on top.
        bs, prefix, suffix, n = 16, 64, 24, 4
        shared = [0, 1, 2, 3]
        table = np.full((n, 6), -1, dtype=np.int32)
        nxt = 4
        for r in range(n):
            table[r, :4] = shared
            table[r, 4:6] = [nxt, nxt + 1]
            nxt += 2
        return prefill_case(44, [suffix] * n, [prefix + suffix] * n, 16, 8, 128, bs, 16, "bf16",
                            pool_scale=0.5, table=table)
    if name.startswith("tc_prefill_g"):
        # Tensor-core prefill shapes: D=128, 2 kv heads, chunks spanning several
        # 128-row query tiles and 128-key tiles, prefixes off tile boundaries,
        # plus a single-token (decode) row in the same launch.
        g, dtype = name[len("tc_prefill_g"):].split("_")
        g = int(g)
        q_lens = [200, 37, 1, 129]
        contexts = [200 + 200, 37 + 5, 1 + 130, 129]
        return prefill_case(90 + g, q_lens, contexts, g, 1, 128, 16, 64, dtype, pool_scale=0.5)
    if name.startswith("tc_prefill_bs"):
        bs, dtype = name[len("tc_prefill_bs"):].split("_")
        bs = int(bs)
        q_lens = [150, 40]
        contexts = [150 + 3 * bs + 7, 40 + 100]
        nb = sum((c + bs - 1) // bs for c in contexts) + 2
        return prefill_case(70 + bs, q_lens, contexts, 2, 1, 128, bs, nb, dtype, pool_scale=0.5)
    if name == "tc_dense_g4_bf16":
        return direct_case(57, [129, 64, 1, 100], 4, 1, 128, "bf16")
    if name == "direct_bf16":
        return direct_case(55, [5, 17, 33, 1], 16, 8, 128, "bf16")
    if name == "direct_f32":
        return direct_case(56, [3, 9, 2], 4, 2, 32, "f32")
    if name == "cow_bf16":
        return cow_case(66, 3, 12, 16, 8, 128, "bf16", [[3, 7], [0, 11], [5, 2]])
    if name == "write_checked_f32":
        return write_checked_case(77)
    raise KeyError(name)


DECODE_REF_CASES = [f"decode_bs{bs}_{dt}" for bs in (16, 32, 64, 128, 256)
                    for dt in ("f32", "f16", "bf16")]
PREFILL_REF_CASES = [f"prefill_bs{bs}_{dt}" for bs in (16, 64) for dt in ("f16", "bf16")]
TC_PREFILL_CASES = (["tc_prefill_g1_bf16", "tc_prefill_g2_bf16", "tc_prefill_g2_f16",
                     "tc_prefill_g4_bf16", "tc_prefill_g4_f16", "tc_prefill_g8_bf16"]
                    + [f"tc_prefill_bs{bs}_bf16" for bs in (32, 64, 128, 256)])
CASES = (["cfg1_decode_f32", "cfg2_layer_bf16", "cfg5b_slice_bf16"] + DECODE_REF_CASES
         + PREFILL_REF_CASES + ["prefill_poison_bf16", "mixed_bf16", "prefix_bf16", "direct_bf16",
                                "direct_f32", "tc_dense_g4_bf16", "cow_bf16", "write_checked_f32"]
         + TC_PREFILL_CASES)


def kind(name: str) -> str:
    """Case kind without building its inputs."""
    if name.startswith(("cfg", "decode_")):
        return "decode"
    if name.startswith(("prefill_", "mixed_", "prefix_", "tc_prefill_")):
        return "prefill"
    if name.startswith(("direct_", "tc_dense_")):
        return "direct"
    if name.startswith("cow_"):
        return "cow"
    return "write_checked"


INPUT_KEYS = ("key_cache", "value_cache", "query", "k_new", "v_new", "slots", "block_tables",
              "contexts", "q_lens", "keys", "values", "key_pool", "value_pool", "pairs",
              "cu_seqlens")
