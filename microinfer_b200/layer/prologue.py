"""Attention prologue: q/k RMSNorm + RoPE + store of k/v, in one launch.

Replaces, in the attention forward of the reference model, the steps between the
QKV projection and paged attention: ``q_norm`` / ``k_norm`` (FuseLayerNorm,
microinfer/layer/transformer.py:222-223, layer/norm.py), ``RotaryCache.apply``
on q and k (transformer.py:224-225, layer/rope.py:6-21, 75-84) and the store of
k/v into the pool that ``CachedAttention`` does before attending
(layer/cached_attention.py:76-85).  Results follow the reference's eager ops
rounding point by rounding point (one rounding after the norm, fp32 rotation
with separately rounded products and sums, one more rounding).
"""
from __future__ import annotations

import torch

from microinfer_b200 import _lib


def qk_norm_rope_store(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                       positions: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor,
                       key_cache: torch.Tensor, value_cache: torch.Tensor,
                       slot_mapping: torch.Tensor, *, num_q_heads: int, num_kv_heads: int,
                       eps: float, interleaved: bool = False,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """Normalise and rotate q and k of the packed projection ``qkv``
    ([T, (Hq + 2 Hkv) * D] or [T, Hq + 2 Hkv, D]), store k and v at
    ``slot_mapping`` (int32, -1 = no store) of the pool ([blocks, block_size,
    Hkv, D]) and return q as [T, Hq, D].  ``cos_table``/``sin_table`` are the
    model's fp32 RotaryCache tables [max_positions, D / 2]; ``positions`` int32
    or int64."""
    if torch.compiler.is_compiling():  # an opaque node for torch.compile
        res = torch.ops.microinfer_b200.qk_norm_rope_store(
            qkv, q_weight, k_weight, positions, cos_table, sin_table, key_cache, value_cache,
            slot_mapping, num_q_heads, num_kv_heads, float(eps), bool(interleaved))
        return res if out is None else out.copy_(res)
    tokens = qkv.shape[0]
    if key_cache.ndim != 4 or value_cache.shape != key_cache.shape:
        raise ValueError("caches must be matching [blocks, block_size, Hkv, D] tensors")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("KV cache views must be contiguous")
    nb, bs, hkv, d = key_cache.shape
    if hkv != num_kv_heads or num_q_heads % num_kv_heads:
        raise ValueError("head counts do not match the cache")
    heads = num_q_heads + 2 * num_kv_heads
    flat = qkv.reshape(tokens, heads * d) if qkv.ndim == 3 else qkv
    if flat.ndim != 2 or flat.shape[1] != heads * d or flat.stride(1) != 1:
        raise ValueError("qkv must be [T, (Hq + 2 Hkv) * D] with contiguous rows")
    dt = key_cache.dtype
    if flat.dtype != dt or q_weight.dtype != dt or k_weight.dtype != dt:
        raise ValueError("qkv, norm weights and cache must share a dtype")
    if q_weight.shape != (d,) or k_weight.shape != (d,):
        raise ValueError("norm weights must be [head_dim]")
    if cos_table.dtype != torch.float32 or sin_table.shape != cos_table.shape or \
            cos_table.ndim != 2 or cos_table.shape[1] != d // 2:
        raise ValueError("cos/sin tables must be fp32 [max_positions, head_dim / 2]")
    if positions.shape != (tokens,) or positions.dtype not in (torch.int32, torch.int64):
        raise ValueError("positions must be int32/int64 with one entry per token")
    if slot_mapping.shape != (tokens,) or slot_mapping.dtype != torch.int32:
        raise ValueError("slot_mapping must be int32 with one entry per token")
    if out is None:
        out = torch.empty(tokens, num_q_heads, d, dtype=dt, device=flat.device)
    elif out.shape != (tokens, num_q_heads, d) or out.dtype != dt or out.stride(2) != 1 or \
            out.stride(1) != d:
        raise ValueError("out must be [T, Hq, D] with contiguous rows")
    if tokens == 0:
        return out
    device = _lib.require_cuda(flat, q_weight, k_weight, positions, cos_table, sin_table,
                               key_cache, value_cache, slot_mapping, out)
    q_weight, k_weight = q_weight.contiguous(), k_weight.contiguous()
    positions, slot_mapping = positions.contiguous(), slot_mapping.contiguous()
    cos_table, sin_table = cos_table.contiguous(), sin_table.contiguous()
    _lib.call(
        "mi_qk_norm_rope_store",
        out.data_ptr(), out.stride(0), flat.data_ptr(), flat.stride(0), q_weight.data_ptr(),
        k_weight.data_ptr(), float(eps), positions.data_ptr(), _lib.index_code(positions.dtype),
        cos_table.data_ptr(), sin_table.data_ptr(), cos_table.shape[0], int(bool(interleaved)),
        slot_mapping.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), nb, bs, tokens,
        num_q_heads, num_kv_heads, d, _lib.dtype_code(dt),
        _lib.status_buffer(device).data_ptr(), _lib.stream_of(device),
    )
    return out
