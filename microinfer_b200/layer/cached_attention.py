"""Per-layer attention over one layer's KV cache (store, then attend).

Mirrors ``CachedAttention`` (microinfer/layer/cached_attention.py:58-101):
the step's K/V are written into the paged pool first, then the queries
attend.  Prefill without a block table ("direct", no cached prefix) attends
to this step's contiguous K/V with the dense varlen kernel, which replaces the
reference's FlashAttention varlen / per-request SDPA paths (:17-55).
"""

from __future__ import annotations

import torch
from torch import nn

from microinfer_b200.layer.paged_attention import (
    paged_attention_meta,
    paged_decode_store,
    varlen_prefill,
)
from microinfer_b200.worker.kv_cache import LayerKVCache


class CachedAttention(nn.Module):
    def __init__(self):
        super().__init__()
        self.cache: LayerKVCache | None = None

    def bind_cache(self, cache: LayerKVCache):
        self.cache = cache

    def forward(self, q, k, v, metadata):
        """Q/K already normalised and rotated; returns [T, Hq, D]."""
        cache = self.cache
        direct = metadata.direct_prefill if metadata.is_prefill else False
        if not direct and (cache is None or metadata.block_tables is None):
            raise RuntimeError("paged attention requires a bound layer cache and block table")
        if cache is not None:
            if metadata.slot_mapping is None:
                raise ValueError("bound cache requires slot_mapping")
            if (metadata.is_decode and not metadata.validate_cache_write
                    and metadata.context_lens is not None):
                # One launch: store this step's K/V, then decode over the cache.
                return paged_decode_store(q, cache.keys, cache.values, metadata.block_tables,
                                          metadata.context_lens, k, v, metadata.slot_mapping)
            if metadata.validate_cache_write:
                cache.write_checked(metadata.slot_mapping, k, v)
            else:
                cache.write_slots(metadata.slot_mapping, k, v)
        if not direct:
            return paged_attention_meta(q, cache.keys, cache.values, metadata)
        if q.shape[1] % k.shape[1]:
            raise ValueError("query heads must be divisible by KV heads")
        cu_q = metadata.cu_seqlens_q
        cu_k = metadata.cu_seqlens_k if metadata.cu_seqlens_k is not None else cu_q
        if cu_q is None:
            cu_q = cu_k = torch.tensor([0, q.shape[0]], dtype=torch.int32, device=q.device)
        max_q = metadata.max_seqlen_q or max(metadata.q_lens_cpu, default=0)
        return varlen_prefill(q, k, v, cu_q, cu_k, max_seqlen_q=max_q)
