"""The hot-path entry points as ``torch.library`` custom ops, so ``torch.compile``
traces them as opaque nodes.

The reference compiles its decode forward (``ModelRunner``, microinfer/runner.py:
88-100, ``torch.compile(model.forward, dynamic=True)``) and its kernels must stay
traceable there.  A ctypes call cannot be traced, so each public function of
this package, when it runs under tracing (``torch.compiler.is_compiling()``),
calls the matching ``torch.ops.microinfer_b200.*`` op instead; the op's real
implementation is the same public function run eagerly, and its fake
implementation gives the output's shape and dtype (outputs are shaped like the
query, caches are mutated in place).  Eager calls never go through the op
dispatcher.
"""
from __future__ import annotations

import torch

from microinfer_b200.layer import paged_attention as _pa
from microinfer_b200.layer import prologue as _pro
from microinfer_b200.worker import kv_store as _store

_NS = "microinfer_b200"


@torch.library.custom_op(f"{_NS}::store_kv", mutates_args=("key_cache", "value_cache"))
def store_kv(key_cache: torch.Tensor, value_cache: torch.Tensor, blocks: torch.Tensor,
             offsets: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
             block_size: int) -> None:
    _store.store_kv(key_cache, value_cache, blocks, offsets, keys, values, block_size)


@store_kv.register_fake
def _(key_cache, value_cache, blocks, offsets, keys, values, block_size):
    return None


@torch.library.custom_op(f"{_NS}::store_kv_slots", mutates_args=("key_cache", "value_cache"))
def store_kv_slots(key_cache: torch.Tensor, value_cache: torch.Tensor, slots: torch.Tensor,
                   keys: torch.Tensor, values: torch.Tensor) -> None:
    _store.store_kv_slots(key_cache, value_cache, slots, keys, values)


@store_kv_slots.register_fake
def _(key_cache, value_cache, slots, keys, values):
    return None


@torch.library.custom_op(f"{_NS}::paged_decode", mutates_args=())
def paged_decode(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 block_tables: torch.Tensor, context_lens: torch.Tensor,
                 scale: float | None = None, split_k: int | None = None) -> torch.Tensor:
    return _pa.paged_decode(query, key_cache, value_cache, block_tables, context_lens,
                            scale=scale, split_k=split_k)


@paged_decode.register_fake
def _(query, key_cache, value_cache, block_tables, context_lens, scale=None, split_k=None):
    return torch.empty_like(query)


@torch.library.custom_op(f"{_NS}::paged_decode_store", mutates_args=("key_cache", "value_cache"))
def paged_decode_store(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                       block_tables: torch.Tensor, context_lens: torch.Tensor,
                       k_new: torch.Tensor, v_new: torch.Tensor, slot_mapping: torch.Tensor,
                       scale: float | None = None, split_k: int | None = None,
                       early_kv: bool = False) -> torch.Tensor:
    return _pa.paged_decode_store(query, key_cache, value_cache, block_tables, context_lens,
                                  k_new, v_new, slot_mapping, scale=scale, split_k=split_k,
                                  early_kv=early_kv)


@paged_decode_store.register_fake
def _(query, key_cache, value_cache, block_tables, context_lens, k_new, v_new, slot_mapping,
      scale=None, split_k=None, early_kv=False):
    return torch.empty_like(query)


@torch.library.custom_op(f"{_NS}::paged_prefill", mutates_args=())
def paged_prefill(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                  cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                  block_tables: torch.Tensor, max_seqlen_q: int,
                  scale: float | None = None) -> torch.Tensor:
    return _pa.paged_prefill(query, key_cache, value_cache, cu_seqlens_q, cu_seqlens_k,
                             block_tables, max_seqlen_q=max_seqlen_q, scale=scale)


@paged_prefill.register_fake
def _(query, key_cache, value_cache, cu_seqlens_q, cu_seqlens_k, block_tables, max_seqlen_q,
      scale=None):
    return torch.empty_like(query)


@torch.library.custom_op(f"{_NS}::qk_norm_rope_store", mutates_args=("key_cache", "value_cache"))
def qk_norm_rope_store(qkv: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                       positions: torch.Tensor, cos_table: torch.Tensor,
                       sin_table: torch.Tensor, key_cache: torch.Tensor,
                       value_cache: torch.Tensor, slot_mapping: torch.Tensor, num_q_heads: int,
                       num_kv_heads: int, eps: float, interleaved: bool = False) -> torch.Tensor:
    return _pro.qk_norm_rope_store(qkv, q_weight, k_weight, positions, cos_table, sin_table,
                                   key_cache, value_cache, slot_mapping,
                                   num_q_heads=num_q_heads, num_kv_heads=num_kv_heads, eps=eps,
                                   interleaved=interleaved)


@qk_norm_rope_store.register_fake
def _(qkv, q_weight, k_weight, positions, cos_table, sin_table, key_cache, value_cache,
      slot_mapping, num_q_heads, num_kv_heads, eps, interleaved=False):
    return qkv.new_empty((qkv.shape[0], num_q_heads, key_cache.shape[-1]))
