"""store_kvcache: append this step's K/V rows into paged pool slots.

``store_kv`` keeps the signature of the reference's Triton launcher
(microinfer/worker/triton_kv_store.py:45-78) so ``LayerKVCache.write_fast``
can call it unchanged; ``store_kv_slots`` takes flat slot ids and splits them
on the device (the reference computes the split per step in
``AttentionMetadata.slot_indices``, microinfer/layer/metadata.py:75-84).
"""

from __future__ import annotations

import torch

from microinfer_b200 import _lib

# The reference gates its fast path on this module flag (kv_cache.py:7, :59).
HAS_KERNEL = True


def _check_kv_rows(keys: torch.Tensor, values: torch.Tensor) -> None:
    if keys.ndim != 3 or values.shape != keys.shape:
        raise ValueError("K/V shapes differ")
    head_dim = keys.shape[-1]
    if keys.stride(-1) != 1 or keys.stride(-2) != head_dim:
        raise ValueError("K/V inner dimensions must be contiguous")
    if values.stride(-1) != 1 or values.stride(-2) != head_dim:
        raise ValueError("V inner dimensions must be contiguous")


def _check_cache(key_cache: torch.Tensor, value_cache: torch.Tensor, keys: torch.Tensor) -> None:
    if key_cache.ndim != 4 or value_cache.shape != key_cache.shape:
        raise ValueError("caches must be matching [blocks, block_size, Hkv, D] tensors")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("KV cache views must be contiguous")
    if tuple(keys.shape[1:]) != tuple(key_cache.shape[2:]):
        raise ValueError("K/V heads do not match the cache")
    if keys.dtype != key_cache.dtype or value_cache.dtype != key_cache.dtype:
        raise ValueError("K/V dtype must match the cache")


def store_kv(key_cache, value_cache, blocks, offsets, keys, values, block_size: int):
    """cache[blocks[t], offsets[t]] = keys[t] (and values); unique slots assumed."""
    if torch.compiler.is_compiling():  # an opaque node for torch.compile
        torch.ops.microinfer_b200.store_kv(key_cache, value_cache, blocks, offsets, keys, values,
                                           block_size)
        return
    _check_kv_rows(keys, values)
    _check_cache(key_cache, value_cache, keys)
    if block_size != key_cache.shape[1]:
        raise ValueError("block_size does not match the cache")
    tokens = keys.shape[0]
    if blocks.shape != (tokens,) or offsets.shape != (tokens,):
        raise ValueError("blocks/offsets must have one entry per token")
    if tokens == 0:
        return
    device = _lib.require_cuda(key_cache, value_cache, blocks, offsets, keys, values)
    if blocks.dtype != offsets.dtype:
        offsets = offsets.to(blocks.dtype)
    blocks = blocks.contiguous()
    offsets = offsets.contiguous()
    _, bs, hkv, d = key_cache.shape
    _lib.call(
        "mi_store_kv",
        key_cache.data_ptr(), value_cache.data_ptr(), key_cache.shape[0], bs, hkv, d,
        _lib.dtype_code(key_cache.dtype), blocks.data_ptr(), offsets.data_ptr(),
        _lib.index_code(blocks.dtype), keys.data_ptr(), values.data_ptr(),
        keys.stride(0), values.stride(0), tokens,
        _lib.status_buffer(device).data_ptr(), _lib.stream_of(device),
    )


def store_kv_slots(key_cache, value_cache, slots, keys, values):
    """cache[slot // bs, slot % bs] = keys[t] (and values); slot -1 writes nothing."""
    if torch.compiler.is_compiling():  # an opaque node for torch.compile
        torch.ops.microinfer_b200.store_kv_slots(key_cache, value_cache, slots, keys, values)
        return
    _check_kv_rows(keys, values)
    _check_cache(key_cache, value_cache, keys)
    tokens = keys.shape[0]
    if slots.shape != (tokens,):
        raise ValueError("slots must have one entry per token")
    if tokens == 0:
        return
    device = _lib.require_cuda(key_cache, value_cache, slots, keys, values)
    slots = slots.contiguous()
    _, bs, hkv, d = key_cache.shape
    _lib.call(
        "mi_store_kv_slots",
        key_cache.data_ptr(), value_cache.data_ptr(), key_cache.shape[0], bs, hkv, d,
        _lib.dtype_code(key_cache.dtype), slots.data_ptr(), _lib.index_code(slots.dtype),
        keys.data_ptr(), values.data_ptr(), keys.stride(0), values.stride(0), tokens,
        _lib.status_buffer(device).data_ptr(), _lib.stream_of(device),
    )
