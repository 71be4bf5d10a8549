"""Runner-owned paged KV pool and its per-layer views, on the sm_100a kernels.

Same API as the reference's ``KVCache`` / ``LayerKVCache``
(microinfer/worker/kv_cache.py:11-118): the pool is two zero-initialised
tensors ``[layers, blocks, block_size, Hkv, D]`` and a layer view is a basic
slice (no copy).  ``write_checked`` keeps the reference's host validation
(-1 padding, range and duplicate checks before anything is written,
kv_cache.py:30-50) and then stores on the device; ``write_fast`` is the
unchecked hot path (kv_cache.py:52-79).  ``KVCache.copy_blocks`` adds the
device-side copy-on-write of whole pages, which the reference lacks.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from microinfer_b200 import _lib
from microinfer_b200.worker.kv_store import store_kv, store_kv_slots


@dataclass(frozen=True)
class LayerKVCache:
    """Only this layer's [blocks, B, Hkv, D] tensors; no pool or layer id."""

    keys: torch.Tensor
    values: torch.Tensor

    def __post_init__(self):
        if self.keys.ndim != 4 or self.keys.shape != self.values.shape:
            raise ValueError("K/V must have matching [blocks, B, Hkv, D] shapes")
        if self.keys.dtype != self.values.dtype or self.keys.device != self.values.device:
            raise ValueError("K/V must have matching dtype and device")

    @property
    def block_size(self) -> int:
        return self.keys.shape[1]

    def write_checked(self, slots, keys, values):
        """Validate every slot first (-1 skips), then write; invalid input writes nothing."""
        if slots.ndim != 1 or slots.dtype not in (torch.int32, torch.int64):
            raise ValueError("slots must be a 1-D integer tensor")
        expected = (slots.numel(), *self.keys.shape[2:])
        if tuple(keys.shape) != expected or tuple(values.shape) != expected:
            raise ValueError("K/V shape must match slots and cache heads")
        if any(t.device != self.keys.device for t in (slots, keys, values)):
            raise ValueError("slots and K/V must be on the cache device")
        capacity = self.keys.shape[0] * self.block_size
        if torch.any(slots < -1) or torch.any(slots >= capacity):
            raise ValueError("slot outside cache")
        valid = slots[slots >= 0]
        if valid.unique().numel() != valid.numel():
            raise ValueError("duplicate slot")
        keys = keys.to(self.keys.dtype)
        values = values.to(self.values.dtype)
        if keys.stride(-1) != 1 or keys.stride(-2) != keys.shape[-1]:
            keys = keys.contiguous()
        if values.stride(-1) != 1 or values.stride(-2) != values.shape[-1]:
            values = values.contiguous()
        store_kv_slots(self.keys, self.values, slots, keys, values)

    def write_fast(self, blocks, offsets, keys, values):
        """Hot path: caller guarantees valid, unique slots and matching dtype."""
        store_kv(self.keys, self.values, blocks, offsets, keys, values, self.block_size)

    def write_slots(self, slots, keys, values):
        """Hot path from flat slot ids (-1 = padding), split on the device."""
        store_kv_slots(self.keys, self.values, slots, keys, values)


class KVCache:
    def __init__(self, num_layers, num_blocks, block_size, num_kv_heads, head_dim, *,
                 dtype=torch.float32, device="cuda"):
        dimensions = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
        if any(d <= 0 for d in dimensions):
            raise ValueError("cache dimensions must be positive")
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        self.keys = torch.zeros(dimensions, dtype=dtype, device=device)
        self.values = torch.zeros_like(self.keys)

    @property
    def num_bytes(self) -> int:
        return self.keys.numel() * self.keys.element_size() * 2

    def layer(self, index: int) -> LayerKVCache:
        if not 0 <= index < self.num_layers:
            raise ValueError("layer outside cache")
        return LayerKVCache(self.keys[index], self.values[index])

    def copy_blocks(self, pairs, *, check: bool = True):
        """Copy-on-write: page src -> dst in every layer, for K and V.

        ``pairs`` is ``[P, 2]`` (src, dst).  With ``check`` the ids are
        validated on the host first (range, unique destinations, no
        destination that is also a source); the kernel itself range-checks
        every id and skips bad ones.
        """
        copy_blocks(self.keys, self.values, pairs, check=check)


def copy_blocks(key_pool: torch.Tensor, value_pool: torch.Tensor, pairs, *, check: bool = True):
    """Device-side copy of pages ``pairs[:, 0] -> pairs[:, 1]`` across all layers."""
    if key_pool.ndim != 5 or value_pool.shape != key_pool.shape:
        raise ValueError("pools must be matching [layers, blocks, bs, Hkv, D] tensors")
    if not (key_pool.is_contiguous() and value_pool.is_contiguous()):
        raise ValueError("pools must be contiguous")
    device = _lib.require_cuda(key_pool, value_pool)
    pairs = torch.as_tensor(pairs, dtype=torch.int32)
    if pairs.numel() == 0:
        return
    if pairs.ndim != 2 or pairs.shape[1] != 2:
        raise ValueError("pairs must have shape [P, 2]")
    num_layers, num_blocks = key_pool.shape[:2]
    if check:
        host = pairs.cpu()
        if torch.any(host < 0) or torch.any(host >= num_blocks):
            raise ValueError("block id outside the pool")
        src, dst = host[:, 0], host[:, 1]
        if dst.unique().numel() != dst.numel():
            raise ValueError("duplicate destination block")
        if torch.isin(dst, src).any():
            raise ValueError("a destination block is also a source")
    pairs = pairs.to(device).contiguous()
    block_bytes = key_pool[0, 0].numel() * key_pool.element_size()
    layer_stride = key_pool.stride(0) * key_pool.element_size()
    _lib.call(
        "mi_copy_blocks", key_pool.data_ptr(), value_pool.data_ptr(), num_layers, layer_stride,
        num_blocks, block_bytes, pairs.data_ptr(), pairs.shape[0],
        _lib.status_buffer(device).data_ptr(), _lib.stream_of(device),
    )
