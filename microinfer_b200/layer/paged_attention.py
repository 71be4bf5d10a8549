"""Paged attention on the sm_100a kernels, behind the reference's backend API.

Entry points keep the reference's signatures so they drop in for its
dispatch targets:

* ``paged_decode``   <- ``triton_paged_decode``  (triton_paged_attention.py:352-457)
* ``paged_prefill``  <- ``triton_paged_prefill`` (triton_paged_attention.py:260-339)
* ``gather_paged_kv`` <- ``_gather_paged_kv``     (paged_attention.py:76-101)
* ``paged_attention_meta`` <- ``paged_attention_meta`` (paged_attention.py:188-293)

Unlike the reference there is one kernel family for every block size and
no FlashAttention, Triton or torch fallback: CPU tensors and shapes no kernel
takes raise.  Split-K decode merges its splits in the kernel (the last split
to finish merges) through one zero-filled workspace per device that the
kernels leave zeroed, so it is allocated once and reused by every launch,
CUDA graph replays included; launches on one device are expected to run one
at a time, as in the reference's single-stream engine.
"""

from __future__ import annotations

import ctypes
import math

import torch

from microinfer_b200 import _lib


def _idx(t: torch.Tensor) -> torch.Tensor:
    """Index tensors are int32 and contiguous (the reference's _index_tensor)."""
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    return t.contiguous()


_WORKSPACES: dict[int, list[torch.Tensor]] = {}


def _split_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """The device's split-K workspace, at least ``nbytes`` long and zero-filled.

    The decode kernels restore its arrival counters to zero, so it is zeroed
    only when allocated.  Outgrown buffers stay alive: a captured CUDA graph
    keeps their addresses.
    """
    bufs = _WORKSPACES.setdefault(device.index or 0, [])
    if not bufs or bufs[-1].numel() * 4 < nbytes:
        size = max(nbytes, 1 << 20)
        bufs.append(torch.zeros((size + 3) // 4, dtype=torch.float32, device=device))
    return bufs[-1]


def _check_common(query, key_cache, value_cache):
    if query.ndim != 3:
        raise ValueError("query must have shape [tokens, Hq, D]")
    if key_cache.ndim != 4 or value_cache.shape != key_cache.shape:
        raise ValueError("caches must be matching [blocks, block_size, Hkv, D] tensors")
    _, num_q_heads, head_dim = query.shape
    _, block_size, num_kv_heads, kv_dim = key_cache.shape
    if query.device != key_cache.device or query.dtype != key_cache.dtype:
        raise ValueError("query and cache must share device/dtype")
    if value_cache.dtype != key_cache.dtype or value_cache.device != key_cache.device:
        raise ValueError("key and value caches must share device/dtype")
    if query.dtype not in _lib.DTYPE_CODES:
        raise ValueError("unsupported query dtype")
    if kv_dim != head_dim:
        raise ValueError("query and cache head dimensions differ")
    if num_q_heads % num_kv_heads:
        raise ValueError("Hq must be divisible by Hkv")
    if head_dim > 256:
        raise ValueError("head_dim above 256 is not supported")
    return num_q_heads, head_dim, block_size, num_kv_heads


def select_split_k(num_requests: int, num_kv_heads: int, device=None,
                   max_context: int = 0) -> int:
    """Split count for decode: fill every SM twice with (split, kv-head, seq) CTAs.

    A launch-shape constant derived from the batch shape only (optionally a
    context bound), so a CUDA graph captured for a batch bucket stays valid
    when context lengths change on replay.
    """
    dev = 0
    if device is not None:
        dev = torch.device(device).index or 0
    return _lib.load().mi_paged_decode_default_splits(num_requests, num_kv_heads, max_context, dev)


DECODE_KERNELS = {1: "generic", 2: "simt", 4: "mma", 5: "mma_pair"}


def decode_plan(num_requests: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                dtype: torch.dtype, block_size: int, split_k: int = 0, device=None,
                table_width: int = 0):
    """(kernel name, split count, workspace bytes) the decode launch will use.

    ``split_k=0`` lets the library size the split for one wave of CTAs;
    ``table_width`` (block-table columns) bounds the context, which picks
    between the tensor-core and SIMT kernels.
    """
    dev = 0 if device is None else (torch.device(device).index or 0)
    splits = ctypes.c_int32(0)
    ws = ctypes.c_size_t(0)
    kernel = _lib.load().mi_paged_decode_plan(num_requests, num_q_heads, num_kv_heads, head_dim,
                                              _lib.dtype_code(dtype), block_size, table_width,
                                              split_k, dev, ctypes.byref(splits), ctypes.byref(ws))
    if kernel < 0:
        _lib.check(kernel)
    return DECODE_KERNELS[kernel], splits.value, ws.value


def _decode_prep(query, key_cache, value_cache, block_tables, context_lens, split_k, scale, out):
    num_q_heads, head_dim, block_size, num_kv_heads = _check_common(query, key_cache, value_cache)
    num_requests = query.shape[0]
    device = _lib.require_cuda(query, key_cache, value_cache, block_tables, context_lens)
    if block_tables.ndim != 2 or block_tables.shape[0] != num_requests:
        raise ValueError("block_tables must have one row per request")
    if context_lens.numel() != num_requests:
        raise ValueError("context_lens must have one entry per request")
    if split_k is None:
        split_k = 0
    if type(split_k) is not int or split_k < 0:
        raise ValueError("split_k must be a positive int (or None for automatic)")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("KV caches must be contiguous")
    # The library plans again from the same shapes; only the workspace size is needed
    # here, and split_k goes through as given (0 = automatic, which may pick the
    # cluster-pair kernel that needs no workspace).
    _, _, ws_bytes = decode_plan(num_requests, num_q_heads, num_kv_heads, head_dim,
                                 query.dtype, block_size, split_k, device, block_tables.shape[1])
    workspace = _split_workspace(device, ws_bytes) if ws_bytes else None
    return dict(
        query=query.contiguous(), block_tables=_idx(block_tables), context_lens=_idx(context_lens),
        out=torch.empty_like(query) if out is None else out, device=device, split_k=split_k,
        scale=1.0 / math.sqrt(head_dim) if scale is None else float(scale),
        workspace=workspace, ws_bytes=ws_bytes,
        dims=(key_cache.shape[0], block_size, num_q_heads, num_kv_heads, head_dim,
              _lib.dtype_code(query.dtype)),
    )


def paged_decode(query, key_cache, value_cache, block_tables, context_lens, *,
                 scale: float | None = None, split_k: int | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """One query token per request over its paged KV (any block size)."""
    if torch.compiler.is_compiling():  # an opaque node for torch.compile
        res = torch.ops.microinfer_b200.paged_decode(query, key_cache, value_cache, block_tables,
                                                     context_lens, scale, split_k)
        return res if out is None else out.copy_(res)
    if query.shape[0] == 0:
        return torch.empty_like(query)
    a = _decode_prep(query, key_cache, value_cache, block_tables, context_lens, split_k, scale, out)
    _lib.call(
        "mi_paged_decode", a["out"].data_ptr(), a["query"].data_ptr(), key_cache.data_ptr(),
        value_cache.data_ptr(), *a["dims"], a["block_tables"].data_ptr(),
        a["block_tables"].stride(0), a["context_lens"].data_ptr(), query.shape[0], a["scale"],
        a["split_k"], _lib.ptr(a["workspace"]), a["ws_bytes"],
        _lib.status_buffer(a["device"]).data_ptr(), _lib.stream_of(a["device"]),
    )
    return a["out"]


def paged_decode_store(query, key_cache, value_cache, block_tables, context_lens, k_new, v_new,
                       slot_mapping, *, scale: float | None = None, split_k: int | None = None,
                       out: torch.Tensor | None = None, early_kv: bool = False) -> torch.Tensor:
    """store_kvcache of this step's token fused into paged decode (one launch).

    ``k_new``/``v_new`` are ``[requests, Hkv, D]`` (inner dims contiguous);
    ``slot_mapping[r]`` (-1 = padding) must address position
    ``context_lens[r] - 1`` of request r, as the reference runner builds it.

    ``early_kv=True`` lets the launch request its cached pages before the
    preceding kernel in the stream has finished (programmatic dependent
    launch); use it only when that kernel writes neither the pool nor the
    tables/lengths (a QKV projection, or another layer's decode).
    """
    if torch.compiler.is_compiling():  # an opaque node for torch.compile
        res = torch.ops.microinfer_b200.paged_decode_store(
            query, key_cache, value_cache, block_tables, context_lens, k_new, v_new,
            slot_mapping, scale, split_k, early_kv)
        return res if out is None else out.copy_(res)
    if query.shape[0] == 0:
        return torch.empty_like(query)
    n = query.shape[0]
    if k_new.shape != (n, *key_cache.shape[2:]) or v_new.shape != k_new.shape:
        raise ValueError("k_new/v_new must be [requests, Hkv, D]")
    if k_new.dtype != key_cache.dtype or v_new.dtype != key_cache.dtype:
        raise ValueError("k_new/v_new dtype must match the cache")
    if k_new.stride(-1) != 1 or k_new.stride(-2) != k_new.shape[-1]:
        k_new = k_new.contiguous()
    if v_new.stride() != k_new.stride():
        v_new = v_new.contiguous()
        k_new = k_new.contiguous()
    if slot_mapping.shape != (n,):
        raise ValueError("slot_mapping must have one entry per request")
    _lib.require_cuda(k_new, v_new, slot_mapping)
    a = _decode_prep(query, key_cache, value_cache, block_tables, context_lens, split_k, scale, out)
    slots = _idx(slot_mapping)
    _lib.call(
        "mi_paged_decode_store", a["out"].data_ptr(), a["query"].data_ptr(), key_cache.data_ptr(),
        value_cache.data_ptr(), *a["dims"], a["block_tables"].data_ptr(),
        a["block_tables"].stride(0), a["context_lens"].data_ptr(), n, k_new.data_ptr(),
        v_new.data_ptr(), k_new.stride(0), slots.data_ptr(), a["scale"], a["split_k"],
        1 if early_kv else 0, _lib.ptr(a["workspace"]), a["ws_bytes"],
        _lib.status_buffer(a["device"]).data_ptr(),
        _lib.stream_of(a["device"]),
    )
    return a["out"]


def paged_prefill(query, key_cache, value_cache, cu_seqlens_q, cu_seqlens_k, block_tables, *,
                  max_seqlen_q: int, scale: float | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal chunked prefill straight from the paged cache; also mixed batches.

    ``cu_seqlens_k`` is cumulative over contexts (context includes the chunk),
    so request r's rows sit at positions ``context_r - q_len_r + i``.
    """
    if torch.compiler.is_compiling():  # an opaque node for torch.compile
        res = torch.ops.microinfer_b200.paged_prefill(query, key_cache, value_cache, cu_seqlens_q,
                                                      cu_seqlens_k, block_tables,
                                                      int(max_seqlen_q), scale)
        return res if out is None else out.copy_(res)
    num_q_heads, head_dim, block_size, num_kv_heads = _check_common(query, key_cache, value_cache)
    num_tokens = query.shape[0]
    num_requests = block_tables.shape[0]
    if num_tokens == 0 or num_requests == 0:
        return torch.empty_like(query)
    device = _lib.require_cuda(query, key_cache, value_cache, cu_seqlens_q, cu_seqlens_k,
                               block_tables)
    if cu_seqlens_q.numel() != num_requests + 1:
        raise ValueError("cu_seqlens_q must have num_requests + 1 entries")
    if cu_seqlens_k.numel() != num_requests + 1:
        raise ValueError("cu_seqlens_k must have num_requests + 1 entries")
    if max_seqlen_q <= 0:
        raise ValueError("max_seqlen_q must be positive")
    query = query.contiguous()
    key_cache = key_cache.contiguous()
    value_cache = value_cache.contiguous()
    cu_seqlens_q = _idx(cu_seqlens_q)
    cu_seqlens_k = _idx(cu_seqlens_k)
    block_tables = _idx(block_tables)
    if out is None:
        out = torch.empty_like(query)
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    _lib.call(
        "mi_paged_prefill", out.data_ptr(), query.data_ptr(), key_cache.data_ptr(),
        value_cache.data_ptr(), key_cache.shape[0], block_size, num_q_heads, num_kv_heads,
        head_dim, _lib.dtype_code(query.dtype), cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(),
        block_tables.data_ptr(), block_tables.stride(0), num_requests, num_tokens,
        int(max_seqlen_q), float(scale), _lib.status_buffer(device).data_ptr(),
        _lib.stream_of(device),
    )
    return out


def varlen_prefill(query, keys, values, cu_seqlens_q, cu_seqlens_k, *, max_seqlen_q: int,
                   scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal varlen attention on contiguous K/V (no cached prefix)."""
    if query.ndim != 3 or keys.ndim != 3 or values.shape != keys.shape:
        raise ValueError("query/keys/values must be [tokens, heads, D]")
    num_tokens, num_q_heads, head_dim = query.shape
    num_kv_heads = keys.shape[1]
    if keys.shape[2] != head_dim:
        raise ValueError("query and K/V head dimensions differ")
    if num_q_heads % num_kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    if query.dtype != keys.dtype or values.dtype != keys.dtype:
        raise ValueError("query and K/V must share dtype")
    num_requests = cu_seqlens_q.numel() - 1
    if num_tokens == 0 or num_requests <= 0:
        return torch.empty_like(query)
    device = _lib.require_cuda(query, keys, values, cu_seqlens_q, cu_seqlens_k)
    if cu_seqlens_k.numel() != num_requests + 1:
        raise ValueError("cu_seqlens_q and cu_seqlens_k lengths differ")
    query = query.contiguous()
    if keys.stride(-1) != 1 or keys.stride(-2) != head_dim:
        keys = keys.contiguous()
    if values.stride(-1) != 1 or values.stride(-2) != head_dim or values.stride(0) != keys.stride(0):
        values = values.contiguous()
        keys = keys.contiguous()
    cu_seqlens_q = _idx(cu_seqlens_q)
    cu_seqlens_k = _idx(cu_seqlens_k)
    if out is None:
        out = torch.empty_like(query)
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    _lib.call(
        "mi_varlen_prefill", out.data_ptr(), query.data_ptr(), keys.data_ptr(), values.data_ptr(),
        keys.stride(0), num_q_heads, num_kv_heads, head_dim, _lib.dtype_code(query.dtype),
        cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), num_requests, num_tokens,
        keys.shape[0], int(max_seqlen_q), float(scale), _lib.status_buffer(device).data_ptr(),
        _lib.stream_of(device),
    )
    return out


def gather_paged_kv(key_cache, value_cache, block_tables, contexts, block_size,
                    *, cu_seqlens_k: torch.Tensor | None = None, out=None):
    """Valid rows of each request in logical order, concatenated request-major.

    ``contexts`` is a host sequence of context lengths (the reference's
    argument); pass ``cu_seqlens_k`` (device, cumulative) to skip the host
    prefix sum and its copy, and ``out=(keys, values)`` (contiguous
    ``[sum(contexts), Hkv, D]``) to write into existing tensors.
    """
    if key_cache.ndim != 4 or value_cache.shape != key_cache.shape:
        raise ValueError("caches must be matching [blocks, block_size, Hkv, D] tensors")
    if block_size != key_cache.shape[1]:
        raise ValueError("block_size does not match the cache")
    device = _lib.require_cuda(key_cache, value_cache, block_tables)
    contexts = [int(c) for c in contexts]
    if any(c < 0 for c in contexts):
        raise ValueError("contexts must be non-negative")
    if len(contexts) != block_tables.shape[0]:
        raise ValueError("one context per block-table row")
    total = sum(contexts)
    _, _, num_kv_heads, head_dim = key_cache.shape
    if out is None:
        keys = torch.empty((total, num_kv_heads, head_dim), dtype=key_cache.dtype, device=device)
        values = torch.empty_like(keys)
    else:
        keys, values = out
        want = (total, num_kv_heads, head_dim)
        if (tuple(keys.shape) != want or tuple(values.shape) != want
                or keys.dtype != key_cache.dtype or values.dtype != key_cache.dtype
                or not (keys.is_contiguous() and values.is_contiguous())):
            raise ValueError("out must be two contiguous [sum(contexts), Hkv, D] tensors of "
                             "the cache dtype")
        _lib.require_cuda(keys, values)
    if total == 0:
        return keys, values
    if cu_seqlens_k is None:
        cu = [0]
        for c in contexts:
            cu.append(cu[-1] + c)
        cu_seqlens_k = torch.tensor(cu, dtype=torch.int32).to(device, non_blocking=True)
    cu_seqlens_k = _idx(cu_seqlens_k)
    block_tables = _idx(block_tables)
    key_cache = key_cache.contiguous()
    value_cache = value_cache.contiguous()
    _lib.call(
        "mi_gather_paged_kv", keys.data_ptr(), values.data_ptr(), key_cache.data_ptr(),
        value_cache.data_ptr(), key_cache.shape[0], block_size, num_kv_heads, head_dim,
        _lib.dtype_code(key_cache.dtype), block_tables.data_ptr(), block_tables.stride(0),
        cu_seqlens_k.data_ptr(), len(contexts), total, max(contexts),
        _lib.status_buffer(device).data_ptr(), _lib.stream_of(device),
    )
    return keys, values


def paged_attention_meta(query, key_cache, value_cache, metadata, *,
                         scale: float | None = None) -> torch.Tensor:
    """Backend dispatch on validated metadata; no host validation or tolist on decode.

    Decode (one query per request) goes to the split-K decode kernels; every
    prefill with a block table (chunked, prefix-hit or mixed) to the paged
    prefill kernels.
    """
    if query.shape[0] == 0:
        return torch.empty_like(query)
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    block_tables = metadata.block_tables
    if block_tables is None:
        raise ValueError("paged attention needs metadata.block_tables")
    if metadata.is_decode and metadata.context_lens is not None:
        return paged_decode(query, key_cache, value_cache, block_tables,
                            metadata.context_lens, scale=scale)
    cu_q, cu_k = metadata.cu_seqlens_q, metadata.cu_seqlens_k
    if cu_q is None:
        cu_q = torch.tensor(metadata.cu_q_cpu, dtype=torch.int32, device=query.device)
    if cu_k is None:
        if metadata.context_lens is None:
            raise ValueError("metadata needs cu_seqlens_k or context_lens")
        cu_k = torch.zeros(metadata.context_lens.numel() + 1, dtype=torch.int32,
                           device=query.device)
        torch.cumsum(metadata.context_lens, 0, out=cu_k[1:])
    max_q = metadata.max_seqlen_q or max(metadata.q_lens_cpu, default=0)
    return paged_prefill(query, key_cache, value_cache, cu_q, cu_k, block_tables,
                         max_seqlen_q=max_q, scale=scale)
