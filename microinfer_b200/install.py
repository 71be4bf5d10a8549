"""Drop the sm_100a kernels into a live ``microinfer`` import.

The reference looks its kernels up as module globals, so rebinding them is
enough for ``microinfer/layer`` and ``runner.py`` to run unchanged:

* ``microinfer.worker.kv_cache.store_kv`` / ``HAS_TRITON``      (kv_cache.py:7, :58-77)
* ``microinfer.layer.paged_attention.triton_paged_decode``      (paged_attention.py:6-10, :233)
* ``microinfer.layer.paged_attention.triton_paged_prefill``     (:109-139)
* ``microinfer.layer.paged_attention._gather_paged_kv``         (:76-101)
* ``microinfer.layer.paged_attention.paged_attention_meta``     (:188-293, imported by
  ``microinfer.layer.cached_attention`` at :5-9)
* ``microinfer.layer.cached_attention.flash_attn_varlen_func`` and
  ``microinfer.layer.paged_attention.flash_attn_varlen_func`` (cached_attention.py:9-13,
  :17-45; paged_attention.py:12-19, :142-185) become ``flash_attn_varlen_compat``, an adapter
  with FlashAttention's varlen signature over ``varlen_prefill`` / ``paged_prefill``, so
  the gathered paged prefill runs on the tcgen05 kernel.  ``flash_attn_with_kvcache`` is
  set to ``None`` (its decode path is this package's ``paged_attention_meta``).
* ``microinfer.layer.cached_attention._direct_prefill_flash`` (cached_attention.py:17-45)
  becomes ``direct_prefill_compat``: the reference's guard sends fp32 (and FA-less installs)
  to per-request SDPA (:93-101), so prefix-free prefill of CUDA tensors of every dtype goes
  to ``varlen_prefill`` instead; CPU tensors still get the reference's own CPU path.

``paged_attention_meta`` is rebound in both modules, so every decode, chunked
and prefix-hit prefill goes to this package's dispatch.
"""

from __future__ import annotations

import importlib
import sys

import torch

from microinfer_b200.layer import paged_attention as _pa
from microinfer_b200.worker import kv_store as _store


def _decode_compat(query, key_cache, value_cache, block_tables, context_lens, *, scale=None,
                   split_k=None):
    return _pa.paged_decode(query, key_cache, value_cache, block_tables, context_lens,
                            scale=scale, split_k=split_k)


def flash_attn_varlen_compat(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                             dropout_p=0.0, softmax_scale=None, causal=False,
                             window_size=(-1, -1), softcap=0.0, alibi_slopes=None,
                             deterministic=False, return_attn_probs=False, block_table=None):
    """``flash_attn.flash_attn_varlen_func`` as the reference calls it, on the sm_100a kernels.

    The reference calls it causal, without dropout, for prefix-free prefill
    (``_direct_prefill_flash``, cached_attention.py:17-45: contiguous K/V,
    ``cu_seqlens_q == cu_seqlens_k``) and for the gathered paged prefill
    (``_paged_prefill_gather``, paged_attention.py:142-185: ``cu_seqlens_k``
    cumulative over contexts, queries aligned to the end of their context);
    with ``block_table`` the K/V arguments are the paged caches.  Options the
    kernels do not implement raise ``ValueError`` instead of running something
    else.
    """
    if not causal:
        raise ValueError("flash_attn_varlen_compat implements causal attention only")
    if dropout_p != 0.0 or tuple(window_size) != (-1, -1) or softcap != 0.0 \
            or alibi_slopes is not None or return_attn_probs:
        raise ValueError("flash_attn_varlen_compat: dropout, windows, softcap, ALiBi and "
                         "returned probabilities are not supported")
    del max_seqlen_k, deterministic  # the kernels are deterministic and bound keys per row
    if block_table is not None:
        return _pa.paged_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, block_table,
                                 max_seqlen_q=int(max_seqlen_q), scale=softmax_scale)
    return _pa.varlen_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k,
                              max_seqlen_q=int(max_seqlen_q), scale=softmax_scale)


def direct_prefill_compat(q, k, v, metadata):
    """``_direct_prefill_flash(q, k, v, metadata)`` (cached_attention.py:17-45) on
    ``varlen_prefill``: causal attention of each request over this step's own K/V,
    for fp16, bf16 and fp32.  Returns ``None`` for CPU tensors, so the reference
    keeps its per-request SDPA there (its CPU path, :93-101)."""
    if not q.is_cuda:
        return None
    cu_q = metadata.cu_seqlens_q
    if cu_q is None:
        cu_q = torch.tensor(list(metadata.cu_q_cpu), dtype=torch.int32, device=q.device)
    cu_k = metadata.cu_seqlens_k if metadata.cu_seqlens_k is not None else cu_q
    max_q = metadata.max_seqlen_q
    if not max_q or max_q <= 0:
        max_q = max(list(metadata.q_lens_cpu), default=0)
    if max_q <= 0:
        return torch.empty_like(q) if q.shape[0] == 0 else None
    return _pa.varlen_prefill(q, k, v, cu_q, cu_k, max_seqlen_q=int(max_q))


def install(package: str = "microinfer") -> dict:
    """Rebind the reference's kernel globals; returns the replaced objects
    (``uninstall(replaced)`` puts them back)."""
    kv_cache = importlib.import_module(f"{package}.worker.kv_cache")
    paged = importlib.import_module(f"{package}.layer.paged_attention")
    cached = importlib.import_module(f"{package}.layer.cached_attention")
    replaced = {}

    def rebind(module, name, value):
        replaced[f"{module.__name__}.{name}"] = getattr(module, name, None)
        setattr(module, name, value)

    rebind(kv_cache, "store_kv", _store.store_kv)
    rebind(kv_cache, "HAS_TRITON", True)
    rebind(paged, "HAS_TRITON", True)
    rebind(paged, "triton_paged_decode", _decode_compat)
    rebind(paged, "triton_paged_prefill", _pa.paged_prefill)
    rebind(paged, "_gather_paged_kv", _pa.gather_paged_kv)
    rebind(paged, "flash_attn_varlen_func", flash_attn_varlen_compat)
    rebind(paged, "flash_attn_with_kvcache", None)
    rebind(paged, "paged_attention_meta", _pa.paged_attention_meta)
    rebind(cached, "paged_attention_meta", _pa.paged_attention_meta)
    rebind(cached, "flash_attn_varlen_func", flash_attn_varlen_compat)
    rebind(cached, "_direct_prefill_flash", direct_prefill_compat)
    return replaced


def uninstall(replaced: dict) -> None:
    """Put back the objects ``install`` replaced (its return value)."""
    for qualified, value in replaced.items():
        module_name, name = qualified.rsplit(".", 1)
        setattr(sys.modules[module_name], name, value)
