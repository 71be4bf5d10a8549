"""Drop the sm_100a kernels into a live ``microinfer`` import.

The reference looks its kernels up as module globals, so rebinding them is
enough for ``microinfer/layer`` and ``runner.py`` to run unchanged:

* ``microinfer.worker.kv_cache.store_kv`` / ``HAS_TRITON``      (kv_cache.py:7, :58-77)
* ``microinfer.layer.paged_attention.triton_paged_decode``      (paged_attention.py:6-10, :233)
* ``microinfer.layer.paged_attention.triton_paged_prefill``     (:109-139)
* ``microinfer.layer.paged_attention._gather_paged_kv``         (:76-101)
* ``microinfer.layer.paged_attention.paged_attention_meta``     (:188-293, imported by
  ``microinfer.layer.cached_attention`` at :5-9)
* FlashAttention symbols are set to ``None`` so no FA path is taken.

``paged_attention_meta`` is rebound in both modules, so every decode, chunked
and prefix-hit prefill goes to this package's dispatch.
"""

from __future__ import annotations

import importlib
import sys

from microinfer_b200.layer import paged_attention as _pa
from microinfer_b200.worker import kv_store as _store


def _decode_compat(query, key_cache, value_cache, block_tables, context_lens, *, scale=None,
                   split_k=None):
    return _pa.paged_decode(query, key_cache, value_cache, block_tables, context_lens,
                            scale=scale, split_k=split_k)


def install(package: str = "microinfer") -> dict:
    """Rebind the reference's kernel globals; returns the replaced objects."""
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
    rebind(paged, "flash_attn_varlen_func", None)
    rebind(paged, "flash_attn_with_kvcache", None)
    rebind(paged, "paged_attention_meta", _pa.paged_attention_meta)
    rebind(cached, "paged_attention_meta", _pa.paged_attention_meta)
    rebind(cached, "flash_attn_varlen_func", None)
    sys.modules.setdefault("microinfer_b200.installed_into", kv_cache)
    return replaced
