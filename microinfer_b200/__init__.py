"""B200-native (sm_100a) paged KV-cache hot path for the MicroInfer engine.

A C-ABI shared library (``libmicroinfer_b200.so``, see include/microinfer_b200.h)
holds the CUDA kernels; this package is the thin host layer that mirrors the
reference's attention-backend interface:

* ``worker.kv_store.store_kv`` / ``store_kv_slots``  - store_kvcache
* ``layer.paged_attention.paged_decode``             - split-K paged decode
* ``layer.paged_attention.paged_prefill``            - paged chunked prefill
* ``layer.paged_attention.varlen_prefill``           - dense (no-prefix) prefill
* ``layer.paged_attention.gather_paged_kv``          - block-table gather
* ``worker.kv_cache.copy_blocks``                    - copy-on-write of pages
* ``worker.block_manager.CowBlockManager``           - refcounted pages, shared partial
  blocks and the (src, dst) copies that ``copy_blocks`` issues
* ``layer.paged_attention.paged_attention_meta``     - backend dispatch
* ``layer.prologue.qk_norm_rope_store``             - q/k RMSNorm + RoPE + k/v store
* ``worker.runner_metadata.DeviceRunnerMetadata``  - per-step metadata from a device page table

``install()`` rebinds a live ``microinfer`` import onto these entry points.
"""

from microinfer_b200._lib import check_device_status, load, read_device_status
from microinfer_b200.install import install, uninstall
from microinfer_b200.layer.metadata import AttentionMetadata
from microinfer_b200.layer.paged_attention import (
    decode_plan,
    gather_paged_kv,
    paged_attention_meta,
    paged_decode,
    paged_decode_store,
    paged_prefill,
    select_split_k,
    varlen_prefill,
)
from microinfer_b200.layer.prologue import qk_norm_rope_store
from microinfer_b200.worker.runner_metadata import DeviceRunnerMetadata
from microinfer_b200.worker.block_manager import CowBlockManager, apply_copies
from microinfer_b200.worker.kv_cache import KVCache, LayerKVCache, copy_blocks
from microinfer_b200.worker.kv_store import store_kv, store_kv_slots
from microinfer_b200 import torch_ops  # noqa: E402,F401  (registers torch.ops.microinfer_b200.*)

__all__ = [
    "AttentionMetadata",
    "CowBlockManager",
    "KVCache",
    "LayerKVCache",
    "apply_copies",
    "check_device_status",
    "copy_blocks",
    "decode_plan",
    "gather_paged_kv",
    "install",
    "uninstall",
    "load",
    "paged_attention_meta",
    "paged_decode",
    "paged_decode_store",
    "paged_prefill",
    "qk_norm_rope_store",
    "DeviceRunnerMetadata",
    "read_device_status",
    "select_split_k",
    "store_kv",
    "store_kv_slots",
    "varlen_prefill",
]
