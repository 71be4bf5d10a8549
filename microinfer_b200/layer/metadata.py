"""Per-step attention metadata: the input contract of the paged hot path.

The public fields and derived views are those the reference's attention
backend reads (microinfer/layer/metadata.py:16-116), so a metadata object
built by the reference runner and one built here are interchangeable; the
kernels in this package only read device tensors.  Host views (the cumulative
query offsets, per-sequence contexts and query lengths as Python tuples) are
derived on first use and then reused by every layer of the step, so at most
one device->host copy happens per step, and none on the graph-captured decode
path.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


def _lengths(cumulative: tuple[int, ...]) -> tuple[int, ...]:
    return tuple(cumulative[i + 1] - cumulative[i] for i in range(len(cumulative) - 1))


@dataclass
class AttentionMetadata:
    is_prefill: bool
    cu_seqlens_q: torch.Tensor | None = None  # int32 [R+1], query offsets
    cu_seqlens_k: torch.Tensor | None = None  # int32 [R+1], cumulative contexts
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None  # int32 [T], block * bs + offset
    context_lens: torch.Tensor | None = None  # int32 [R], decode only
    block_tables: torch.Tensor | None = None  # int32 [R, W], -1 padded
    direct_prefill: bool = False
    validate_cache_write: bool = True
    _host: dict = field(default_factory=dict, repr=False, compare=False)

    @classmethod
    def build(cls, *, is_prefill: bool, block_tables=None, **fields) -> "AttentionMetadata":
        """Prefill without a block table is "direct": attend to this step's K/V only."""
        return cls(
            is_prefill=is_prefill,
            block_tables=block_tables,
            direct_prefill=bool(is_prefill and block_tables is None),
            **fields,
        )

    @property
    def is_decode(self) -> bool:
        return not self.is_prefill

    # -- host views, computed once per step -----------------------------------
    def _memo(self, key, make):
        if key not in self._host:
            self._host[key] = make()
        return self._host[key]

    @property
    def cu_q_cpu(self) -> tuple[int, ...]:
        def make():
            if self.cu_seqlens_q is not None:
                return tuple(int(x) for x in self.cu_seqlens_q.tolist())
            if self.context_lens is not None:  # decode: one query per sequence
                return tuple(range(self.context_lens.numel() + 1))
            return (0,)

        return self._memo("cu_q", make)

    @property
    def context_lens_cpu(self) -> tuple[int, ...]:
        def make():
            if self.context_lens is not None:
                return tuple(int(x) for x in self.context_lens.tolist())
            if self.cu_seqlens_k is not None:
                return _lengths(tuple(int(x) for x in self.cu_seqlens_k.tolist()))
            return ()

        return self._memo("contexts", make)

    @property
    def q_lens_cpu(self) -> tuple[int, ...]:
        return self._memo("q_lens", lambda: _lengths(self.cu_q_cpu))

    # -- slot split (for callers of the (blocks, offsets) store signature) ----
    @property
    def slot_mapping_long(self) -> torch.Tensor:
        if self.slot_mapping is None:
            raise ValueError("metadata has no slot_mapping")
        return self._memo("slots_i64", lambda: self.slot_mapping.long())

    def slot_indices(self, block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
        if block_size <= 0:
            raise ValueError("block_size must be positive")

        def make():
            slots = self.slot_mapping_long
            blocks = torch.div(slots, block_size, rounding_mode="floor")
            return blocks, slots - blocks * block_size

        return self._memo(("split", block_size), make)
