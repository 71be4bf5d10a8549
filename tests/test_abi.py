"""The C-ABI library: loads, exports every declared symbol, validates on the host.

No kernel runs here: every call below is rejected (or answered) before any
CUDA work, so these run on a machine without a GPU.
"""

import ctypes
import re
from pathlib import Path

import pytest

from microinfer_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "microinfer_b200.h"


def _declared():
    text = HEADER.read_text()
    decls = {}
    for m in re.finditer(r"MI_API\s+[\w\s\*]+?\b(mi_\w+)\s*\(([^;]*?)\);", text, re.S):
        args = m.group(2).strip()
        n = 0 if args in ("void", "") else args.count(",") + 1
        decls[m.group(1)] = n
    return decls


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    decls = _declared()
    assert len(decls) >= 12
    for name in decls:
        assert hasattr(lib, name), name


def test_ctypes_signatures_match_header_arity():
    decls = _declared()
    assert set(decls) == set(_lib.SIGNATURES)
    for name, nargs in decls.items():
        assert len(_lib.SIGNATURES[name][1]) == nargs, name


def test_abi_version():
    assert _lib.load().mi_abi_version() == 1


def test_workspace_and_split_policy():
    lib = _lib.load()
    assert lib.mi_paged_decode_workspace_bytes(8, 16, 128, 1) == 0
    # a fixed 64 KiB region of arrival counters, then the split states
    assert lib.mi_paged_decode_workspace_bytes(8, 16, 128, 5) == 65536 + 8 * 16 * 5 * 130 * 4
    assert lib.mi_paged_decode_workspace_bytes(1, 4, 64, 2) == 65536 + 1 * 4 * 2 * 66 * 4
    # 148 SMs assumed without a device.  Small batches stay within half the
    # SMs (74 CTAs) so the next layer's CTAs fit beside them: 74 // (8*8) = 1
    assert lib.mi_paged_decode_default_splits(8, 8, 0, 0) == 1
    assert lib.mi_paged_decode_default_splits(1, 8, 0, 0) == 9
    # ... and a context hint gives each split >= 384 keys
    assert lib.mi_paged_decode_default_splits(1, 8, 256, 0) == 1
    assert lib.mi_paged_decode_default_splits(1, 8, 2000, 0) == 6
    # larger batches: one wave of two CTAs per SM, >= 2 chunks of 8 keys per warp
    assert lib.mi_paged_decode_default_splits(16, 8, 0, 0) == 2
    assert lib.mi_paged_decode_default_splits(256, 8, 0, 0) == 1


def _decode_args(**over):
    # 16-byte aligned fake addresses: the shape goes to a fast kernel, and every
    # rejection below happens on the host before any pointer is touched.
    args = dict(out=256, query=256, key_cache=256, value_cache=256, num_blocks=4, block_size=16,
                num_q_heads=16, num_kv_heads=8, head_dim=128, dtype=2, block_tables=1,
                block_table_stride=4, context_lens=1, num_seqs=2, scale=0.1, num_splits=1,
                workspace=None, workspace_bytes=0, dev_status=None, stream=None)
    args.update(over)
    return list(args.values())


@pytest.mark.parametrize("over,fragment", [
    (dict(num_q_heads=12, num_kv_heads=8), "divisible"),
    (dict(dtype=7), "dtype"),
    (dict(head_dim=512), "head_dim"),
    (dict(num_splits=-1), "num_splits"),
    (dict(num_splits=16, workspace=None, workspace_bytes=0), "workspace"),
    (dict(out=None), "null"),
])
def test_decode_rejects_invalid_arguments_before_launch(over, fragment):
    lib = _lib.load()
    status = lib.mi_paged_decode(*_decode_args(**over))
    assert status < 0
    assert fragment in lib.mi_last_error().decode()
    with pytest.raises(ValueError):
        _lib.check(status)


def test_workspace_needed_for_every_split_count_above_one():
    lib = _lib.load()
    assert [lib.mi_paged_decode_uses_workspace(s) for s in (1, 2, 8, 9, 37)] == [0, 1, 1, 1, 1]


def test_decode_with_no_sequences_is_a_no_op():
    assert _lib.load().mi_paged_decode(*_decode_args(num_seqs=0)) == 0


def test_store_rejects_bad_index_dtype():
    lib = _lib.load()
    st = lib.mi_store_kv(1, 1, 4, 16, 8, 128, 2, 1, 1, 5, 1, 1, 1024, 1024, 3, None, None)
    assert st == -1 and "index" in lib.mi_last_error().decode()


def test_copy_blocks_rejects_short_layer_stride():
    lib = _lib.load()
    st = lib.mi_copy_blocks(1, 1, 2, 100, 4, 64, 1, 1, None, None)
    assert st == -1 and "layer_stride" in lib.mi_last_error().decode()


def test_wait_selftest_rejects_unbounded_timeout():
    lib = _lib.load()
    assert lib.mi_wait_flag_selftest(1, 0, 1, None) == -1
    assert lib.mi_wait_flag_selftest(1, 11_000_000_000, 1, None) == -1


def test_host_pointer_is_rejected_not_dereferenced():
    """A host address passed as device memory is refused by the driver lookup."""
    lib = _lib.load()
    buf = (ctypes.c_char * 4096)()
    addr = ctypes.addressof(buf)
    st = lib.mi_copy_blocks(addr, addr, 1, 1024, 4, 256, addr, 1, None, None)
    assert st < 0
