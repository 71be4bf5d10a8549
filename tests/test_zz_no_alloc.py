"""mi_paged_decode_noalloc: decode without any device allocation by the caller.

The entry point is for callers that cannot allocate device memory on the
call path (a serving loop whose HBM was reserved up front, or an FFI host
holding only the buffers it was given).  It keeps its split-K states in a
2 MiB array built into the library instead of a workspace the caller passes.

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.  It must pass on its own in a fresh
process as well as after the rest of the suite.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from microinfer_b200 import _lib
from oracle import paged_oracle as po

pytestmark = pytest.mark.gpu

DTYPES = {torch.bfloat16: (2, "bf16"), torch.float16: (1, "f16")}


def _decode_batch(seed, n, hq, hkv, d, bs, nb, lo, hi, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    ctx = torch.randint(lo, hi + 1, (n,), generator=g, dtype=torch.int32)
    need = [(int(c) + bs - 1) // bs for c in ctx]
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    table = torch.full((n, max(need)), -1, dtype=torch.int32)
    at = 0
    for r, k in enumerate(need):
        table[r, :k] = perm[at:at + k]
        at += k
    kc = (torch.randn(nb, bs, hkv, d, generator=g) * 0.5).to(dtype)
    vc = (torch.randn(nb, bs, hkv, d, generator=g) * 0.5).to(dtype)
    q = torch.randn(n, hq, d, generator=g).to(dtype)
    dev = torch.device("cuda", 0)
    return (q.to(dev), kc.to(dev), vc.to(dev), table.to(dev), ctx.to(dev))


def _with_workspace(q, kc, vc, table, ctx, splits, status, stream):
    """The existing entry point, with a workspace allocated by the caller."""
    lib = _lib.load()
    n, hq, d = q.shape
    out = torch.empty_like(q)
    planned, ws_size = ctypes.c_int32(0), ctypes.c_size_t(0)
    assert lib.mi_paged_decode_plan(n, hq, kc.shape[2], d, DTYPES[q.dtype][0], kc.shape[1],
                                    table.shape[1], splits, q.device.index or 0,
                                    ctypes.byref(planned), ctypes.byref(ws_size)) > 0
    ws_bytes = ws_size.value
    # zero-filled once: the kernels leave the split-K arrival counters at zero
    ws = torch.zeros(max(ws_bytes // 4, 1), dtype=torch.float32, device=q.device)
    _lib.check(lib.mi_paged_decode(
        out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], kc.shape[1],
        hq, kc.shape[2], d, DTYPES[q.dtype][0], table.data_ptr(), table.stride(0), ctx.data_ptr(),
        n, 1 / math.sqrt(d), splits, ws.data_ptr(), ws_bytes, status.data_ptr(), stream))
    return out


def _no_alloc(q, kc, vc, table, ctx, splits, status, stream):
    """The allocation-free entry point; `out` is the only buffer passed."""
    lib = _lib.load()
    n, hq, d = q.shape
    out = torch.empty_like(q)
    _lib.check(lib.mi_paged_decode_noalloc(
        out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], kc.shape[1],
        hq, kc.shape[2], d, DTYPES[q.dtype][0], table.data_ptr(), table.stride(0), ctx.data_ptr(),
        n, 1 / math.sqrt(d), splits, status.data_ptr(), stream))
    return out


def _bits(t, dt):
    t = t.detach().contiguous().cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if dt == "bf16" else t.numpy()


def _oracle(q, kc, vc, table, ctx):
    """The CPU oracle's decode (the reference's _paged_attention_reference restated)."""
    dt = DTYPES[q.dtype][1]
    exp = po.paged_decode(_bits(q, dt), _bits(kc, dt), _bits(vc, dt), table.cpu().numpy(),
                          ctx.cpu().numpy(), scale=1 / math.sqrt(q.shape[-1]), dtype=dt)
    return torch.from_numpy(po.to_f32(exp, dt))


@pytest.mark.parametrize("shape", [
    # Qwen3-0.6B decode step, 4 splits per (seq, kv head)
    dict(seed=0, n=8, hq=16, hkv=8, d=128, bs=16, nb=1024, lo=128, hi=512, splits=4),
    # one long Qwen3-8B-shaped sequence, 37 splits (the batch-1 split-K case)
    dict(seed=1, n=1, hq=32, hkv=8, d=128, bs=16, nb=640, lo=9000, hi=10000, splits=37),
    # the library's default split count (num_splits = 0)
    dict(seed=3, n=8, hq=16, hkv=8, d=128, bs=16, nb=1024, lo=128, hi=512, splits=0),
    # default splits near the scratch limit: 148 seqs x 8 heads x D 256 would want two
    # splits (2.5 MB of states); the default is capped to what the 2 MiB scratch holds
    dict(seed=4, n=148, hq=8, hkv=1, d=256, bs=16, nb=6000, lo=200, hi=600, splits=0),
    # one split: no scratch at all
    dict(seed=5, n=8, hq=16, hkv=8, d=128, bs=16, nb=1024, lo=128, hi=512, splits=1),
    # fp16, head_dim 64, GQA group 4
    dict(seed=6, n=6, hq=16, hkv=4, d=64, bs=32, nb=256, lo=40, hi=900, splits=3,
         dtype=torch.float16),
])
def test_no_alloc_decode_matches_workspace_decode_twice(shape):
    if not torch.cuda.is_available():
        pytest.skip("CUDA device is not available")
    splits = shape.pop("splits")
    q, kc, vc, table, ctx = _decode_batch(**shape)
    dev = q.device
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    expected = _with_workspace(q, kc, vc, table, ctx, splits, status, stream)
    first = _no_alloc(q, kc, vc, table, ctx, splits, status, stream)
    # The scratch keeps the first call's states; a second call must not depend on them.
    q2 = torch.flip(q, dims=[0]).contiguous()
    expected2 = _with_workspace(q2, kc, vc, table, ctx, splits, status, stream)
    second = _no_alloc(q2, kc, vc, table, ctx, splits, status, stream)
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 0
    torch.testing.assert_close(first.float(), expected.float(), atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(second.float(), expected2.float(), atol=2e-2, rtol=1e-2)
    # and both against the CPU oracle
    torch.testing.assert_close(first.float().cpu(), _oracle(q, kc, vc, table, ctx), atol=2e-2,
                               rtol=1e-2)
    torch.testing.assert_close(second.float().cpu(), _oracle(q2, kc, vc, table, ctx), atol=2e-2,
                               rtol=1e-2)


def test_no_alloc_rejects_states_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device is not available")
    lib = _lib.load()
    q, kc, vc, table, ctx = _decode_batch(2, 4, 16, 8, 128, 16, 64, 16, 200)
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=q.device)
    # 4 seqs * 16 heads * 300 splits * 130 floats * 4 B = 9.98 MB > 2 MiB
    rc = lib.mi_paged_decode_noalloc(
        out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], 16, 16, 8, 128,
        2, table.data_ptr(), table.stride(0), ctx.data_ptr(), 4, 0.088, 300, status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc == -1
    assert "2 MiB" in lib.mi_last_error().decode()
