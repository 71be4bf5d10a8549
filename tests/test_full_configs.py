"""Parity at the full sizes of the BASELINE configs, and the launch branches
only those sizes reach.

Each case runs the same seeded workload ``bench.py`` times
(``tests/golden/configs.py``) through the package API and checks every output
row against a device fp32 restatement of the reference's
``_paged_attention_reference`` (microinfer/layer/paged_attention.py:22-67),
and a few whole requests against the numpy oracle on the host (requests are
independent, so a subset is an exact check of those rows).  Tolerance: 2e-2
abs / 1e-2 rel (bf16 with fp32 accumulation).
"""

import math

import numpy as np
import pytest
import torch

import microinfer_b200 as mi
from microinfer_b200 import _lib
from oracle import paged_oracle as po
from tests.golden import configs

pytestmark = pytest.mark.gpu

HQ, HKV, D, BS = 16, 8, 128, 16
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(autouse=True)
def _clean_status(cuda_device):
    _lib.read_device_status(cuda_device)
    yield
    assert _lib.read_device_status(cuda_device) == 0, "a kernel flagged a bad id or timeout"


def _bits(t):
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _pool(nb, hkv, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    kc = torch.empty(nb, BS, hkv, D, dtype=torch.bfloat16, device=device)
    vc = torch.empty_like(kc)
    kc.normal_(generator=g).mul_(0.5)
    vc.normal_(generator=g).mul_(0.5)
    return kc, vc, g


def _oracle_rows(out, q, kc, vc, b, rows, scale):
    """Whole requests `rows` against the numpy oracle (host copies of their pages only)."""
    cu = b["cu_q"].tolist()
    for r in rows:
        ctx = b["contexts"][r]
        nblk = (ctx + BS - 1) // BS
        blocks = b["table"][r, :nblk].long().to(kc.device)
        s, e = cu[r], cu[r + 1]
        exp = po.paged_attention(_bits(q[s:e]), _bits(kc[blocks]), _bits(vc[blocks]),
                                 np.arange(nblk, dtype=np.int32)[None, :], [ctx], [0, e - s],
                                 scale=scale, dtype="bf16")
        np.testing.assert_allclose(out[s:e].float().cpu().numpy(), po.to_f32(exp, "bf16"),
                                   atol=ATOL, rtol=RTOL, err_msg=f"request {r}")


def _prefill_case(b, hq, hkv, seed, device):
    kc, vc, g = _pool(b["nb"], hkv, seed, device)
    q = torch.randn(b["tokens"], hq, D, generator=g, device=device).to(torch.bfloat16)
    kn = torch.randn(b["tokens"], hkv, D, generator=g, device=device).to(torch.bfloat16)
    vn = torch.randn(b["tokens"], hkv, D, generator=g, device=device).to(torch.bfloat16)
    layer = mi.LayerKVCache(kc, vc)
    layer.write_slots(b["slots"].to(device), kn, vn)
    table, cu_q, cu_k = b["table"].to(device), b["cu_q"].to(device), b["cu_k"].to(device)
    out = mi.paged_prefill(q, kc, vc, cu_q, cu_k, table, max_seqlen_q=b["max_q"])
    torch.cuda.synchronize()
    return q, kc, vc, out


def _check_all_rows(out, q, kc, vc, b, scale):
    assert torch.isfinite(out.float()).all()
    ref = configs.torch_paged_attention(q, kc, vc, b["table"].to(q.device), b["contexts"],
                                        b["cu_q"], scale)
    torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)


def _pair_units(max_q, hq, hkv, seqs):
    tq = 128 // (hq // hkv)
    return ((max_q + 2 * tq - 1) // (2 * tq)) * hkv * seqs


def test_config3_mixed_batch_full_size(cuda_device):
    """24 decode rows + 8 x 512-token chunks in one mi_paged_prefill call
    (chunks on the tcgen05 kernel, one-token rows on the mma decode kernel behind it)."""
    b = configs.mixed_batch()
    q, kc, vc, out = _prefill_case(b, HQ, HKV, 11, cuda_device)
    scale = 1 / math.sqrt(D)
    _check_all_rows(out, q, kc, vc, b, scale)
    ctx = b["contexts"]
    dec = sorted(range(24), key=lambda r: ctx[r])
    _oracle_rows(out, q, kc, vc, b, [dec[0], dec[-1], 24, 31], scale)


def test_config4_shared_prefix_full_size_takes_the_single_tile_branch(cuda_device):
    """64 x 128-token suffixes on one shared 1024-token prefix.  512 tile-pair
    units on 148 SMs leave a last wave of 68 pairs, which the launch runs as 136
    single-tile CTAs (the branch every bench number of this config goes through)."""
    b = configs.shared_prefix_batch()
    sms = _lib.load().mi_device_sm_count(0)
    units = _pair_units(b["max_q"], HQ, HKV, len(b["q_lens"]))
    rem = units % sms
    assert units > sms and 0 < rem and 2 * rem <= sms, "shape no longer reaches the branch"
    q, kc, vc, out = _prefill_case(b, HQ, HKV, 12, cuda_device)
    scale = 1 / math.sqrt(D)
    _check_all_rows(out, q, kc, vc, b, scale)
    _oracle_rows(out, q, kc, vc, b, [0, 37, 63], scale)


@pytest.mark.parametrize("hq,q_len", [(16, 256), (32, 128), (16, 200)])
def test_last_wave_single_tiles_at_a_small_size(cuda_device, hq, q_len):
    """Just over one wave of tile-pair units with a last wave at most half full: the
    units past split_from run as two single-tile CTAs.  Every row against the oracle."""
    gen = torch.Generator().manual_seed(hq + q_len)
    n = 12
    prefixes = torch.randint(0, 200, (n,), generator=gen).tolist()
    contexts = [p + q_len for p in prefixes]
    nb = sum((c + BS - 1) // BS for c in contexts) + 4
    table = configs._tables(gen, contexts, nb)
    b = configs._finish([q_len] * n, contexts, table, nb)
    sms = _lib.load().mi_device_sm_count(0)
    units = _pair_units(q_len, hq, HKV, n)
    if not (units > sms and 2 * (units % sms) <= sms and units % sms):
        pytest.skip(f"{units} units on {sms} SMs do not reach the single-tile branch")
    q, kc, vc, out = _prefill_case(b, hq, HKV, 13, cuda_device)
    _oracle_rows(out, q, kc, vc, b, list(range(n)), 1 / math.sqrt(D))


def test_config5b_32k_split_decode_full_size(cuda_device):
    """configs[4] run (b): one Qwen3-8B-shaped sequence at 32768 context, store fused
    into the split-K decode with the library's default split count."""
    hq, hkv, ctx = 32, 8, 32768
    nb = ctx // BS
    kc, vc, g = _pool(nb, hkv, 14, cuda_device)
    table = torch.randperm(nb, generator=g, device=cuda_device).to(torch.int32).view(1, nb)
    ctx_d = torch.tensor([ctx], dtype=torch.int32, device=cuda_device)
    slot = (table[0, -1].long() * BS + BS - 1).to(torch.int32).view(1)
    q = torch.randn(1, hq, D, generator=g, device=cuda_device).to(torch.bfloat16)
    kn = torch.randn(1, hkv, D, generator=g, device=cuda_device).to(torch.bfloat16)
    vn = torch.randn(1, hkv, D, generator=g, device=cuda_device).to(torch.bfloat16)
    _, split, _ = mi.decode_plan(1, hq, hkv, D, torch.bfloat16, BS, 0, cuda_device, nb)
    assert split > 1
    out = mi.paged_decode_store(q, kc, vc, table, ctx_d, kn, vn, slot)
    torch.cuda.synchronize()
    assert torch.equal(kc.view(-1, hkv, D)[slot.long()], kn)
    exp = po.paged_decode(_bits(q), _bits(kc), _bits(vc), table.cpu().numpy(), [ctx],
                          scale=1 / math.sqrt(D), dtype="bf16")
    np.testing.assert_allclose(out.float().cpu().numpy(), po.to_f32(exp, "bf16"), atol=ATOL,
                               rtol=RTOL)


def test_config5a_256_sequences_full_size(cuda_device):
    """configs[4] run (a), one GPU's layer: 256 Qwen3-8B-shaped sequences with contexts
    U[4096, 32768] (a ~19 GB pool), fused store + decode with the default plan."""
    hq, hkv = 32, 8
    b = configs.long_batch(256)
    kc, vc, g = _pool(b["nb"], hkv, 15, cuda_device)
    n = len(b["contexts"])
    q = torch.randn(n, hq, D, generator=g, device=cuda_device).to(torch.bfloat16)
    kn = torch.randn(n, hkv, D, generator=g, device=cuda_device).to(torch.bfloat16)
    vn = torch.randn(n, hkv, D, generator=g, device=cuda_device).to(torch.bfloat16)
    table = b["table"].to(cuda_device)
    ctx_d = torch.tensor(b["contexts"], dtype=torch.int32, device=cuda_device)
    out = mi.paged_decode_store(q, kc, vc, table, ctx_d, kn, vn, b["slots"].to(cuda_device))
    torch.cuda.synchronize()
    scale = 1 / math.sqrt(D)
    _check_all_rows(out, q, kc, vc, b, scale)
    ctx = b["contexts"]
    _oracle_rows(out, q, kc, vc, b, [min(range(n), key=ctx.__getitem__),
                                     max(range(n), key=ctx.__getitem__)], scale)


def test_direct_prefill_config3_sized(cuda_device):
    """Prefix-free prefill of a config-3-sized batch (8 x 512 + 24 x U[1, 64] tokens) on
    contiguous K/V through varlen_prefill, against the dense oracle on the host."""
    gen = torch.Generator().manual_seed(16)
    lens = [512] * 8 + torch.randint(1, 65, (24,), generator=gen).tolist()
    total = sum(lens)
    g = torch.Generator(device=cuda_device).manual_seed(16)
    q = torch.randn(total, HQ, D, generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(total, HKV, D, generator=g, device=cuda_device).to(torch.bfloat16)
    v = torch.randn(total, HKV, D, generator=g, device=cuda_device).to(torch.bfloat16)
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0)
    out = mi.varlen_prefill(q, k, v, cu.to(cuda_device), cu.to(cuda_device), max_seqlen_q=512)
    torch.cuda.synchronize()
    exp = po.dense_varlen_attention(_bits(q), _bits(k), _bits(v), cu.numpy(),
                                    scale=1 / math.sqrt(D), dtype="bf16")
    np.testing.assert_allclose(out.float().cpu().numpy(), po.to_f32(exp, "bf16"), atol=ATOL,
                               rtol=RTOL)
