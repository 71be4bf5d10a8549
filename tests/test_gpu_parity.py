"""sm_100a kernels vs the reference (golden fixtures) and the CPU oracle.

Every call goes through the package API, which calls the C ABI of
libmicroinfer_b200.so.  Tolerances (from the spec): bit-exact for store,
gather and copy-on-write; attention within 2e-2 abs / 1e-2 rel for fp16/bf16
(fp32 accumulation) and 1e-5 for fp32.
"""

import math
import os

import numpy as np
import pytest
import torch

import microinfer_b200 as mi
from microinfer_b200 import _lib
from oracle import paged_oracle as po
from tests.conftest import load_golden
from tests.golden import cases

pytestmark = pytest.mark.gpu

TORCH = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
TOL = {"f32": (1e-5, 1e-5), "f16": (2e-2, 1e-2), "bf16": (2e-2, 1e-2)}


def dev(a, dtype=None, device="cuda"):
    a = np.ascontiguousarray(a)
    if dtype == "bf16":
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(a).to(device)


def host(t, dtype):
    t = t.detach().contiguous().cpu()
    if dtype == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def assert_close(actual, expected_bits, dtype):
    atol, rtol = TOL[dtype]
    np.testing.assert_allclose(po.to_f32(host(actual, dtype), dtype),
                               po.to_f32(expected_bits, dtype), atol=atol, rtol=rtol)


def _store(case, fast=False):
    dt = case["dtype"]
    kc, vc = dev(case["key_cache"], dt), dev(case["value_cache"], dt)
    slots = dev(case["slots"])
    k_new, v_new = dev(case["k_new"], dt), dev(case["v_new"], dt)
    layer = mi.LayerKVCache(kc, vc)
    if fast:
        bs = case["block_size"]
        sl = slots.long()
        layer.write_fast(sl // bs, sl % bs, k_new, v_new)
    else:
        layer.write_checked(slots, k_new, v_new)
    return layer


@pytest.fixture(autouse=True)
def _clean_status(cuda_device):
    _lib.read_device_status(cuda_device)
    yield
    assert _lib.read_device_status(cuda_device) == 0, "a kernel flagged a bad id or timeout"


PAGED = [c for c in cases.CASES if cases.kind(c) in ("decode", "prefill")]


@pytest.mark.parametrize("name", PAGED)
@pytest.mark.parametrize("fast", [False, True])
def test_store_is_bit_exact(name, fast):
    case = cases.build(name)
    gold = load_golden(name)
    layer = _store(case, fast=fast)
    slots = case["slots"].astype(np.int64)
    bs = case["block_size"]
    dt = case["dtype"]
    assert cases.digest(host(layer.keys, dt)[slots // bs, slots % bs]) == str(gold["stored_k_digest"])
    assert cases.digest(host(layer.values, dt)[slots // bs, slots % bs]) == str(gold["stored_v_digest"])
    # nothing else in the pool changed
    untouched = np.ones(case["key_cache"].shape[:2], bool)
    untouched[slots // bs, slots % bs] = False
    np.testing.assert_array_equal(host(layer.keys, dt)[untouched], case["key_cache"][untouched])


@pytest.mark.parametrize("name", PAGED)
def test_attention_matches_reference_and_oracle(name):
    case = cases.build(name)
    gold = load_golden(name)
    dt = case["dtype"]
    layer = _store(case)
    q = dev(case["query"], dt)
    table = dev(case["block_tables"])
    if case["kind"] == "decode":
        out = mi.paged_decode(q, layer.keys, layer.values, table, dev(case["contexts"]),
                              scale=case["scale"])
        cu_q = np.arange(len(case["contexts"]) + 1)
    else:
        out = mi.paged_prefill(q, layer.keys, layer.values, dev(case["cu_seqlens_q"]),
                               dev(case["cu_seqlens_k"]), table,
                               max_seqlen_q=int(case["q_lens"].max()), scale=case["scale"])
        cu_q = case["cu_seqlens_q"]
    assert out.dtype == TORCH[dt] and out.shape == q.shape
    assert torch.isfinite(out.float()).all()
    assert_close(out, gold["out"], dt)
    kc, vc = host(layer.keys, dt), host(layer.values, dt)
    expected = po.paged_attention(case["query"], kc, vc, case["block_tables"], case["contexts"],
                                  cu_q, scale=case["scale"], dtype=dt)
    assert_close(out, expected, dt)


MIXED = ["mixed_bf16"] + [c for c in cases.CASES if c.startswith("tc_prefill_g")]


@pytest.mark.parametrize("name", MIXED)
def test_mixed_batch_decode_rows_through_the_c_abi(name):
    """Mixed batches: the one-token rows run on the decode kernel launched behind
    the tensor-core prefill (its programmatic dependent); called twice in a row
    through mi_paged_prefill, every row matches the reference."""
    case = cases.build(name)
    gold = load_golden(name)
    dt = case["dtype"]
    layer = _store(case)
    q = dev(case["query"], dt)
    table = dev(case["block_tables"])
    cu_q, cu_k = dev(case["cu_seqlens_q"]), dev(case["cu_seqlens_k"])
    n = len(case["contexts"])
    hq, d = q.shape[1], q.shape[2]
    nb, bs, hkv, _ = layer.keys.shape
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _lib.call("mi_paged_prefill", out.data_ptr(), q.data_ptr(), layer.keys.data_ptr(),
                  layer.values.data_ptr(), nb, bs, hq, hkv, d, _lib.dtype_code(q.dtype),
                  cu_q.data_ptr(), cu_k.data_ptr(), table.data_ptr(), table.stride(0), n,
                  q.shape[0], int(case["q_lens"].max()), float(case["scale"]),
                  _lib.status_buffer(q.device).data_ptr(), _lib.stream_of(q.device))
        torch.cuda.synchronize()
        assert_close(out, gold["out"], dt)


@pytest.mark.parametrize("name", [c for c in PAGED if cases.kind(c) == "decode"])
@pytest.mark.parametrize("split_k", [1, 2, 3, 7, 37])
def test_decode_split_k_matches_reference(name, split_k):
    case = cases.build(name)
    gold = load_golden(name)
    dt = case["dtype"]
    layer = _store(case)
    out = mi.paged_decode(dev(case["query"], dt), layer.keys, layer.values,
                          dev(case["block_tables"]), dev(case["contexts"]), scale=case["scale"],
                          split_k=split_k)
    assert_close(out, gold["out"], dt)


@pytest.mark.parametrize("name", [c for c in PAGED if cases.kind(c) == "decode"])
@pytest.mark.parametrize("split_k,early_kv", [(1, False), (2, False), (2, True), (4, False),
                                              (16, False), (4, True), (37, True)])
def test_fused_store_decode_matches_reference(name, split_k, early_kv):
    """store_kvcache fused into the decode launch: same cache bytes, same output."""
    case = cases.build(name)
    gold = load_golden(name)
    dt = case["dtype"]
    kc, vc = dev(case["key_cache"], dt), dev(case["value_cache"], dt)
    out = mi.paged_decode_store(dev(case["query"], dt), kc, vc, dev(case["block_tables"]),
                                dev(case["contexts"]), dev(case["k_new"], dt),
                                dev(case["v_new"], dt), dev(case["slots"]), scale=case["scale"],
                                split_k=split_k, early_kv=early_kv)
    slots = case["slots"].astype(np.int64)
    bs = case["block_size"]
    assert cases.digest(host(kc, dt)[slots // bs, slots % bs]) == str(gold["stored_k_digest"])
    assert cases.digest(host(vc, dt)[slots // bs, slots % bs]) == str(gold["stored_v_digest"])
    assert_close(out, gold["out"], dt)


def test_fused_store_skips_padding_slots():
    case = cases.build("cfg2_layer_bf16")
    dt = "bf16"
    kc, vc = dev(case["key_cache"], dt), dev(case["value_cache"], dt)
    before = host(kc, dt)
    slots = dev(case["slots"])
    slots[0] = -1  # padding row: nothing written for sequence 0
    mi.paged_decode_store(dev(case["query"], dt), kc, vc, dev(case["block_tables"]),
                          dev(case["contexts"]), dev(case["k_new"], dt), dev(case["v_new"], dt),
                          slots, split_k=4)
    s0 = int(case["slots"][0])
    np.testing.assert_array_equal(host(kc, dt)[s0 // 16, s0 % 16], before[s0 // 16, s0 % 16])
    s1 = int(case["slots"][1])
    np.testing.assert_array_equal(host(kc, dt)[s1 // 16, s1 % 16], case["k_new"][1])


@pytest.mark.parametrize("width", [4, 160])  # table bound 64 / 2560 keys
@pytest.mark.parametrize("split_k,early_kv", [(1, False), (3, True)])
def test_fused_store_with_only_the_new_token(width, split_k, early_kv):
    """Context 1: the token being stored is the whole context, so out = v_new."""
    n, hq, hkv, d, bs = 3, 16, 8, 128, 16
    kernel, _, _ = mi.decode_plan(n, hq, hkv, d, torch.bfloat16, bs, split_k, "cuda", width)
    if "MICROINFER_B200_DECODE" not in os.environ:  # not pinned to one kernel
        assert kernel in ("mma", "mma_pair")
    g = torch.Generator(device="cuda").manual_seed(3)
    kc = torch.randn(8, bs, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(n, hq, d, generator=g, device="cuda").to(torch.bfloat16)
    kn = torch.randn(n, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    vn = torch.randn(n, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    table = torch.full((n, width), -1, dtype=torch.int32, device="cuda")
    table[:, 0] = torch.tensor([5, 2, 7], dtype=torch.int32)
    ctx = torch.ones(n, dtype=torch.int32, device="cuda")
    slots = (table[:, 0] * bs).to(torch.int32)
    out = mi.paged_decode_store(q, kc, vc, table, ctx, kn, vn, slots, split_k=split_k,
                                early_kv=early_kv)
    torch.cuda.synchronize()
    expected = vn.repeat_interleave(hq // hkv, dim=1)
    torch.testing.assert_close(out, expected, atol=0, rtol=0)
    torch.testing.assert_close(kc[table[:, 0].long(), 0], kn, atol=0, rtol=0)
    torch.testing.assert_close(vc[table[:, 0].long(), 0], vn, atol=0, rtol=0)


def _Seq(num_tokens, block_size=16):
    from tests.golden.block_trace import TraceSequence

    s = TraceSequence(list(range(1, num_tokens + 1)))
    s.block_size = block_size
    return s


def test_forked_sequences_copy_on_write_then_decode_in_isolation():
    """Two sequences share a partial page (CowBlockManager.fork); each appends its
    own token.  apply_copies issues the page copy on the device (every layer),
    then the fused store+decode writes and attends: each sequence's output is
    attention over its own 21 tokens only, in every layer."""
    bs, hkv, hq, d, nb, layers = 16, 8, 16, 128, 16, 2
    gen = torch.Generator(device="cuda").manual_seed(21)
    cache = mi.KVCache(layers, nb, bs, hkv, d, dtype=torch.bfloat16, device="cuda")
    m = mi.CowBlockManager(nb, bs)
    a = _Seq(20)
    m.allocate(a, 0)
    hist = [(torch.randn(20, hkv, d, generator=gen, device="cuda").to(torch.bfloat16),
             torch.randn(20, hkv, d, generator=gen, device="cuda").to(torch.bfloat16))
            for _ in range(layers)]
    pos = torch.arange(20)
    slots = (torch.tensor(a.block_table)[pos // bs] * bs + pos % bs).to(torch.int32).cuda()
    for li in range(layers):
        cache.layer(li).write_slots(slots, *hist[li])
    b = _Seq(20)
    m.fork(a, b)
    new_slots = torch.tensor([m.prepare_append(a), m.prepare_append(b)], dtype=torch.int32)
    assert mi.apply_copies(m, cache) == 1  # b's copy of the shared partial page
    a.num_tokens = b.num_tokens = 21
    width = max(len(a.block_table), len(b.block_table))
    table = torch.full((2, width), -1, dtype=torch.int32)
    table[0, :len(a.block_table)] = torch.tensor(a.block_table)
    table[1, :len(b.block_table)] = torch.tensor(b.block_table)
    ctx = torch.tensor([21, 21], dtype=torch.int32, device="cuda")
    for li in range(layers):
        q = torch.randn(2, hq, d, generator=gen, device="cuda").to(torch.bfloat16)
        kn = torch.randn(2, hkv, d, generator=gen, device="cuda").to(torch.bfloat16)
        vn = torch.randn(2, hkv, d, generator=gen, device="cuda").to(torch.bfloat16)
        view = cache.layer(li)
        out = mi.paged_decode_store(q, view.keys, view.values, table.cuda(), ctx, kn, vn,
                                    new_slots.cuda())
        torch.cuda.synchronize()
        for i in range(2):
            keys = torch.cat([hist[li][0], kn[i:i + 1]]).float()
            vals = torch.cat([hist[li][1], vn[i:i + 1]]).float()
            kh = keys.repeat_interleave(hq // hkv, dim=1)  # [21, hq, d]
            vh = vals.repeat_interleave(hq // hkv, dim=1)
            sc = torch.einsum("hd,thd->ht", q[i].float(), kh) * d ** -0.5
            want = torch.einsum("ht,thd->hd", torch.softmax(sc, dim=-1), vh)
            torch.testing.assert_close(out[i].float(), want, atol=2e-2, rtol=1e-2)


def test_mma_plan_takes_one_split_past_half_the_sms():
    """The mma kernel holds one CTA per SM: once the (sequence, kv head) pairs
    exceed half the SMs, the automatic plan uses no split (and no workspace)."""
    if "MICROINFER_B200_DECODE" in os.environ:
        pytest.skip("kernel pinned")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n = sms // 16 + 1  # 2 * n * 8 kv heads > sms
    kernel, split, ws = mi.decode_plan(n, 16, 8, 128, torch.bfloat16, 16, 0, "cuda", 32)
    assert (kernel, split, ws) == ("mma", 1, 0)
    kernel, split, _ = mi.decode_plan(8, 16, 8, 128, torch.bfloat16, 16, 0, "cuda", 256)
    # small batch, 4096-key tables: two splits, as a cluster pair (no workspace)
    assert kernel == "mma_pair" and split == 2


@pytest.mark.parametrize("width", [40, 160])  # 640 / 2560-key table bound
def test_split_workspace_counters_return_to_zero(width):
    """The last split to finish resets its arrival counter, so the shared
    workspace serves the next launch of any shape (fresh inputs every launch,
    so a skipped merge cannot pass on a stale output)."""
    from microinfer_b200.layer import paged_attention as pa

    g = torch.Generator(device="cuda").manual_seed(9)
    kc = (torch.randn(640, 16, 8, 128, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    vc = (torch.randn_like(kc, dtype=torch.float32) * 0.5).to(torch.bfloat16)
    for n, hq in ((1, 32), (64, 16), (3, 8), (16, 64)):
        table = torch.full((n, width), -1, dtype=torch.int32, device="cuda")
        table[:, :32] = torch.randint(0, 640, (n, 32), generator=g, device="cuda",
                                      dtype=torch.int32)
        ctx = torch.randint(1, 513, (n,), generator=g, device="cuda", dtype=torch.int32)
        for split in (2, 5, 37):
            q = torch.randn(n, hq, 128, generator=g, device="cuda").to(torch.bfloat16)
            ref = mi.paged_decode(q, kc, vc, table, ctx, split_k=1)
            out = mi.paged_decode(q, kc, vc, table, ctx, split_k=split)
            torch.testing.assert_close(out, ref, atol=2e-2, rtol=1e-2)
    torch.cuda.synchronize()
    for ws in pa._WORKSPACES[torch.cuda.current_device()]:
        assert int(ws.view(torch.int32)[:16384].abs().sum().item()) == 0


@pytest.mark.parametrize("name", ["cfg1_decode_f32", "cfg2_layer_bf16", "decode_bs64_bf16"])
def test_decode_kernel_agrees_with_prefill_kernel(name):
    """The decode kernels and the varlen prefill kernels are separate code."""
    case = cases.build(name)
    dt = case["dtype"]
    layer = _store(case)
    q, table, ctx = dev(case["query"], dt), dev(case["block_tables"]), dev(case["contexts"])
    a = mi.paged_decode(q, layer.keys, layer.values, table, ctx, scale=case["scale"])
    n = q.shape[0]
    cu_q = torch.arange(n + 1, dtype=torch.int32, device="cuda")
    cu_k = torch.zeros(n + 1, dtype=torch.int32, device="cuda")
    cu_k[1:] = torch.cumsum(ctx, 0)
    b = mi.paged_prefill(q, layer.keys, layer.values, cu_q, cu_k, table, max_seqlen_q=1,
                         scale=case["scale"])
    atol, rtol = TOL[dt]
    torch.testing.assert_close(a.float(), b.float(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("name", PAGED)
def test_gather_is_bit_exact(name):
    case = cases.build(name)
    gold = load_golden(name)
    dt = case["dtype"]
    layer = _store(case)
    keys, values = mi.gather_paged_kv(layer.keys, layer.values, dev(case["block_tables"]),
                                      case["contexts"].tolist(), case["block_size"])
    assert keys.shape[0] == int(gold["gather_rows"])
    assert cases.digest(host(keys, dt)) == str(gold["gather_k_digest"])
    assert cases.digest(host(values, dt)) == str(gold["gather_v_digest"])


@pytest.mark.parametrize("name", [c for c in cases.CASES if cases.kind(c) == "direct"])
def test_direct_prefill_matches_reference(name):
    case = cases.build(name)
    gold = load_golden(name)
    dt = case["dtype"]
    cu = dev(case["cu_seqlens"])
    lengths = np.diff(case["cu_seqlens"])
    out = mi.varlen_prefill(dev(case["query"], dt), dev(case["keys"], dt), dev(case["values"], dt),
                            cu, cu, max_seqlen_q=int(lengths.max()), scale=case["scale"])
    assert_close(out, gold["out"], dt)


def test_copy_on_write_is_bit_exact():
    case = cases.build("cow_bf16")
    gold = load_golden("cow_bf16")
    kp, vp = dev(case["key_pool"], "bf16"), dev(case["value_pool"], "bf16")
    mi.copy_blocks(kp, vp, torch.from_numpy(case["pairs"]))
    assert cases.digest(host(kp, "bf16")) == str(gold["key_pool_digest"])
    assert cases.digest(host(vp, "bf16")) == str(gold["value_pool_digest"])


def test_write_checked_padding_matches_reference():
    case = cases.build("write_checked_f32")
    gold = load_golden("write_checked_f32")
    layer = mi.LayerKVCache(dev(case["key_cache"]), dev(case["value_cache"]))
    layer.write_checked(dev(case["slots"]), dev(case["keys"]), dev(case["values"]))
    np.testing.assert_array_equal(host(layer.keys, "f32"), gold["key_cache"])
    np.testing.assert_array_equal(host(layer.values, "f32"), gold["value_cache"])


@pytest.mark.parametrize("slots", [[0, 8], [0, -2], [0, 0]])
def test_invalid_writes_are_atomic_on_device(slots, cuda_device):
    layer = mi.LayerKVCache(torch.full((2, 4, 1, 2), 7.0, device="cuda"),
                            torch.full((2, 4, 1, 2), 7.0, device="cuda"))
    with pytest.raises(ValueError):
        layer.write_checked(torch.tensor(slots, device="cuda"), torch.zeros(2, 1, 2, device="cuda"),
                            torch.zeros(2, 1, 2, device="cuda"))
    assert (layer.keys == 7).all() and (layer.values == 7).all()


@pytest.mark.parametrize("dtype,hq,hkv,bs", [(2, 16, 8, 16), (2, 32, 8, 16), (1, 16, 8, 64),
                                             (2, 8, 8, 256), (2, 64, 8, 16), (2, 16, 8, 0)])
def test_tensor_core_prefill_is_the_path_taken(dtype, hq, hkv, bs):
    """Qwen3 shapes (D=128, fp16/bf16, block sizes >= 16, dense mode) run on tcgen05."""
    assert _lib.load().mi_prefill_kernel_for(dtype, 128, hq, hkv, bs) == 2


# --- known answers of the reference tests, on the device ---------------------

def test_kat_isolation_and_padding():
    q = torch.zeros(2, 1, 2, device="cuda")
    k = torch.zeros(3, 2, 1, 2, device="cuda")
    v = torch.full_like(k, 999)
    v[2, 0], v[2, 1], v[0, 0] = 2, 4, 10
    table = torch.tensor([[2, -1], [0, -1]], device="cuda")
    out = mi.paged_decode(q, k, v, table, torch.tensor([2, 1], device="cuda"))
    torch.testing.assert_close(out.cpu(), torch.tensor([[[3.0, 3.0]], [[10.0, 10.0]]]))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_kat_large_logits(dtype):
    query = torch.full((1, 2, 4), 1000.0, dtype=dtype, device="cuda")
    keys = torch.full((1, 2, 1, 4), 1000.0, dtype=dtype, device="cuda")
    values = torch.tensor([2.0, 4.0], dtype=dtype, device="cuda").reshape(1, 2, 1, 1).expand_as(
        keys).contiguous()
    table = torch.tensor([[0]], device="cuda")
    out = mi.paged_decode(query, keys, values, table, torch.tensor([2], device="cuda"))
    torch.testing.assert_close(out, torch.full_like(query, 3.0))
    meta = mi.AttentionMetadata.build(is_prefill=True, cu_seqlens_q=torch.tensor([0, 1], device="cuda"),
                                      cu_seqlens_k=torch.tensor([0, 2], device="cuda"),
                                      max_seqlen_q=1, block_tables=table)
    torch.testing.assert_close(mi.paged_attention_meta(query, keys, values, meta),
                               torch.full_like(query, 3.0))


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("prefix,q_len", [(0, 3), (2, 1), (1, 2)])
def test_tiny_paged_causal_gqa(dtype, prefix, q_len):
    """tests/components/test_paged_attention.py:10-46 shape: D=4, bs=2, blocks [2, 0]."""
    rng = np.random.default_rng(prefix * 10 + q_len)
    ctx = prefix + q_len
    q = po.from_f32(rng.standard_normal((q_len, 4, 4), dtype=np.float32), dtype)
    kc = po.from_f32(np.full((3, 2, 2, 4), 1000.0, np.float32), dtype)
    vc = po.from_f32(np.full((3, 2, 2, 4), -1000.0, np.float32), dtype)
    table = [2, 0]
    for pos in range(ctx):
        kc[table[pos // 2], pos % 2] = po.from_f32(rng.standard_normal((2, 4), dtype=np.float32), dtype)
        vc[table[pos // 2], pos % 2] = po.from_f32(rng.standard_normal((2, 4), dtype=np.float32), dtype)
    expected = po.paged_attention(q, kc, vc, np.array([table]), [ctx], [0, q_len], scale=0.5,
                                  dtype=dtype)
    meta = mi.AttentionMetadata.build(
        is_prefill=q_len > 1 or prefix == 0,
        cu_seqlens_q=torch.tensor([0, q_len], device="cuda"),
        cu_seqlens_k=torch.tensor([0, ctx], device="cuda"),
        max_seqlen_q=q_len, context_lens=torch.tensor([ctx], device="cuda"),
        block_tables=torch.tensor([table], device="cuda"))
    out = mi.paged_attention_meta(dev(q, dtype), dev(kc, dtype), dev(vc, dtype), meta, scale=0.5)
    assert_close(out, expected, dtype)


# --- full-size properties ------------------------------------------------------

def test_config2_full_28_layers_split_invariance_and_roundtrip():
    """BASELINE config 2 at full size: 28 layers x 1024 blocks, N=8, ctx U[128,512]."""
    g = torch.Generator(device="cuda").manual_seed(0)
    layers, nb, bs, hkv, hq, d, n = 28, 1024, 16, 8, 16, 128, 8
    pool = mi.KVCache(layers, nb, bs, hkv, d, dtype=torch.bfloat16, device="cuda")
    pool.keys.normal_(generator=g).mul_(0.5)
    pool.values.normal_(generator=g).mul_(0.5)
    ctx = torch.randint(128, 513, (n,), generator=g, device="cuda", dtype=torch.int32)
    need = ((ctx + bs - 1) // bs).tolist()
    perm = torch.randperm(nb, generator=g, device="cuda").to(torch.int32)
    table = torch.full((n, max(need)), -1, dtype=torch.int32, device="cuda")
    at = 0
    for r, k in enumerate(need):
        table[r, :k] = perm[at:at + k]
        at += k
    pos = (ctx - 1).long()
    slots = (table[torch.arange(n, device="cuda"), pos // bs].long() * bs + pos % bs).to(torch.int32)
    q = torch.randn(layers, n, hq, d, generator=g, device="cuda").to(torch.bfloat16)
    kn = torch.randn(layers, n, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    vn = torch.randn(layers, n, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    outs = {}
    for split in (1, 5, 16):
        res = []
        for layer in range(layers):
            view = pool.layer(layer)
            view.write_slots(slots, kn[layer], vn[layer])
            res.append(mi.paged_decode(q[layer], view.keys, view.values, table, ctx, split_k=split))
        outs[split] = torch.stack(res).float()
    torch.testing.assert_close(outs[5], outs[1], atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(outs[16], outs[1], atol=2e-2, rtol=1e-2)
    # store -> gather round trip: the gathered last row of each sequence is the stored token
    view = pool.layer(layers - 1)
    keys, values = mi.gather_paged_kv(view.keys, view.values, table, ctx.tolist(), bs)
    ends = torch.cumsum(ctx.long(), 0) - 1
    assert torch.equal(keys[ends], kn[-1]) and torch.equal(values[ends], vn[-1])
    # spot-check one layer against the oracle
    dt = "bf16"
    expected = po.paged_decode(host(q[0], dt), host(pool.keys[0], dt), host(pool.values[0], dt),
                               table.cpu().numpy(), ctx.cpu().numpy(), scale=1 / math.sqrt(d),
                               dtype=dt)
    assert_close(outs[1][0].to(torch.bfloat16), expected, dt)


def test_decode_is_cuda_graph_capturable():
    case = cases.build("cfg2_layer_bf16")
    dt = case["dtype"]
    layer = _store(case)
    q = dev(case["query"], dt)
    table = dev(case["block_tables"])
    ctx = dev(case["contexts"])
    split = mi.select_split_k(q.shape[0], 8, q.device)
    eager = mi.paged_decode(q, layer.keys, layer.values, table, ctx, split_k=split)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        mi.paged_decode(q, layer.keys, layer.values, table, ctx, split_k=split)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = mi.paged_decode(q, layer.keys, layer.values, table, ctx, split_k=split)
    graph.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out, eager)
    # replay with shorter contexts: the graph reads context_lens from the device
    ctx.sub_(7)
    expected = mi.paged_decode(q, layer.keys, layer.values, table, ctx, split_k=split)
    graph.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out, expected)


# --- device status: bad ids are flagged and skipped, never dereferenced -------

def test_bad_block_id_is_flagged_not_dereferenced(cuda_device):
    kc = torch.randn(4, 16, 8, 128, device="cuda").to(torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(1, 16, 128, device="cuda").to(torch.bfloat16)
    table = torch.tensor([[0, 1_000_000]], dtype=torch.int32, device="cuda")
    mi.paged_decode(q, kc, vc, table, torch.tensor([20], device="cuda"), split_k=1)
    assert _lib.read_device_status(cuda_device) & _lib.DEV_BAD_BLOCK
    # context longer than the table row: read stops at the row's end
    table = torch.tensor([[0, 1]], dtype=torch.int32, device="cuda")
    mi.paged_decode(q, kc, vc, table, torch.tensor([40], device="cuda"), split_k=2)
    assert _lib.read_device_status(cuda_device) & _lib.DEV_BAD_BLOCK
    with pytest.raises(RuntimeError):
        mi.paged_decode(q, kc, vc, table, torch.tensor([40], device="cuda"), split_k=1)
        mi.check_device_status(cuda_device)


def test_bad_slot_is_flagged_not_written(cuda_device):
    kc = torch.zeros(2, 4, 1, 8, device="cuda")
    vc = torch.zeros_like(kc)
    mi.store_kv_slots(kc, vc, torch.tensor([3, 99], dtype=torch.int32, device="cuda"),
                      torch.ones(2, 1, 8, device="cuda"), torch.ones(2, 1, 8, device="cuda"))
    assert _lib.read_device_status(cuda_device) & _lib.DEV_BAD_SLOT
    assert kc.sum().item() == 8 and vc.sum().item() == 8


def test_bounded_wait_times_out_and_context_survives(cuda_device):
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = _lib.status_buffer(cuda_device)
    _lib.call("mi_wait_flag_selftest", flag.data_ptr(), 200_000_000, status.data_ptr(),
              _lib.stream_of(cuda_device))
    assert _lib.read_device_status(cuda_device) & _lib.DEV_TIMEOUT
    # flag already set: returns at once, no timeout
    flag.fill_(1)
    _lib.call("mi_wait_flag_selftest", flag.data_ptr(), 200_000_000, status.data_ptr(),
              _lib.stream_of(cuda_device))
    assert _lib.read_device_status(cuda_device) == 0
    assert (torch.ones(4, device="cuda") * 2).sum().item() == 8


# --- warp-level MMA decode over the shapes the golden cases do not reach ----

@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("d,g", [(64, 1), (64, 8), (128, 4), (128, 8)])
@pytest.mark.parametrize("bs,split", [(16, 1), (32, 3), (64, 0)])
@pytest.mark.parametrize("fused", [False, True])
def test_mma_decode_shapes_match_oracle(dtype, d, g, bs, split, fused):
    torch_dt = TORCH[dtype]
    n, hkv, nb = 3, 2, 48
    hq = hkv * g
    gen = torch.Generator().manual_seed(d * 100 + g * 10 + bs)
    ctx = torch.randint(1, nb * bs // n, (n,), generator=gen, dtype=torch.int32)
    width = (int(ctx.max()) + bs - 1) // bs
    table = torch.full((n, width), -1, dtype=torch.int32)
    perm = torch.randperm(nb, generator=gen).to(torch.int32)
    at = 0
    for r in range(n):
        k = (int(ctx[r]) + bs - 1) // bs
        table[r, :k] = perm[at:at + k]
        at += k
    kernel, _, _ = mi.decode_plan(n, hq, hkv, d, torch_dt, bs, split, "cuda", width)
    if "MICROINFER_B200_DECODE" not in os.environ:
        assert kernel in ("mma", "mma_pair")
    kc = (torch.randn(nb, bs, hkv, d, generator=gen) * 0.5).to(torch_dt).cuda()
    vc = (torch.randn(nb, bs, hkv, d, generator=gen) * 0.5).to(torch_dt).cuda()
    q = torch.randn(n, hq, d, generator=gen).to(torch_dt).cuda()
    table_d, ctx_d = table.cuda(), ctx.cuda()
    scale = 1.0 / math.sqrt(d)
    if fused:
        kn = (torch.randn(n, hkv, d, generator=gen) * 0.5).to(torch_dt).cuda()
        vn = (torch.randn(n, hkv, d, generator=gen) * 0.5).to(torch_dt).cuda()
        pos = (ctx - 1).long()
        slots = (table[torch.arange(n), pos // bs].long() * bs + pos % bs).to(torch.int32).cuda()
        out = mi.paged_decode_store(q, kc, vc, table_d, ctx_d, kn, vn, slots, scale=scale,
                                    split_k=split or None, early_kv=True)
    else:
        out = mi.paged_decode(q, kc, vc, table_d, ctx_d, scale=scale, split_k=split or None)
    torch.cuda.synchronize()
    expected = po.paged_decode(host(q, dtype), host(kc, dtype), host(vc, dtype), table.numpy(),
                               ctx.numpy(), scale=scale, dtype=dtype)
    assert_close(out, expected, dtype)


@pytest.mark.parametrize("poison", [float("inf"), float("nan"), -float("inf")])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_non_finite_rows_past_the_context_never_reach_the_output(poison, dtype, cuda_device):
    """Pool rows past each context (inside its last, partial page, and the rest of the
    pool) hold Inf or NaN, as a freed page reused after an overflow could.  The reference
    slices exactly `ctx` rows, so its output stays finite; the tcgen05 prefill (multi-token
    chunks, partial 16-key groups at the end of every context), the mma decode and the dense
    prefill must too.  Rows within the contexts are finite random values."""
    torch_dt = TORCH[dtype]
    hq, hkv, d, bs = 16, 8, 128, 16
    q_lens, contexts = [150, 37, 1, 129], [173, 37, 301, 500]
    need = [(c + bs - 1) // bs for c in contexts]
    nb = sum(need) + 2
    g = torch.Generator(device="cpu").manual_seed(41)
    table = torch.full((len(contexts), max(need)), -1, dtype=torch.int32)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    at = 0
    for r, k in enumerate(need):
        table[r, :k] = perm[at:at + k]
        at += k
    kc = torch.full((nb, bs, hkv, d), poison, dtype=torch.float32)
    vc = torch.full_like(kc, poison)
    for r, c in enumerate(contexts):  # finite rows only inside the contexts
        for pos in range(c):
            blk, off = int(table[r, pos // bs]), pos % bs
            kc[blk, off] = torch.randn(hkv, d, generator=g)
            vc[blk, off] = torch.randn(hkv, d, generator=g)
    kc, vc = kc.to(torch_dt).to(cuda_device), vc.to(torch_dt).to(cuda_device)
    total = sum(q_lens)
    q = torch.randn(total, hq, d, generator=g).to(torch_dt).to(cuda_device)
    cu_q = torch.tensor([0] + np.cumsum(q_lens).tolist(), dtype=torch.int32)
    cu_k = torch.tensor([0] + np.cumsum(contexts).tolist(), dtype=torch.int32)
    out = mi.paged_prefill(q, kc, vc, cu_q.to(cuda_device), cu_k.to(cuda_device),
                           table.to(cuda_device), max_seqlen_q=max(q_lens))
    assert torch.isfinite(out.float()).all(), "prefill read a non-finite row past a context"
    expected = po.paged_attention(host(q, dtype), host(kc, dtype), host(vc, dtype),
                                  table.numpy(), contexts, cu_q.numpy(), scale=1 / math.sqrt(d),
                                  dtype=dtype)
    assert_close(out, expected, dtype)
    # decode over the same pool (one query per sequence), with and without splits
    qd = torch.randn(len(contexts), hq, d, generator=g).to(torch_dt).to(cuda_device)
    ctx_d = torch.tensor(contexts, dtype=torch.int32, device=cuda_device)
    exp_d = po.paged_decode(host(qd, dtype), host(kc, dtype), host(vc, dtype), table.numpy(),
                            contexts, scale=1 / math.sqrt(d), dtype=dtype)
    for split in (1, 3):
        outd = mi.paged_decode(qd, kc, vc, table.to(cuda_device), ctx_d, split_k=split)
        assert torch.isfinite(outd.float()).all()
        assert_close(outd, exp_d, dtype)
    # dense (no-prefix) prefill whose last sequence ends inside a 16-row group and is
    # followed by non-finite rows of the packed tensor
    lens = [40, 21]
    kd = torch.randn(64, hkv, d, generator=g).to(torch_dt)
    vd = torch.randn(64, hkv, d, generator=g).to(torch_dt)
    kd[61:], vd[61:] = poison, poison
    qd2 = torch.randn(61, hq, d, generator=g).to(torch_dt)
    cu = torch.tensor([0, 40, 61], dtype=torch.int32)
    outv = mi.varlen_prefill(qd2.to(cuda_device), kd.to(cuda_device), vd.to(cuda_device),
                             cu.to(cuda_device), cu.to(cuda_device), max_seqlen_q=max(lens))
    assert torch.isfinite(outv.float()).all()
    exp_v = po.dense_varlen_attention(host(qd2, dtype), host(kd[:61], dtype), host(vd[:61], dtype),
                                      cu.numpy(), scale=1 / math.sqrt(d), dtype=dtype)
    assert_close(outv, exp_v, dtype)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("d,g", [(64, 1), (128, 2), (128, 4), (64, 8), (128, 8)])
@pytest.mark.parametrize("lo,hi", [(1, 40), (100, 600)])
@pytest.mark.parametrize("fused", [False, True])
def test_cluster_pair_decode_matches_oracle(dtype, d, g, lo, hi, fused):
    """Small batches take the cluster-pair plan: two CTAs per (sequence, kv head),
    every other 16-key chunk each, merged through distributed shared memory.
    Contexts from 1 key (the second CTA has no chunk at all) up to 600; with the
    fused store the new token's chunk belongs to either CTA.  Twice in a row."""
    torch_dt = TORCH[dtype]
    n, hkv, bs = 5, 4, 16
    hq = hkv * g
    gen = torch.Generator().manual_seed(d + g + lo)
    ctx = torch.randint(lo, hi + 1, (n,), generator=gen, dtype=torch.int32)
    need = [(int(c) + bs - 1) // bs for c in ctx]
    nb = sum(need) + 3
    width = max(need)
    table = torch.full((n, width), -1, dtype=torch.int32)
    perm = torch.randperm(nb, generator=gen).to(torch.int32)
    at = 0
    for r, k in enumerate(need):
        table[r, :k] = perm[at:at + k]
        at += k
    kernel, split, ws = mi.decode_plan(n, hq, hkv, d, torch_dt, bs, 0, "cuda", width)
    if "MICROINFER_B200_DECODE" in os.environ or os.environ.get("MICROINFER_B200_DECODE_PAIR") == "0":
        pytest.skip("kernel pinned")
    assert (kernel, split, ws) == ("mma_pair", 2, 0)
    kc = (torch.randn(nb, bs, hkv, d, generator=gen) * 0.5).to(torch_dt).cuda()
    vc = (torch.randn(nb, bs, hkv, d, generator=gen) * 0.5).to(torch_dt).cuda()
    table_d, ctx_d = table.cuda(), ctx.cuda()
    for rep in range(2):
        q = torch.randn(n, hq, d, generator=gen).to(torch_dt).cuda()
        if fused:
            kn = (torch.randn(n, hkv, d, generator=gen) * 0.5).to(torch_dt).cuda()
            vn = (torch.randn(n, hkv, d, generator=gen) * 0.5).to(torch_dt).cuda()
            pos = (ctx - 1).long()
            slots = (table[torch.arange(n), pos // bs].long() * bs + pos % bs).to(torch.int32)
            out = mi.paged_decode_store(q, kc, vc, table_d, ctx_d, kn, vn, slots.cuda(),
                                        early_kv=rep == 1)
        else:
            out = mi.paged_decode(q, kc, vc, table_d, ctx_d)
        torch.cuda.synchronize()
        expected = po.paged_decode(host(q, dtype), host(kc, dtype), host(vc, dtype),
                                   table.numpy(), ctx.numpy(), scale=1.0 / math.sqrt(d),
                                   dtype=dtype)
        assert_close(out, expected, dtype)
