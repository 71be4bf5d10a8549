"""The CPU oracle against the reference's own outputs (golden fixtures) and KATs.

Fixtures come from tests/golden/make_golden.py, which runs the reference
MicroInfer functions on the seeded inputs of tests/golden/cases.py.  These
tests pin the oracle before any kernel is compared with it.
"""

import numpy as np
import pytest

from oracle import paged_oracle as po
from tests.conftest import load_golden
from tests.golden import cases


def _attn_tol(dtype):
    # Oracle and reference both accumulate in fp32; they differ by summation order only.
    return (1e-5, 1e-5) if dtype == "f32" else (2e-2, 1e-2)


def _run_store(case):
    kc, vc = case["key_cache"].copy(), case["value_cache"].copy()
    po.write_checked(kc, vc, case["slots"].astype(np.int64), case["k_new"], case["v_new"])
    return kc, vc


@pytest.mark.parametrize("name", cases.CASES)
def test_inputs_regenerate_bit_exactly(name):
    case = cases.build(name)
    gold = load_golden(name)
    for key in cases.INPUT_KEYS:
        if key in case:
            assert cases.digest(case[key]) == str(gold["digest_" + key]), key


@pytest.mark.parametrize("name", [c for c in cases.CASES
                                  if cases.kind(c) in ("decode", "prefill")])
def test_oracle_matches_reference_store_attention_gather(name):
    case = cases.build(name)
    gold = load_golden(name)
    dt = case["dtype"]
    kc, vc = _run_store(case)
    slots = case["slots"].astype(np.int64)
    bs = case["block_size"]
    assert cases.digest(kc[slots // bs, slots % bs]) == str(gold["stored_k_digest"])
    assert cases.digest(vc[slots // bs, slots % bs]) == str(gold["stored_v_digest"])
    if case["kind"] == "decode":
        cu_q = np.arange(len(case["contexts"]) + 1)
    else:
        cu_q = case["cu_seqlens_q"]
    out = po.paged_attention(case["query"], kc, vc, case["block_tables"], case["contexts"], cu_q,
                             scale=case["scale"], dtype=dt)
    atol, rtol = _attn_tol(dt)
    np.testing.assert_allclose(po.to_f32(out, dt), po.to_f32(gold["out"], dt), atol=atol, rtol=rtol)
    gk, gv = po.gather_paged_kv(kc, vc, case["block_tables"], case["contexts"], bs)
    assert gk.shape[0] == int(gold["gather_rows"])
    assert cases.digest(gk) == str(gold["gather_k_digest"])
    assert cases.digest(gv) == str(gold["gather_v_digest"])


@pytest.mark.parametrize("name", [c for c in cases.CASES if cases.kind(c) == "direct"])
def test_oracle_matches_reference_direct_prefill(name):
    case = cases.build(name)
    gold = load_golden(name)
    dt = case["dtype"]
    out = po.dense_varlen_attention(case["query"], case["keys"], case["values"],
                                    case["cu_seqlens"], scale=case["scale"], dtype=dt)
    atol, rtol = _attn_tol(dt)
    np.testing.assert_allclose(po.to_f32(out, dt), po.to_f32(gold["out"], dt), atol=atol, rtol=rtol)


def test_oracle_copy_on_write_matches_torch_restatement():
    case = cases.build("cow_bf16")
    gold = load_golden("cow_bf16")
    kp, vp = case["key_pool"].copy(), case["value_pool"].copy()
    po.copy_blocks(kp, vp, case["pairs"])
    assert cases.digest(kp) == str(gold["key_pool_digest"])
    assert cases.digest(vp) == str(gold["value_pool_digest"])


def test_oracle_write_checked_matches_reference():
    case = cases.build("write_checked_f32")
    gold = load_golden("write_checked_f32")
    kc, vc = case["key_cache"].copy(), case["value_cache"].copy()
    po.write_checked(kc, vc, case["slots"], case["keys"], case["values"])
    np.testing.assert_array_equal(kc, gold["key_cache"])
    np.testing.assert_array_equal(vc, gold["value_cache"])


# --- known answers from the reference's own tests ---------------------------

def test_kat_requests_cannot_attend_to_each_other_or_padding():
    # tests/components/test_paged_attention.py:49-64 of the reference.
    q = np.zeros((2, 1, 2), np.float32)
    k = np.zeros((3, 2, 1, 2), np.float32)
    v = np.full_like(k, 999)
    v[2, 0], v[2, 1], v[0, 0] = 2, 4, 10
    out = po.paged_attention(q, k, v, np.array([[2, -1], [0, -1]]), [2, 1], [0, 1, 2],
                             scale=1 / np.sqrt(2), dtype="f32")
    np.testing.assert_allclose(out, [[[3.0, 3.0]], [[10.0, 10.0]]])


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_kat_large_logits_do_not_overflow(dtype):
    # tests/components/test_paged_attention.py:82-103 of the reference.
    q = po.from_f32(np.full((1, 2, 4), 1000.0, np.float32), dtype)
    k = po.from_f32(np.full((1, 2, 1, 4), 1000.0, np.float32), dtype)
    v = po.from_f32(np.broadcast_to(np.array([2.0, 4.0], np.float32).reshape(1, 2, 1, 1),
                                    (1, 2, 1, 4)).copy(), dtype)
    out = po.paged_attention(q, k, v, np.array([[0]]), [2], [0, 1], scale=0.5, dtype=dtype)
    np.testing.assert_array_equal(po.to_f32(out, dtype), np.full((1, 2, 4), 3.0, np.float32))


@pytest.mark.parametrize("slots", [[0, 8], [0, -2], [0, 0]])
def test_invalid_writes_are_atomic(slots):
    # tests/components/test_kv_cache.py:35-42 of the reference.
    kc = np.full((2, 4, 1, 2), 7.0, np.float32)
    vc = kc.copy()
    with pytest.raises(ValueError):
        po.write_checked(kc, vc, np.array(slots), np.zeros((2, 1, 2), np.float32),
                         np.zeros((2, 1, 2), np.float32))
    assert (kc == 7).all() and (vc == 7).all()


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5e-41, 3.0e38, np.inf, -np.inf], np.float32)
    import torch

    expected = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(po.f32_to_bf16(x), expected)
    np.testing.assert_array_equal(po.bf16_to_f32(expected), torch.from_numpy(x).to(
        torch.bfloat16).float().numpy())


def test_roofline_accounting_formulas():
    # decode: 2*ctx*Hkv*D*e per sequence + Q/O + table entries + lengths
    assert po.decode_bytes([16], 16, 8, 128, 2, 16) == 2 * 16 * 8 * 128 * 2 + 2 * 16 * 128 * 2 + 4 + 4
    assert po.store_bytes(1, 8, 128, 2) == 4 * 8 * 128 * 2 + 4
    # one chunk of 2 on a prefix of 3: pairs = 2*3 + 3 = 9
    assert po.prefill_flops([2], [5], 1, 1) == 4 * 9
