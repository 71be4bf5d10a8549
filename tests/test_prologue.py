"""Attention prologue (q/k RMSNorm + RoPE + k/v store): the oracle restatement
against golden vectors produced by the reference's own modules
(tests/golden/make_prologue_golden.py), and the ABI surface."""
from pathlib import Path

import numpy as np
import pytest
import torch

import microinfer_b200 as mi
from microinfer_b200 import _lib
from oracle import paged_oracle as po

GOLDEN = Path(__file__).resolve().parent / "golden"
PROLOGUE_CASES = ["bf16_d128", "bf16_d64_inter", "f16_d128", "f32_d64"]


def load_prologue(name):
    z = np.load(GOLDEN / f"prologue_{name}.npz")
    dtype = str(z["dtype"])
    d, hq, hkv, tokens, inter = (int(v) for v in z["meta"])

    def arr(key):
        a = z[key]
        return a.view(np.float16) if dtype == "f16" else a

    return dict(dtype=dtype, d=d, hq=hq, hkv=hkv, tokens=tokens, interleaved=bool(inter),
                eps=float(z["eps"]), qkv=arr("qkv"), q_weight=arr("q_weight"),
                k_weight=arr("k_weight"), positions=z["positions"], cos=z["cos"], sin=z["sin"],
                q=arr("q"), k=arr("k"))


def as_f32(a, dtype):
    return po.to_f32(a, dtype)


def pair_norm(w, interleaved):
    """|(a, b)| of the rotated pair each element belongs to (rotation keeps it)."""
    if interleaved:
        partner = w.reshape(*w.shape[:-1], -1, 2)[..., ::-1].reshape(w.shape)
    else:
        half = w.shape[-1] // 2
        partner = np.concatenate([w[..., half:], w[..., :half]], axis=-1)
    return np.hypot(w, partner)


def ulp_close(got, want, dtype, *, interleaved=False, min_exact=0.98):
    """Rotated 16-bit rows: the only freedom is the order of the sum of squares
    inside the norm, which can move a normalised value y by one unit in the last
    place; through out = a*c - b*s (|c|, |s| <= 1) that is at most one unit of
    |(a, b)| on top of the output's own half unit.  So each element must be
    within 2^-p * (|(a, b)| + |out|) and nearly every element bit-equal.  fp32
    results: within 1e-5 relative (that order shows through when no 16-bit
    rounding absorbs it)."""
    g, w = as_f32(got, dtype), as_f32(want, dtype)
    if dtype == "f32":
        np.testing.assert_allclose(g, w, rtol=1e-5, atol=1e-6)
        return
    mant = {"bf16": 7, "f16": 10}[dtype]
    tol = (pair_norm(w, interleaved) + np.maximum(np.abs(w), 2.0 ** -14)) * 2.0 ** -mant
    assert np.all(np.abs(g - w) <= tol * 1.0001), float(np.max(np.abs(g - w) / tol))
    assert np.mean(g == w) >= min_exact, float(np.mean(g == w))


@pytest.mark.parametrize("name", PROLOGUE_CASES)
def test_oracle_matches_reference_prologue(name):
    c = load_prologue(name)
    q, k, v = po.qk_norm_rope(c["qkv"], c["q_weight"], c["k_weight"], c["positions"], c["cos"],
                              c["sin"], num_q_heads=c["hq"], num_kv_heads=c["hkv"],
                              head_dim=c["d"], eps=c["eps"], interleaved=c["interleaved"],
                              dtype=c["dtype"])
    ulp_close(q, c["q"], c["dtype"], interleaved=c["interleaved"])
    ulp_close(k, c["k"], c["dtype"], interleaved=c["interleaved"])
    qkv = c["qkv"].reshape(c["tokens"], c["hq"] + 2 * c["hkv"], c["d"])
    np.testing.assert_array_equal(np.asarray(v).view(np.uint8),
                                  np.ascontiguousarray(qkv[:, c["hq"] + c["hkv"]:]).view(np.uint8))


def test_prologue_symbol_declared_and_exported():
    import ctypes

    header = (Path(__file__).resolve().parents[1] / "include" / "microinfer_b200.h").read_text()
    assert "mi_qk_norm_rope_store(" in header
    assert hasattr(ctypes.CDLL(str(_lib.LIB_PATH)), "mi_qk_norm_rope_store")


# --- sm_100a kernel through the C ABI -------------------------------------

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _torch_dtype(dtype):
    return TORCH_DT[dtype]


def _dev(a, dtype):
    a = np.ascontiguousarray(a)
    if dtype in ("bf16", "f16"):
        return torch.from_numpy(a.view(np.int16)).view(_torch_dtype(dtype)).cuda()
    return torch.from_numpy(a).cuda()


def _host(t, dtype):
    t = t.detach().contiguous().cpu()
    if dtype in ("bf16", "f16"):
        a = t.view(torch.int16).numpy().view(np.uint16).copy()
        return a.view(np.float16) if dtype == "f16" else a
    return t.numpy().copy()


@pytest.fixture
def clean_status(cuda_device):
    _lib.read_device_status(cuda_device)
    yield cuda_device
    assert _lib.read_device_status(cuda_device) == 0, "the prologue flagged a bad slot or position"


def _pool(tokens, hkv, d, dt, block_size=16, seed=0):
    """A pool with room for every token plus spare pages, filled with a marker so
    that untouched slots stay recognisable; slots are a seeded permutation."""
    nb = (tokens + block_size - 1) // block_size + 3
    kc = torch.full((nb, block_size, hkv, d), 7.0, dtype=dt, device="cuda")
    vc = torch.full_like(kc, -7.0)
    g = torch.Generator().manual_seed(seed)
    slots = torch.randperm(nb * block_size, generator=g)[:tokens].to(torch.int32).cuda()
    return kc, vc, slots


@pytest.mark.gpu
@pytest.mark.parametrize("name", PROLOGUE_CASES)
def test_kernel_matches_reference_prologue(name, clean_status):
    c = load_prologue(name)
    dt, d, hq, hkv, t = c["dtype"], c["d"], c["hq"], c["hkv"], c["tokens"]
    tdt = _torch_dtype(dt)
    kc, vc, slots = _pool(t, hkv, d, tdt)
    q = mi.qk_norm_rope_store(
        _dev(c["qkv"], dt), _dev(c["q_weight"], dt), _dev(c["k_weight"], dt),
        torch.from_numpy(c["positions"]).cuda(), torch.from_numpy(c["cos"]).cuda(),
        torch.from_numpy(c["sin"]).cuda(), kc, vc, slots, num_q_heads=hq, num_kv_heads=hkv,
        eps=c["eps"], interleaved=c["interleaved"])
    torch.cuda.synchronize()
    ulp_close(_host(q, dt), c["q"], dt, interleaved=c["interleaved"])
    sl = slots.long().cpu()
    bs = kc.shape[1]
    k_stored = _host(kc.view(-1, hkv, d)[sl.cuda()], dt)
    v_stored = _host(vc.view(-1, hkv, d)[sl.cuda()], dt)
    ulp_close(k_stored, c["k"], dt, interleaved=c["interleaved"])
    qkv = c["qkv"].reshape(t, hq + 2 * hkv, d)
    np.testing.assert_array_equal(np.asarray(v_stored).view(np.uint8),
                                  np.ascontiguousarray(qkv[:, hq + hkv:]).view(np.uint8))
    # every other slot keeps its marker
    mask = torch.ones(kc.shape[0] * bs, dtype=torch.bool)
    mask[sl] = False
    assert bool((kc.view(-1, hkv, d)[mask.cuda()] == 7.0).all())
    assert bool((vc.view(-1, hkv, d)[mask.cuda()] == -7.0).all())


def _torch_prologue(qkv, q_weight, k_weight, positions, cos, sin, hq, hkv, d, eps, interleaved):
    """The reference's eager op sequence restated with torch ops on the device:
    fp32 RMSNorm with one rounding, fp32 rotation with separately rounded
    element-wise ops, one more rounding."""
    t = qkv.shape[0]
    dt = qkv.dtype
    x = qkv.view(t, hq + 2 * hkv, d)

    def norm(v, w):
        vf = v.float()
        inv = 1.0 / torch.sqrt(vf.pow(2).mean(-1, keepdim=True) + eps)
        return (vf * inv * w.float()).to(dt)

    def rope(v):
        vf = v.float()
        c = cos[positions].unsqueeze(1)
        s = sin[positions].unsqueeze(1)
        if interleaved:
            a, b = vf[..., 0::2], vf[..., 1::2]
            return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2).to(dt)
        a, b = vf.chunk(2, dim=-1)
        return torch.cat((a * c - b * s, b * c + a * s), dim=-1).to(dt)

    q = rope(norm(x[:, :hq], q_weight))
    k = rope(norm(x[:, hq:hq + hkv], k_weight))
    return q, k, x[:, hq + hkv:]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("d,hq,hkv,interleaved", [(128, 16, 8, False), (128, 32, 8, True),
                                                  (64, 8, 1, False), (64, 16, 4, True),
                                                  # rows too wide for the shared-memory stages
                                                  # in fp32: the register form
                                                  (128, 96, 16, False), (128, 96, 16, True)])
@pytest.mark.parametrize("tokens", [1, 37, 1500])
def test_kernel_matches_torch_ops(dtype, d, hq, hkv, interleaved, tokens, clean_status):
    tdt = _torch_dtype(dtype)
    g = torch.Generator(device="cuda").manual_seed(tokens * 7 + d)
    qkv = (torch.randn(tokens, (hq + 2 * hkv) * d, device="cuda", generator=g) * 3).to(tdt)
    qw = (torch.rand(d, device="cuda", generator=g) + 0.5).to(tdt)
    kw = (torch.rand(d, device="cuda", generator=g) + 0.5).to(tdt)
    max_pos = 4096
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, d, 2, device="cuda").float() / d))
    ang = torch.outer(torch.arange(max_pos, device="cuda").float(), inv_freq)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    positions = torch.randint(0, max_pos, (tokens,), device="cuda", generator=g)
    if tokens % 2:
        positions = positions.to(torch.int32)
    kc, vc, slots = _pool(tokens, hkv, d, tdt, seed=tokens)
    q = mi.qk_norm_rope_store(qkv, qw, kw, positions, cos, sin, kc, vc, slots, num_q_heads=hq,
                              num_kv_heads=hkv, eps=1e-6, interleaved=interleaved)
    wq, wk, wv = _torch_prologue(qkv, qw, kw, positions.long(), cos, sin, hq, hkv, d, 1e-6,
                                 interleaved)
    torch.cuda.synchronize()
    sl = slots.long()
    ulp_close(_host(q, dtype), _host(wq, dtype), dtype, interleaved=interleaved)
    ulp_close(_host(kc.view(-1, hkv, d)[sl], dtype), _host(wk, dtype), dtype,
              interleaved=interleaved)
    assert torch.equal(vc.view(-1, hkv, d)[sl], wv)


@pytest.mark.gpu
def test_padding_slot_skips_store_and_packed_3d_input(clean_status):
    t, hq, hkv, d = 5, 8, 2, 128
    qkv = torch.randn(t, hq + 2 * hkv, d, device="cuda").to(torch.bfloat16)
    w = torch.ones(d, device="cuda", dtype=torch.bfloat16)
    cos = torch.ones(8, d // 2, device="cuda")
    sin = torch.zeros(8, d // 2, device="cuda")
    kc, vc, _ = _pool(t, hkv, d, torch.bfloat16)
    slots = torch.tensor([0, -1, 5, -1, 9], dtype=torch.int32, device="cuda")
    pos = torch.zeros(t, dtype=torch.int64, device="cuda")
    out = torch.empty(t, hq, d, device="cuda", dtype=torch.bfloat16)
    q = mi.qk_norm_rope_store(qkv, w, w, pos, cos, sin, kc, vc, slots, num_q_heads=hq,
                              num_kv_heads=hkv, eps=1e-6, out=out)
    assert q is out
    flat_k, flat_v = kc.view(-1, hkv, d), vc.view(-1, hkv, d)
    written = {0, 5, 9}
    for s in range(flat_k.shape[0]):
        if s not in written:
            assert bool((flat_k[s] == 7.0).all()) and bool((flat_v[s] == -7.0).all())
    assert torch.equal(flat_v[5], qkv[2, hq + hkv:])
    # identity rotation: q is the plain normalised row
    xf = qkv[:, :hq].float()
    want = (xf / torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    ulp_close(_host(q, "bf16"), _host(want, "bf16"), "bf16")
    # no tokens: nothing launched, q is empty
    empty = mi.qk_norm_rope_store(qkv[:0], w, w, pos[:0], cos, sin, kc, vc, slots[:0],
                                  num_q_heads=hq, num_kv_heads=hkv, eps=1e-6)
    assert empty.shape == (0, hq, d)


@pytest.mark.gpu
def test_bad_slot_and_position_are_flagged_not_used(cuda_device):
    _lib.read_device_status(cuda_device)
    t, hq, hkv, d = 3, 4, 2, 64
    qkv = torch.randn(t, (hq + 2 * hkv) * d, device="cuda")
    w = torch.ones(d, device="cuda")
    cos, sin = torch.ones(4, d // 2, device="cuda"), torch.zeros(4, d // 2, device="cuda")
    kc, vc, _ = _pool(t, hkv, d, torch.float32)
    n_slots = kc.shape[0] * kc.shape[1]
    slots = torch.tensor([0, n_slots, 2], dtype=torch.int32, device="cuda")
    pos = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    mi.qk_norm_rope_store(qkv, w, w, pos, cos, sin, kc, vc, slots, num_q_heads=hq,
                          num_kv_heads=hkv, eps=1e-6)
    assert _lib.read_device_status(cuda_device) == _lib.DEV_BAD_SLOT
    assert bool((kc.view(-1, hkv, d)[1] == 7.0).all())  # nothing landed beside the good slots
    pos = torch.tensor([0, 4, -1], dtype=torch.int32, device="cuda")
    q = mi.qk_norm_rope_store(qkv, w, w, pos, cos, sin, kc, vc, slots[[0, 2, 0]],
                              num_q_heads=hq, num_kv_heads=hkv, eps=1e-6)
    assert _lib.read_device_status(cuda_device) == _lib.DEV_BAD_POSITION
    assert bool((q[1:] == 0).all()) and bool((q[0] != 0).any())


def test_wrapper_rejects_bad_shapes_without_a_device():
    kc = torch.zeros(2, 16, 2, 64)
    qkv = torch.zeros(3, 8 * 64)
    w = torch.ones(64)
    tab = torch.zeros(4, 32)
    pos = torch.zeros(3, dtype=torch.int32)
    slots = torch.zeros(3, dtype=torch.int32)
    with pytest.raises(ValueError):  # 4 + 2*2 heads need 8*64 columns: ok; wrong head count
        mi.qk_norm_rope_store(qkv, w, w, pos, tab, tab, kc, kc.clone(), slots, num_q_heads=5,
                              num_kv_heads=2, eps=1e-6)
    with pytest.raises(ValueError):  # int64 slots
        mi.qk_norm_rope_store(qkv, w, w, pos, tab, tab, kc, kc.clone(), slots.long(),
                              num_q_heads=4, num_kv_heads=2, eps=1e-6)
    with pytest.raises(ValueError):  # table width is not D/2
        mi.qk_norm_rope_store(qkv, w, w, pos, torch.zeros(4, 64), torch.zeros(4, 64), kc,
                              kc.clone(), slots, num_q_heads=4, num_kv_heads=2, eps=1e-6)
    with pytest.raises(ValueError):  # CPU tensors: the sm_100a kernel is the only path
        mi.qk_norm_rope_store(qkv, w, w, pos, tab, tab, kc, kc.clone(), slots, num_q_heads=4,
                              num_kv_heads=2, eps=1e-6)
