"""The reference's own modules, unchanged, running on this package after ``install()``.

The reference is imported from its pip install under ``baseline/_ref`` (it
travels to the GPU box with the repository); the tests skip when that install
is absent.  ``install()`` rebinds the module globals the reference looks its
kernels up by; these tests then drive the reference's ``CachedAttention``,
``LayerKVCache`` and ``ModelRunner`` exactly as its own tests do:

* tests/components/test_cache_binding.py:102-136  chunk + chunk + decode over
  physical blocks [2, 0, 3] == dense causal attention;
* tests/components/test_cache_binding.py:138-152  prefix-free prefill keeps
  requests apart;
* tests/integration/test_cuda_graph.py:37-143     graph decode == eager decode
  through the reference runner (block sizes 16 and 256).

and check that only this library's kernels did the attention: the reference's
SDPA fallback is replaced by a function that raises, and the CUDA kernels the
profiler saw are this library's or torch's elementwise/copy kernels, never a
Triton, FlashAttention or SDPA kernel.
"""

import math
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "baseline" / "_ref"

pytestmark = pytest.mark.skipif(not (REF / "microinfer").is_dir(),
                                reason="reference install baseline/_ref is absent")


@pytest.fixture(scope="module")
def ref():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import importlib

    mods = {name: importlib.import_module(f"microinfer.{name}") for name in
            ("layer.cached_attention", "layer.paged_attention", "layer.metadata",
             "worker.kv_cache")}
    return mods


@pytest.fixture
def installed(ref):
    import microinfer_b200 as mi

    replaced = mi.install()
    yield ref
    mi.uninstall(replaced)


def test_install_rebinds_every_dispatch_symbol_and_uninstall_restores(ref):
    import microinfer_b200 as mi
    from microinfer_b200.layer import paged_attention as pa
    from microinfer_b200.worker import kv_store

    cached, paged, kv = (ref["layer.cached_attention"], ref["layer.paged_attention"],
                         ref["worker.kv_cache"])
    before = {n: getattr(cached, n) for n in ("flash_attn_varlen_func", "paged_attention_meta",
                                              "_direct_prefill_flash")}
    inst = sys.modules["microinfer_b200.install"]
    replaced = mi.install()
    try:
        assert cached.flash_attn_varlen_func is inst.flash_attn_varlen_compat
        assert cached._direct_prefill_flash is inst.direct_prefill_compat
        assert cached.paged_attention_meta is pa.paged_attention_meta
        assert paged.paged_attention_meta is pa.paged_attention_meta
        assert paged.flash_attn_varlen_func is inst.flash_attn_varlen_compat
        assert paged.flash_attn_with_kvcache is None
        assert paged.triton_paged_prefill is pa.paged_prefill
        assert paged._gather_paged_kv is pa.gather_paged_kv
        assert kv.store_kv is kv_store.store_kv and kv.HAS_TRITON
    finally:
        mi.uninstall(replaced)
    for name, obj in before.items():
        assert getattr(cached, name) is obj


def test_flash_adapter_refuses_what_the_kernels_do_not_implement():
    from microinfer_b200.install import flash_attn_varlen_compat

    x = torch.zeros(2, 2, 8)
    cu = torch.tensor([0, 2], dtype=torch.int32)
    with pytest.raises(ValueError, match="causal"):
        flash_attn_varlen_compat(x, x, x, cu, cu, 2, 2, causal=False)
    with pytest.raises(ValueError, match="dropout"):
        flash_attn_varlen_compat(x, x, x, cu, cu, 2, 2, dropout_p=0.1, causal=True)
    with pytest.raises(ValueError, match="CUDA|cuda|device"):
        flash_attn_varlen_compat(x, x, x, cu, cu, 2, 2, causal=True)


# ---------------------------------------------------------------------------- GPU
FORBIDDEN = ("flash", "fmha", "sdpa", "scaled_dot", "triton", "_paged_decode_kernel",
             "_paged_prefill_kernel", "_store_kv_kernel", "efficient_attention")


def _no_foreign_attention(prof):
    names = {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}
    foreign = [n for n in names if any(f in n.lower() for f in FORBIDDEN)
               and not n.startswith("void mi::") and "mi::" not in n]
    assert not foreign, f"attention ran outside libmicroinfer_b200: {foreign}"
    assert any("mi::" in n for n in names), f"no kernel of this library ran: {sorted(names)}"


def _dense(q, k, v):
    """Causal GQA attention in fp32 (the reference test's dense_reference)."""
    n, hq, d = q.shape
    rep = hq // k.shape[1]
    kk = k.float().repeat_interleave(rep, 1).transpose(0, 1)
    vv = v.float().repeat_interleave(rep, 1).transpose(0, 1)
    s = q.float().transpose(0, 1) @ kk.transpose(1, 2) / math.sqrt(d)
    s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool, device=q.device), 1),
                      float("-inf"))
    return (s.softmax(-1) @ vv).transpose(0, 1)


def _sdpa_forbidden(*_a, **_k):
    raise AssertionError("the reference's per-request SDPA fallback ran")


SHAPES = [  # (dtype, Hq, Hkv, D, block_size, chunk bounds, tolerance)
    (torch.float32, 4, 2, 4, 2, [(0, 3), (3, 5), (5, 6)], 1e-5),
    (torch.bfloat16, 16, 8, 128, 16, [(0, 20), (20, 40), (40, 41)], 2e-2),
    (torch.float16, 16, 8, 128, 16, [(0, 17), (17, 33), (33, 34)], 2e-2),
]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,hq,hkv,d,bs,chunks,tol", SHAPES)
def test_reference_cached_attention_chunks_then_decode_match_dense(installed, cuda_device,
                                                                   monkeypatch, dtype, hq, hkv,
                                                                   d, bs, chunks, tol):
    cached, meta = installed["layer.cached_attention"], installed["layer.metadata"]
    kvmod = installed["worker.kv_cache"]
    monkeypatch.setattr(cached, "_direct_prefill_sdpa", _sdpa_forbidden)
    total = chunks[-1][1]
    g = torch.Generator(device=cuda_device).manual_seed(0)
    q = torch.randn(total, hq, d, generator=g, device=cuda_device).to(dtype)
    k = torch.randn(total, hkv, d, generator=g, device=cuda_device).to(dtype)
    v = torch.randn(total, hkv, d, generator=g, device=cuda_device).to(dtype)
    expected = _dense(q, k, v)
    pool = kvmod.KVCache(2, 4, bs, hkv, d, dtype=dtype, device=cuda_device)
    backend = cached.CachedAttention()
    backend.bind_cache(pool.layer(1))
    phys = [2, 0, 3]  # logical block i lives in physical block phys[i]
    slots = torch.tensor([phys[p // bs] * bs + p % bs for p in range(total)], device=cuda_device)
    table = torch.tensor([phys], device=cuda_device)
    outputs = []
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        for start, end in chunks:
            if end - start > 1:
                md = meta.AttentionMetadata.build(
                    is_prefill=True, cu_seqlens_q=torch.tensor([0, end - start], device=cuda_device),
                    cu_seqlens_k=torch.tensor([0, end], device=cuda_device),
                    max_seqlen_q=end - start, max_seqlen_k=end,
                    slot_mapping=slots[start:end], block_tables=None if start == 0 else table)
            else:
                md = meta.AttentionMetadata.build(
                    is_prefill=False, slot_mapping=slots[start:end],
                    context_lens=torch.tensor([end], device=cuda_device), block_tables=table)
            outputs.append(backend(q[start:end], k[start:end], v[start:end], md))
        torch.cuda.synchronize()
    _no_foreign_attention(prof)
    torch.testing.assert_close(torch.cat(outputs).float(), expected, atol=tol, rtol=tol / 2)
    assert pool.keys[0].eq(0).all()
    gathered = pool.keys[1][phys].reshape(-1, hkv, d)[:total]
    assert torch.equal(gathered, k)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,hq,hkv,d,tol", [(torch.float32, 4, 2, 4, 1e-5),
                                                 (torch.bfloat16, 16, 8, 128, 2e-2)])
def test_reference_no_prefix_prefill_isolates_requests(installed, cuda_device, monkeypatch,
                                                       dtype, hq, hkv, d, tol):
    cached, meta = installed["layer.cached_attention"], installed["layer.metadata"]
    monkeypatch.setattr(cached, "_direct_prefill_sdpa", _sdpa_forbidden)
    g = torch.Generator(device=cuda_device).manual_seed(1)
    lens = [3, 2, 150]
    cu = [0, 3, 5, 155]
    q = torch.randn(cu[-1], hq, d, generator=g, device=cuda_device).to(dtype)
    k = torch.randn(cu[-1], hkv, d, generator=g, device=cuda_device).to(dtype)
    v = torch.randn(cu[-1], hkv, d, generator=g, device=cuda_device).to(dtype)
    md = meta.AttentionMetadata.build(
        is_prefill=True, cu_seqlens_q=torch.tensor(cu, device=cuda_device),
        cu_seqlens_k=torch.tensor(cu, device=cuda_device), max_seqlen_q=max(lens),
        max_seqlen_k=max(lens))
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        actual = cached.CachedAttention()(q, k, v, md)
        torch.cuda.synchronize()
    _no_foreign_attention(prof)
    expected = torch.cat([_dense(q[a:b], k[a:b], v[a:b]) for a, b in zip(cu, cu[1:])])
    torch.testing.assert_close(actual.float(), expected, atol=tol, rtol=tol / 2)


def _runner_config():
    from microinfer.config import QwenConfig

    return QwenConfig(vocab_size=32, hidden_dim=16, MLP_inter_dim=32, num_q_head=2,
                      num_kv_head=1, head_dim=8, num_hidden_layer=1, max_pos_embed=64,
                      rope_base=10000.0)


def _decode_seq(tokens):
    from microinfer.config import SampleParameter
    from microinfer.engine.sequence import Sequence

    seq = Sequence(tokens, SampleParameter(max_tokens=1, greedy=True, ignore_eos=True))
    seq.block_table = [0]
    seq.num_cached_tokens = len(tokens) - 1
    seq.num_scheduled_tokens = 1
    return seq


@pytest.mark.gpu
@pytest.mark.parametrize("block_size", [16, 256])
def test_reference_runner_graph_decode_matches_eager(installed, cuda_device, block_size):
    """The reference ModelRunner (graph buckets 1/2/4, three requests padded to bucket 4)
    with every attention call on this library: graph tokens == eager tokens."""
    from microinfer.layer.sampler import Sampler
    from microinfer.model.qwen3 import QwenModel
    from microinfer.runner import ModelRunner

    torch.manual_seed(0)
    cfg = _runner_config()
    graph_model = QwenModel(cfg).to("cuda", dtype=torch.bfloat16).eval()
    eager_model = QwenModel(cfg).to("cuda", dtype=torch.bfloat16).eval()
    eager_model.load_state_dict(graph_model.state_dict())
    graph_runner = ModelRunner(graph_model, None, Sampler(), block_size=block_size, device="cuda",
                               use_cuda_graph=True, max_num_seqs=4)
    graph_runner.allocate_kv_cache(2)
    eager_runner = ModelRunner(eager_model, None, Sampler(), block_size=block_size, device="cuda")
    eager_runner.allocate_kv_cache(2)
    assert [bucket.batch for bucket in graph_runner._graph_buckets] == [1, 2, 4]
    graph_seqs = [_decode_seq(t) for t in ([1], [2, 3], [4, 5, 6])]
    eager_seqs = [_decode_seq(t) for t in ([1], [2, 3], [4, 5, 6])]
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        with torch.inference_mode():
            graph_tokens = graph_runner.run(graph_seqs, False)
            eager_tokens = eager_runner.run(eager_seqs, False)
        torch.cuda.synchronize()
    _no_foreign_attention(prof)
    assert graph_tokens == eager_tokens and len(graph_tokens) == 3
    del graph_runner
