"""The entry points as torch.library custom ops (microinfer_b200/torch_ops.py):
torch.compile traces a decode / prefill step into one graph of opaque
``microinfer_b200`` nodes (the reference compiles its decode forward,
microinfer/runner.py:88-100), and the compiled step computes what eager does."""
import pytest
import torch

import microinfer_b200 as mi
from microinfer_b200 import _lib


def _capture_backend(graphs):
    """A backend that keeps the traced graph and returns zeros in its place, so
    the trace can be inspected on a machine without the GPU kernels."""

    def backend(gm, example_inputs):
        graphs.append(gm)
        out = [n for n in gm.graph.nodes if n.op == "output"][0].args[0]
        shapes = [n.meta.get("val", n.meta.get("example_value")).shape for n in out]

        def run(*args):
            return tuple(torch.zeros(s) for s in shapes)

        return run

    return backend


def _decode_inputs(device="cpu"):
    g = torch.Generator(device=device).manual_seed(0)
    q = torch.randn(4, 16, 128, generator=g, device=device).to(torch.bfloat16)
    kc = (torch.randn(8, 16, 8, 128, generator=g, device=device) * 0.5).to(torch.bfloat16)
    vc = (torch.randn(8, 16, 8, 128, generator=g, device=device) * 0.5).to(torch.bfloat16)
    bt = torch.tensor([[0, 1], [2, 3], [4, 5], [6, 7]], dtype=torch.int32, device=device)
    ctx = torch.tensor([20, 5, 32, 17], dtype=torch.int32, device=device)
    kn = torch.randn(4, 8, 128, generator=g, device=device).to(torch.bfloat16)
    vn = torch.randn(4, 8, 128, generator=g, device=device).to(torch.bfloat16)
    slots = ((bt.gather(1, ((ctx - 1) // 16).long().unsqueeze(1)).squeeze(1) * 16 +
              (ctx - 1) % 16)).to(torch.int32)
    return q, kc, vc, bt, ctx, kn, vn, slots


def decode_step(q, kc, vc, bt, ctx, kn, vn, slots):
    mi.store_kv_slots(kc, vc, slots, kn, vn)
    md = mi.AttentionMetadata.build(is_prefill=False, slot_mapping=slots, context_lens=ctx,
                                    block_tables=bt)
    return mi.paged_attention_meta(q, kc, vc, md)


def fused_step(q, kc, vc, bt, ctx, kn, vn, slots):
    return mi.paged_decode_store(q, kc, vc, bt, ctx, kn, vn, slots, split_k=2)


def test_fake_kernels_give_output_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q = torch.empty(4, 16, 128, dtype=torch.bfloat16)
        kc = torch.empty(8, 16, 8, 128, dtype=torch.bfloat16)
        idx = torch.empty(4, dtype=torch.int32)
        bt = torch.empty(4, 2, dtype=torch.int32)
        assert torch.ops.microinfer_b200.paged_decode(q, kc, kc, bt, idx, None, None).shape == \
            q.shape
        cu = torch.empty(5, dtype=torch.int32)
        assert torch.ops.microinfer_b200.paged_prefill(q, kc, kc, cu, cu, bt, 1, None).shape == \
            q.shape
        qkv = torch.empty(4, 32 * 128, dtype=torch.bfloat16)
        tab = torch.empty(16, 64)
        out = torch.ops.microinfer_b200.qk_norm_rope_store(qkv, q[0, 0], q[0, 0], idx, tab, tab,
                                                           kc, kc, idx, 16, 8, 1e-6, False)
        assert out.shape == (4, 16, 128) and out.dtype == torch.bfloat16


@pytest.mark.parametrize("step,ops", [(decode_step, ["store_kv_slots", "paged_decode"]),
                                      (fused_step, ["paged_decode_store"])])
def test_step_traces_into_one_graph(step, ops):
    graphs = []
    torch._dynamo.reset()
    f = torch.compile(step, backend=_capture_backend(graphs), fullgraph=True)
    f(*_decode_inputs())
    assert len(graphs) == 1
    code = graphs[0].code
    for op in ops:
        assert f"torch.ops.microinfer_b200.{op}" in code


def test_prefill_with_prologue_traces_into_one_graph():
    graphs = []
    torch._dynamo.reset()

    def step(qkv, w, pos, cos, sin, kc, vc, slots, cu, bt):
        q = mi.qk_norm_rope_store(qkv, w, w, pos, cos, sin, kc, vc, slots, num_q_heads=16,
                                  num_kv_heads=8, eps=1e-6)
        md = mi.AttentionMetadata.build(is_prefill=True, cu_seqlens_q=cu, cu_seqlens_k=cu,
                                        max_seqlen_q=6, slot_mapping=slots, block_tables=bt)
        return mi.paged_attention_meta(q, kc, vc, md)

    t = 6
    args = (torch.randn(t, 32 * 128).to(torch.bfloat16), torch.ones(128, dtype=torch.bfloat16),
            torch.arange(t), torch.ones(16, 64), torch.zeros(16, 64),
            torch.zeros(4, 16, 8, 128, dtype=torch.bfloat16),
            torch.zeros(4, 16, 8, 128, dtype=torch.bfloat16), torch.arange(t, dtype=torch.int32),
            torch.tensor([0, t], dtype=torch.int32), torch.zeros(1, 1, dtype=torch.int32))
    torch.compile(step, backend=_capture_backend(graphs), fullgraph=True)(*args)
    assert len(graphs) == 1
    assert "qk_norm_rope_store" in graphs[0].code and "paged_prefill" in graphs[0].code


@pytest.mark.gpu
@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
@pytest.mark.parametrize("step", [decode_step, fused_step])
def test_compiled_step_matches_eager(backend, step, cuda_device):
    _lib.read_device_status(cuda_device)
    torch._dynamo.reset()
    eager_in = _decode_inputs("cuda")
    comp_in = [t.clone() for t in eager_in]
    want = step(*eager_in)
    got = torch.compile(step, backend=backend, fullgraph=True)(*comp_in)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(comp_in[1], eager_in[1]) and torch.equal(comp_in[2], eager_in[2])
    assert _lib.read_device_status(cuda_device) == 0
