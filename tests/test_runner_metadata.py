"""Device-side runner metadata (worker/runner_metadata.py, csrc/runner_meta.cu).

The fixture ``tests/golden/runner_scenario.npz`` holds what the reference's own
``ModelRunner.prepare_prefill`` / ``prepare_decode`` produced over a seeded
engine scenario (``tests/golden/make_runner_golden.py``).  CPU tests pin the
oracle to it and replay the scenario through the host planning with a numpy
model of the kernel; GPU tests replay it through the real launch and compare
every tensor bit for bit.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import microinfer_b200 as mi
from microinfer_b200 import _lib
from oracle import runner_oracle as ro

GOLDEN = Path(__file__).resolve().parent / "golden" / "runner_scenario.npz"


class FakeSeq:
    """Just the fields the runner reads from the reference's ``Sequence``."""

    def __init__(self, seq_id):
        self.seq_id = seq_id
        self.token_ids = []
        self.block_table = []
        self.num_cached_tokens = 0
        self.num_scheduled_tokens = 0

    @property
    def num_tokens(self):
        return len(self.token_ids)

    @property
    def last_token(self):
        return self.token_ids[-1]

    def __len__(self):
        return len(self.token_ids)

    def __getitem__(self, key):
        return self.token_ids[key]


def scenario():
    """Per step (is_prefill, batch, expected outputs, ended seq ids).  ``batch``
    is a function: it sets the step's state on the persistent FakeSeq objects
    (the engine's sequences live across steps) and returns them in order."""
    z = np.load(GOLDEN)
    seqs = {}
    raw = []
    for i in range(int(z["num_steps"])):
        p = f"s{i}_"
        pf = bool(z[p + "is_prefill"])
        states = []
        for j, sid in enumerate(z[p + "seq_ids"].tolist()):
            n = int(z[p + "num_tokens"][j])
            if pf:
                tokens = [int(t) for t in z[p + "tokens"][j, :n]]
            else:  # only the last token matters for decode; keep the length right
                tokens = [0] * (n - 1) + [int(z[p + "last_token"][j])]
            table = [int(b) for b in z[p + "tables"][j, :int(z[p + "num_pages"][j])]]
            states.append((sid, tokens, table, int(z[p + "cached"][j]), int(z[p + "sched"][j])))
        want = {k[len(p) + 4:]: z[k] for k in z.files if k.startswith(p + "out_")}
        want["max_q"], want["max_k"] = int(z[p + "max_q"]), int(z[p + "max_k"])
        raw.append((pf, states, want))

    def batch_of(states):
        def make():
            out = []
            for sid, tokens, table, cached, sched in states:
                s = seqs.setdefault(sid, FakeSeq(sid))
                s.token_ids, s.block_table = list(tokens), list(table)
                s.num_cached_tokens, s.num_scheduled_tokens = cached, sched
                out.append(s)
            return out
        return make

    last_seen = {}
    for k, (_, states, _) in enumerate(raw):
        for st in states:
            last_seen[st[0]] = k
    steps = []
    for k, (pf, states, want) in enumerate(raw):
        ended = [sid for sid, last in last_seen.items() if last == k - 1]
        steps.append((pf, batch_of(states), want, ended))
    return steps, int(z["block_size"]), int(z["num_blocks"])


def snapshot(seqs):
    return [(list(s.token_ids), list(s.block_table), s.num_cached_tokens,
             s.num_scheduled_tokens) for s in seqs]


# --- CPU: oracle against the reference's outputs --------------------------

def test_oracle_matches_reference_runner():
    steps, bs, _ = scenario()
    for pf, make, want, _ in steps:
        got = (ro.prefill_metadata if pf else ro.decode_metadata)(snapshot(make()), bs)
        for key in ("input_ids", "positions", "slot_mapping", "context_lens", "cu_q", "cu_k",
                    "block_tables"):
            if key in want:
                assert got[key] is not None, key
                assert got[key].dtype == want[key].dtype, key
                if key == "block_tables" and not pf:
                    # the reference's decode buffers only ever grow in width
                    w = got[key].shape[1]
                    np.testing.assert_array_equal(got[key], want[key][:, :w])
                    assert (want[key][:, w:] == -1).all()
                else:
                    np.testing.assert_array_equal(got[key], want[key], err_msg=key)
            elif key in ("cu_q", "cu_k", "context_lens", "block_tables"):
                assert key not in got or got[key] is None, key
        if pf:
            assert (got["max_q"], got["max_k"]) == (want["max_q"], want["max_k"])


# --- CPU: host planning + a numpy model of the kernel ----------------------

def emulate(table, plan, bs, prefill):
    """What mi_build_*_metadata computes from a plan, on a numpy page table."""
    rec, upd = plan["records"], plan["updates"]
    for row, _, _, _, begin, count in rec:
        for col, page in upd[begin:begin + count]:
            table[row, col] = page
    out = {}
    if not prefill:
        width = plan["width"]
        out["input_ids"] = rec[:, 2].astype(np.int64)
        out["positions"] = (rec[:, 1] - 1).astype(np.int64)
        out["context_lens"] = rec[:, 1].astype(np.int32)
        out["slot_mapping"] = np.array(
            [table[r, (n - 1) // bs] * bs + (n - 1) % bs for r, n in rec[:, :2]], np.int32)
        bt = np.full((len(rec), width), -1, np.int32)
        for i, (row, _, _, pages, _, _) in enumerate(rec):
            bt[i, :pages] = table[row, :pages]
        out["block_tables"] = bt
        return out
    pos = np.concatenate([np.arange(a, b) for _, a, b, _, _, _ in rec])
    rows = np.concatenate([np.full(b - a, r) for r, a, b, _, _, _ in rec])
    out["input_ids"] = plan["tokens"].astype(np.int64)
    out["positions"] = pos.astype(np.int64)
    out["slot_mapping"] = (table[rows, pos // bs] * bs + pos % bs).astype(np.int32)
    out["cu_q"] = np.concatenate([[0], np.cumsum(rec[:, 2] - rec[:, 1])]).astype(np.int32)
    out["cu_k"] = np.concatenate([[0], np.cumsum(rec[:, 2])]).astype(np.int32)
    if plan["table_width"]:
        bt = np.full((len(rec), plan["table_width"]), -1, np.int32)
        for i, (row, _, _, pages, _, _) in enumerate(rec):
            bt[i, :pages] = table[row, :pages]
        out["block_tables"] = bt
    return out


@pytest.mark.parametrize("verify", [False, True])
def test_host_plan_reproduces_reference_with_emulated_kernel(verify):
    steps, bs, nb = scenario()
    meta = mi.DeviceRunnerMetadata(bs, nb, max_rows=6, device="cpu", verify=verify)
    table = np.full((6, nb), -1, np.int32)
    sent_updates = 0
    whole = 0
    for pf, make, want, ended in steps:
        for sid in ended:
            meta.release(FakeSeq(sid))
        batch = make()
        whole += sum(len(s.block_table) for s in batch)
        plan = meta.plan_prefill(batch) if pf else meta.plan_decode(batch)
        sent_updates += len(plan["updates"])
        got = emulate(table, plan, bs, pf)
        meta._commit(plan["commits"])
        for key, val in got.items():
            exp = want[key]
            if key == "block_tables" and not pf:
                exp = exp[:, :val.shape[1]]
            np.testing.assert_array_equal(val, exp, err_msg=key)
        if pf:
            assert (plan["max_q"], plan["max_k"]) == (want["max_q"], want["max_k"])
            assert ("block_tables" in want) == bool(plan["table_width"])
    # only changed entries cross: far fewer than whole tables every step
    assert sent_updates < whole / 4


def test_plan_rejects_bad_batches():
    meta = mi.DeviceRunnerMetadata(16, 8, max_rows=2, device="cpu")
    s = FakeSeq(1)
    s.token_ids, s.block_table = [5] * 20, [3]  # 20 tokens need 2 pages
    with pytest.raises(ValueError):
        meta.plan_decode([s])
    s.block_table = [3, 99]  # page outside the pool
    with pytest.raises(ValueError):
        meta.plan_decode([s])
    s.block_table = [3, 4]
    with pytest.raises(ValueError):  # same sequence twice
        meta.plan_decode([s, s])
    t, u = FakeSeq(2), FakeSeq(3)
    for x in (t, u):
        x.token_ids, x.block_table = [1], [0]
    meta.plan_decode([s, t])
    meta.release(s)
    meta.plan_decode([t, u])  # s's row went back to the pool
    with pytest.raises(RuntimeError):
        v = FakeSeq(4)
        v.token_ids, v.block_table = [1], [1]
        meta.plan_decode([v])  # both rows taken
    p = FakeSeq(5)
    p.token_ids, p.block_table = [1, 2, 3], [2]
    p.num_cached_tokens, p.num_scheduled_tokens = 2, 2  # past the end
    meta.release(t)
    with pytest.raises(ValueError):
        meta.plan_prefill([p])
    with pytest.raises(ValueError):
        meta.prepare_decode([u])  # CPU tables: there is no CPU path


def test_runner_symbols_declared_and_exported():
    import ctypes

    header = (Path(__file__).resolve().parents[1] / "include" / "microinfer_b200.h").read_text()
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in ("mi_build_decode_metadata", "mi_build_prefill_metadata"):
        assert name + "(" in header
        assert hasattr(lib, name)


# --- GPU: the launch itself ------------------------------------------------

def _check(got, want, key, pf):
    g = got.cpu().numpy()
    exp = want[key]
    assert g.dtype == exp.dtype, key
    np.testing.assert_array_equal(g, exp, err_msg=key)


@pytest.mark.gpu
def test_device_metadata_matches_reference_runner(cuda_device):
    _lib.read_device_status(cuda_device)
    steps, bs, nb = scenario()
    meta = mi.DeviceRunnerMetadata(bs, nb, max_rows=6, device=cuda_device)
    for pf, make, want, ended in steps:
        for sid in ended:
            meta.release(FakeSeq(sid))
        batch = make()
        if pf:
            ids, pos, md = meta.prepare_prefill(batch)
            _check(md.cu_seqlens_q, want, "cu_q", pf)
            _check(md.cu_seqlens_k, want, "cu_k", pf)
            assert (md.max_seqlen_q, md.max_seqlen_k) == (want["max_q"], want["max_k"])
            assert (md.block_tables is None) == ("block_tables" not in want)
            assert md.direct_prefill == ("block_tables" not in want)
        else:
            ids, pos, md = meta.prepare_decode(batch)
            _check(md.context_lens, want, "context_lens", pf)
        _check(ids, want, "input_ids", pf)
        _check(pos, want, "positions", pf)
        _check(md.slot_mapping, want, "slot_mapping", pf)
        if md.block_tables is not None:
            _check(md.block_tables, want, "block_tables", pf)
    torch.cuda.synchronize()
    assert _lib.read_device_status(cuda_device) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [0, 1])
def test_device_metadata_random_engine_against_oracle(seed, cuda_device):
    """Many sequences, random lengths, page growth, copy-on-write replacements,
    finishes and arrivals; every step against the oracle."""
    rng = np.random.default_rng(seed)
    bs, nb, rows = 16, 4096, 64
    meta = mi.DeviceRunnerMetadata(bs, nb, max_rows=rows, device=cuda_device)
    free = list(rng.permutation(nb))
    live, next_id = [], 0
    _lib.read_device_status(cuda_device)
    for step in range(60):
        if len(live) < rows and (step % 5 == 0 or not live):  # arrivals: prefill
            new = []
            for _ in range(int(rng.integers(1, 6))):
                if len(live) + len(new) >= rows:
                    break
                s = FakeSeq(next_id)
                next_id += 1
                n = int(rng.integers(1, 300))
                s.token_ids = [int(x) for x in rng.integers(0, 150000, n)]
                s.block_table = [int(free.pop()) for _ in range((n + bs - 1) // bs)]
                s.num_cached_tokens = int(rng.integers(0, n)) if rng.random() < 0.5 else 0
                s.num_scheduled_tokens = n - s.num_cached_tokens
                new.append(s)
            ids, pos, md = meta.prepare_prefill(new)
            want = ro.prefill_metadata(snapshot(new), bs)
            np.testing.assert_array_equal(ids.cpu().numpy(), want["input_ids"])
            np.testing.assert_array_equal(pos.cpu().numpy(), want["positions"])
            np.testing.assert_array_equal(md.slot_mapping.cpu().numpy(), want["slot_mapping"])
            np.testing.assert_array_equal(md.cu_seqlens_q.cpu().numpy(), want["cu_q"])
            np.testing.assert_array_equal(md.cu_seqlens_k.cpu().numpy(), want["cu_k"])
            if want["block_tables"] is None:
                assert md.block_tables is None
            else:
                np.testing.assert_array_equal(md.block_tables.cpu().numpy(), want["block_tables"])
            for s in new:
                s.token_ids.append(int(rng.integers(0, 150000)))
            live.extend(new)
        for s in live:  # grow, sometimes replace the written page (copy-on-write)
            need = (len(s) + bs - 1) // bs
            while len(s.block_table) < need:
                s.block_table.append(int(free.pop()))
            if rng.random() < 0.1:
                k = (len(s) - 1) // bs
                free.insert(0, s.block_table[k])
                s.block_table[k] = int(free.pop())
        order = list(rng.permutation(len(live)))
        batch = [live[i] for i in order]
        ids, pos, md = meta.prepare_decode(batch)
        want = ro.decode_metadata(snapshot(batch), bs)
        np.testing.assert_array_equal(ids.cpu().numpy(), want["input_ids"])
        np.testing.assert_array_equal(pos.cpu().numpy(), want["positions"])
        np.testing.assert_array_equal(md.slot_mapping.cpu().numpy(), want["slot_mapping"])
        np.testing.assert_array_equal(md.context_lens.cpu().numpy(), want["context_lens"])
        bt = md.block_tables.cpu().numpy()
        w = want["block_tables"].shape[1]
        np.testing.assert_array_equal(bt[:, :w], want["block_tables"])
        assert (bt[:, w:] == -1).all()
        for s in live:
            s.token_ids.append(int(rng.integers(0, 150000)))
        for s in [x for x in live if rng.random() < 0.05]:  # finishes
            live.remove(s)
            meta.release(s)
            free.extend(s.block_table)
    torch.cuda.synchronize()
    assert _lib.read_device_status(cuda_device) == 0


@pytest.mark.gpu
def test_bad_records_are_flagged(cuda_device):
    _lib.read_device_status(cuda_device)
    meta = mi.DeviceRunnerMetadata(16, 8, max_rows=2, device=cuda_device)
    dev = cuda_device
    rec = torch.tensor([[5, 3, 7, 1, 0, 0],      # row outside the table
                        [0, 40, 7, 1, 0, 1]],    # position 39 needs page 2 of 1
                       dtype=torch.int32, device=dev)
    upd = torch.tensor([[0, 9]], dtype=torch.int32, device=dev)  # page outside the pool
    out_i = torch.empty(2, dtype=torch.int64, device=dev)
    out_p = torch.empty(2, dtype=torch.int64, device=dev)
    out_s = torch.empty(2, dtype=torch.int32, device=dev)
    out_c = torch.empty(2, dtype=torch.int32, device=dev)
    out_b = torch.empty(2, 4, dtype=torch.int32, device=dev)
    _lib.call("mi_build_decode_metadata", meta.page_table.data_ptr(), 2, meta.max_pages,
              rec.data_ptr(), 2, upd.data_ptr(), 1, 16, 8, 4, out_i.data_ptr(), out_p.data_ptr(),
              out_s.data_ptr(), out_c.data_ptr(), out_b.data_ptr(),
              _lib.status_buffer(dev).data_ptr(), _lib.stream_of(dev))
    status = _lib.read_device_status(dev)
    assert status & _lib.DEV_BAD_ROW and status & _lib.DEV_BAD_BLOCK
    assert out_s.tolist() == [-1, -1]
    assert (out_b[0] == -1).all() and int(meta.page_table[0, 0]) == -1


@pytest.mark.gpu
def test_persistent_decode_outputs_feed_a_captured_graph(cuda_device):
    """As the reference runner does with its decode buffers: capture attention once
    on the builder's persistent outputs, then each step rebuild the metadata
    (eager, one launch) and replay; the replay must equal an eager decode."""
    _lib.read_device_status(cuda_device)
    bs, nb, hq, hkv, d = 16, 64, 16, 8, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    kc = (torch.randn(nb, bs, hkv, d, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    vc = (torch.randn(nb, bs, hkv, d, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    q = torch.randn(3, hq, d, device="cuda", generator=g).to(torch.bfloat16)
    seqs = []
    for i, n in enumerate((17, 40, 33)):
        s = FakeSeq(i)
        s.token_ids = list(range(n))
        s.block_table = list(range(i * 8, i * 8 + 4))
        seqs.append(s)
    meta = mi.DeviceRunnerMetadata(bs, nb, max_rows=4, max_pages=8, device=cuda_device)
    _, _, md = meta.prepare_decode(seqs)  # sizes the persistent buffers (width 4)
    out = torch.empty_like(q)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        mi.paged_decode(q, kc, vc, md.block_tables, md.context_lens, split_k=1, out=out)
    for step in range(5):
        for s in seqs:
            s.token_ids.append(step)
        _, _, md2 = meta.prepare_decode(seqs)
        assert md2.block_tables.data_ptr() == md.block_tables.data_ptr()
        graph.replay()
        want = mi.paged_decode(q, kc, vc, md2.block_tables.clone(), md2.context_lens.clone(),
                               split_k=1)
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    assert _lib.read_device_status(cuda_device) == 0
