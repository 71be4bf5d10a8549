"""Host-side page allocator (worker/block_manager.py): the reference block
manager's prefix cache, replayed on a recorded trace, plus copy-on-write.

The trace (``tests/golden/block_trace.py``) was recorded from the reference
``BlockManager`` itself (``tests/golden/make_block_golden.py``); every record
(reuse counts, block tables, free pages, stats) must match.  Copy-on-write has
no reference counterpart (the reference never shares a partial page), so those
cases check the allocator's invariants and, on the CPU oracle, that a forked
sequence writing into a shared partial page leaves the other's attention as it
was.
"""
import importlib.util
import inspect
import json
import sys
from pathlib import Path

import numpy as np
import pytest

from microinfer_b200.worker.block_manager import CowBlockManager
from oracle import paged_oracle as po
from tests.conftest import GOLDEN
from tests.golden.block_trace import TraceSequence, run_trace


def Seq(num_tokens, block_size=16, first=1):
    s = TraceSequence(list(range(first, first + num_tokens)))
    s.block_size = block_size
    return s


@pytest.mark.parametrize("seed", ["0", "1", "2"])
def test_trace_matches_the_reference_block_manager(seed):
    trace = json.loads((GOLDEN / "block_manager_trace.json").read_text())[seed]
    got = run_trace(CowBlockManager(trace["pages"], 4), TraceSequence, int(seed), trace["steps"])
    want = trace["records"]
    assert len(got) == len(want)
    for i, (g, w) in enumerate(zip(got, want)):
        assert g == w, f"record {i} differs: ours {g}, reference {w}"


def test_prefix_hits_are_checked_by_tokens_and_never_take_the_last_page():
    m = CowBlockManager(8, 4)
    a = Seq(10, 4)  # pages [1-4] [5-8] [9-10]
    assert m.can_allocate(a) == 0
    m.allocate(a, 0)
    a.num_scheduled_tokens = 10
    m.hash_blocks(a)  # publishes the two full pages
    a.num_cached_tokens, a.num_scheduled_tokens = 10, 0
    b = Seq(9, 4)  # same first 8 tokens, then its own 9th
    assert m.can_allocate(b) == 2
    m.allocate(b, 2)
    assert b.block_table[:2] == a.block_table[:2] and b.num_cached_tokens == 8
    assert m.ref_count[a.block_table[0]] == 2 and b.block_table[2] != a.block_table[2]
    c = Seq(8, 4)  # exactly two full pages: the last is never reused
    assert m.can_allocate(c) == 1
    d = Seq(10, 4, first=2)  # different tokens: no hit
    assert m.can_allocate(d) == 0
    assert m.stats()["prefix_cache_hit_blocks"] == 2


def test_may_append_copies_a_shared_write_page():
    """The scheduler's convention: before a decode step the token at num_tokens - 1
    is the one stored; a fork shares the partial page it goes to."""
    m = CowBlockManager(8, 4)
    a = Seq(6, 4)
    m.allocate(a, 0)
    b = Seq(6, 4)
    m.fork(a, b)
    for s in (a, b):  # each samples its own 7th token
        s.append_token(100 + len(s.block_table))
    assert m.can_append(b)
    m.may_append(b)
    assert b.block_table[1] != a.block_table[1] and b.block_table[0] == a.block_table[0]
    m.may_append(a)  # a is alone on the old page now: no copy
    assert m.take_copies() == [(a.block_table[1], b.block_table[1])]


def test_allocate_fork_free_balance():
    m = CowBlockManager(8, 16)
    a = Seq(20)  # 2 pages, the second partial
    m.allocate(a, 0)
    assert m.num_free_blocks == 6 and [m.ref_count[b] for b in a.block_table] == [1, 1]
    b = Seq(20)
    m.fork(a, b)
    assert b.block_table == a.block_table and [m.ref_count[x] for x in a.block_table] == [2, 2]
    m.deallocate(a)
    assert m.num_free_blocks == 6  # b keeps both pages
    m.deallocate(b)
    assert m.num_free_blocks == 8 and sum(m.ref_count) == 0


def test_append_into_shared_partial_page_copies_once():
    m = CowBlockManager(8, 16)
    a = Seq(20)
    m.allocate(a, 0)
    b = Seq(20)
    m.fork(a, b)
    shared = a.block_table[1]
    slot_b = m.prepare_append(b)  # position 20: page 1, offset 4, shared -> private copy
    new = b.block_table[1]
    assert new != shared and slot_b == new * 16 + 4
    assert b.block_table[0] == a.block_table[0]  # full page stays shared
    # a is the only sequence left on the old page: it appends in place, no copy
    slot_a = m.prepare_append(a)
    assert a.block_table[1] == shared and slot_a == shared * 16 + 4
    assert m.take_copies() == [(shared, new)]
    assert m.take_copies() == []
    assert m.ref_count[shared] == 1 and m.ref_count[new] == 1 and m.ref_count[a.block_table[0]] == 2


def test_append_at_page_boundary_takes_a_fresh_page():
    m = CowBlockManager(4, 16)
    a = Seq(16)
    m.allocate(a, 0)
    b = Seq(16)
    m.fork(a, b)
    slot = m.prepare_append(b)  # position 16 starts page 1: nothing to copy
    assert len(b.block_table) == 2 and slot == b.block_table[1] * 16
    assert m.take_copies() == []


def test_exclusive_partial_page_needs_no_copy():
    m = CowBlockManager(4, 16)
    a = Seq(5)
    m.allocate(a, 0)
    assert m.prepare_append(a) == a.block_table[0] * 16 + 5
    assert m.take_copies() == []


def test_queued_copy_pins_its_source_until_issued():
    m = CowBlockManager(3, 16)
    a = Seq(4)
    m.allocate(a, 0)
    b = Seq(4)
    m.fork(a, b)
    src = a.block_table[0]
    m.prepare_append(b)  # copy src -> fresh
    m.deallocate(a)  # a gone: src must survive until the copy is handed out
    assert src not in list(m._free)
    pairs = m.take_copies()
    assert pairs == [(src, b.block_table[0])]
    assert src in list(m._free)  # released once the copy has been issued


def test_freed_destination_drops_its_copy():
    m = CowBlockManager(3, 16)
    a = Seq(4)
    m.allocate(a, 0)
    b = Seq(4)
    m.fork(a, b)
    m.prepare_append(b)
    m.deallocate(b)  # the copy's destination is gone: nothing to issue
    assert m.take_copies() == []
    assert m.num_free_blocks == 2 and m.ref_count[a.block_table[0]] == 1


def test_fork_with_queued_copies_is_refused_and_pool_exhaustion_raises():
    m = CowBlockManager(2, 16)
    a = Seq(4)
    m.allocate(a, 0)
    b = Seq(4)
    m.fork(a, b)
    m.prepare_append(b)
    with pytest.raises(RuntimeError):
        m.fork(a, Seq(4))
    m.take_copies()
    c = Seq(4)
    m.fork(a, c)
    assert not m.can_append(c)  # shared page, no free page for the copy
    with pytest.raises(RuntimeError):
        m.prepare_append(c)
    with pytest.raises(ValueError):
        CowBlockManager(0, 16)


def test_forked_sequences_attend_to_their_own_tokens_on_the_oracle():
    """Parent and child share a partial page; each appends a different token.
    With the copy issued before the stores, each one's decode equals attention
    over its own history, the other's token invisible."""
    rng = np.random.default_rng(7)
    bs, hkv, hq, d, nb = 16, 2, 4, 32, 8
    kc = np.zeros((1, nb, bs, hkv, d), np.float32)
    vc = np.zeros_like(kc)
    m = CowBlockManager(nb, bs)
    a = Seq(20)
    m.allocate(a, 0)
    hist_k = rng.standard_normal((20, hkv, d)).astype(np.float32)
    hist_v = rng.standard_normal((20, hkv, d)).astype(np.float32)
    for pos in range(20):
        blk = a.block_table[pos // bs]
        kc[0, blk, pos % bs], vc[0, blk, pos % bs] = hist_k[pos], hist_v[pos]
    b = Seq(20)
    m.fork(a, b)
    new_k = rng.standard_normal((2, hkv, d)).astype(np.float32)
    new_v = rng.standard_normal((2, hkv, d)).astype(np.float32)
    slots = [m.prepare_append(a), m.prepare_append(b)]
    po.copy_blocks(kc, vc, m.take_copies())  # copies first, then the step's stores
    for i, slot in enumerate(slots):
        kc[0, slot // bs, slot % bs], vc[0, slot // bs, slot % bs] = new_k[i], new_v[i]
    a.num_tokens = b.num_tokens = 21
    q = rng.standard_normal((2, hq, d)).astype(np.float32)
    width = max(len(a.block_table), len(b.block_table))
    tables = np.full((2, width), -1, np.int32)
    tables[0, :len(a.block_table)] = a.block_table
    tables[1, :len(b.block_table)] = b.block_table
    out = po.paged_decode(q, kc[0], vc[0], tables, np.array([21, 21]), scale=d ** -0.5,
                          dtype="float32")
    for i in range(2):  # dense attention over this sequence's own 21 tokens
        keys = np.concatenate([hist_k, new_k[i:i + 1]])
        vals = np.concatenate([hist_v, new_v[i:i + 1]])
        # the query at position 20 sees all 21 keys: plain softmax attention
        g = hq // hkv
        want = np.zeros((hq, d), np.float32)
        for h in range(hq):
            s = keys[:, h // g] @ q[i, h] * d ** -0.5
            p = np.exp(s - s.max())
            want[h] = (p / p.sum()) @ vals[:, h // g]
        np.testing.assert_allclose(out[i], want, rtol=1e-5, atol=1e-5)


REF_TESTS = Path("/root/reference/tests/engine/test_blockmanager.py")


def _reference_block_manager_tests():
    """(name, function, kwargs) for every case of the reference's own block-manager
    tests, parametrize marks expanded; empty when the reference tree is absent."""
    if not REF_TESTS.exists():
        return []
    ref_pkg = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    for p in (str(ref_pkg), "/root/reference"):
        if p not in sys.path:
            sys.path.append(p)  # after this repository: its tests package must not shadow ours
    spec = importlib.util.spec_from_file_location("reference_test_blockmanager", REF_TESTS)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.BlockManager = CowBlockManager  # the module's tests now build our manager
    cases = []
    for name in sorted(n for n in vars(mod) if n.startswith("test_")):
        if name == "test_block_reset_discards_previous_content":
            continue  # a test of the reference's Block class itself
        fn = getattr(mod, name)
        grids = [({},)]
        for mark in getattr(fn, "pytestmark", []):
            if mark.name == "parametrize":
                names = [a.strip() for a in mark.args[0].split(",")]
                vals = [v if len(names) > 1 else (v,) for v in mark.args[1]]
                grids.append(tuple(dict(zip(names, v)) for v in vals))
        combos = [{}]
        for grid in grids:
            combos = [dict(c, **g) for c in combos for g in grid]
        cases += [(f"{name}{sorted(c.items())}", fn, c) for c in combos]
    return cases


@pytest.mark.parametrize("case", _reference_block_manager_tests(), ids=lambda c: c[0])
def test_reference_block_manager_tests_pass_on_ours(case, monkeypatch):
    """The reference's tests/engine/test_blockmanager.py, unchanged, with its
    BlockManager replaced by CowBlockManager and its sequence_cls fixture (the
    reference Sequence with block size 4)."""
    from microinfer.engine.sequence import Sequence

    monkeypatch.setattr(Sequence, "block_size", 4)
    _, fn, kwargs = case
    params = inspect.signature(fn).parameters
    if "sequence_cls" in params:
        kwargs = dict(kwargs, sequence_cls=Sequence)
    fn(**kwargs)
