"""Sequence sharding host logic on CPU: gloo process groups of two ranks.

The attention itself is per sequence; what sharding adds is the assignment of
sequences to ranks and the token-id all_gather.  Failure detection is tested
on the host only: a rank that dies before the collective makes the survivor's
collective fail within the process-group timeout, with no GPU involved.
"""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from microinfer_b200.sharding import assign_sequences, gather_tokens
from oracle import paged_oracle as po


def test_assignment_is_balanced_deterministic_and_complete():
    contexts = [4096, 128, 2048, 2048, 512, 30000, 1, 900]
    a = assign_sequences(contexts, 3)
    assert sorted(i for shard in a for i in shard) == list(range(len(contexts)))
    assert a == assign_sequences(contexts, 3)
    loads = [sum(contexts[i] for i in shard) for shard in a]
    assert max(loads) == 30000  # the one long sequence sits alone
    assert assign_sequences([5, 5, 5, 5], 2) == [[0, 2], [1, 3]]
    assert assign_sequences([], 4) == [[], [], [], []]
    with pytest.raises(ValueError):
        assign_sequences([1], 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode_tokens(seqs, rng_seed=0):
    """Per-sequence 'sampled token': argmax of the oracle decode output row."""
    rng = np.random.default_rng(rng_seed)
    n, hq, hkv, d, bs, nb = 6, 4, 2, 16, 4, 64
    ctx = rng.integers(1, 40, size=n)
    table = np.arange(nb, dtype=np.int32)[: n * 10].reshape(n, 10)
    kc = rng.standard_normal((nb, bs, hkv, d), dtype=np.float32)
    vc = rng.standard_normal((nb, bs, hkv, d), dtype=np.float32)
    q = rng.standard_normal((n, hq, d), dtype=np.float32)
    sel = list(seqs)
    out = po.paged_decode(q[sel], kc, vc, table[sel], ctx[sel], scale=0.25, dtype="f32")
    return torch.tensor(out[:, 0, :].argmax(-1), dtype=torch.int32), ctx


def _worker(rank, world, port, mode, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
    try:
        _, ctx = _decode_tokens(range(6))
        assignment = assign_sequences(ctx.tolist(), world)
        local, _ = _decode_tokens(assignment[rank])
        if mode == "die" and rank == 1:
            os._exit(3)  # leaves between steps, before the collective
        tokens = gather_tokens(local, assignment)
        result_q.put((rank, "ok", tokens.tolist()))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        result_q.put((rank, "error", repr(exc)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world if mode == "ok" else world - 1):
        rank, status, payload = q.get(timeout=90)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_two_ranks_gather_the_single_process_tokens():
    expected, _ = _decode_tokens(range(6))
    results = _run(2, "ok")
    for rank in (0, 1):
        status, payload = results[rank]
        assert status == "ok", payload
        assert payload == expected.tolist()


def test_dead_rank_surfaces_as_a_collective_error():
    results = _run(2, "die")
    status, payload = results[0]
    assert status == "error"
