"""Benchmark of the B200 paged KV-cache hot path (one JSON line on rank 0).

Workload ("Qwen3-0.6B-shaped decode step, bf16"):
per GPU, 8 sequences with contexts U[128, 512], 16 q heads / 8 kv heads,
head_dim 128, block_size 16, a distinct 1024-block pool per layer (28 layers,
1.88 GB, far larger than L2), pool ~N(0,1)*0.5, random non-contiguous block
tables.  One step = for each of the 28 layers: store_kvcache of the new token
then paged decode attention (split-K + combine), replayed as one CUDA graph.
Multi-GPU: every rank owns its own pool and 8 sequences (weak scaling by
sequence sharding); after the layer loop the ranks all_gather their sampled
token ids over NCCL -- the only collective.

Metric: algorithmic HBM bytes of the step (decode: K/V once per kv head + Q/O
+ tables; store: K/V rows read and written) / device time, summed over ranks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LAYERS, HQ, HKV, D, BS, NB, NSEQ = 28, 16, 8, 128, 16, 1024, 8
E2E_GROUP = 7  # layers per input copy on the end-to-end path
# Sampled-token buffers in flight with N > 1 (step k reuses slot k % n once the
# gather that read it is done); one GPU has no gather and keeps two.  (8 GPUs, 200
# steps: 0.206 ms per step with 4, 0.222 with 32.)
TOKEN_SLOTS = 4
# Whole-step graph of the end-to-end path: inputs go in as runs of layers ending at
# E2E_IN_ENDS (a one-layer first run, so layer 0 waits for 64 KB only), outputs come back as
# runs ending at E2E_OUT_ENDS (a one-layer last run).  On B200 this beat groups of 7 both ways
# (0.212 ms per step against 0.202) and one copy per layer (0.325 ms: each wait on the copy
# stream in front of a decode launch delays it by a few us).
E2E_IN_ENDS = (1, 4, 12, 28)
E2E_OUT_ENDS = (16, 24, 27, 28)
CTX_LO, CTX_HI = 128, 512
METRIC = "paged decode attn HBM GB/s (Qwen3-0.6B decode step, store+decode x28 layers)"
WORKLOAD = "BASELINE configs[1]: Qwen3-0.6B decode step, bf16, 28 layers, batch 8/GPU"


# kernel names for the roofline entry and the ncu summaries that measured them
DECODE_KERNEL_NAMES = {"mma": "paged_decode_mma_kernel", "simt": "paged_decode_kernel",
                       "mma_pair": "paged_decode_mma_kernel (cluster pairs)",
                       "generic": "attn_generic_kernel"}
DECODE_PROFILES = {"mma_pair": "decode_mma_pair_qwen3_0.6b_config2.md"}


def _peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def _profiled_traffic(summary: str):
    """DRAM bytes per launch (read + write) recorded in a profiles/ ncu summary."""
    try:
        for line in (ROOT / "profiles" / summary).read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def make_batch(seed: int, device):
    """Seeded synthetic step on the device (torch generators, no host data)."""
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    ctx = torch.randint(CTX_LO, CTX_HI + 1, (NSEQ,), generator=g, dtype=torch.int32)
    need = [(int(c) + BS - 1) // BS for c in ctx]
    perm = torch.randperm(NB, generator=g).to(torch.int32)
    table = torch.full((NSEQ, max(need)), -1, dtype=torch.int32)
    at = 0
    for r, k in enumerate(need):
        table[r, :k] = perm[at:at + k]
        at += k
    pos = (ctx - 1).long()
    slots = (table[torch.arange(NSEQ), pos // BS].long() * BS + pos % BS).to(torch.int32)
    return ctx, table, slots


def algorithmic_bytes(ctx_list):
    from tests.golden.configs import decode_bytes, store_bytes

    dec = decode_bytes(ctx_list, HQ, HKV, D, 2, BS)
    st = store_bytes(len(ctx_list), HKV, D, 2)
    return dec, st


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.period = period_s
        self.device_index = device_index
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples), "source": "nvml" if self._nv else "unavailable"}


def bench_config(world: int) -> dict:
    """The workload's `config`, identical in both arms."""
    return {"workload": WORKLOAD, "global_batch": NSEQ * world, "per_gpu_batch": NSEQ,
            "context": [CTX_LO, CTX_HI], "layers": LAYERS, "block_size": BS,
            "num_blocks_per_layer": NB, "heads": [HQ, HKV], "head_dim": D,
            "parallelism": f"sequence-sharded x{world}",
            "l2": "inputs larger than L2: 28 distinct layer pools (1.88 GB) per GPU"}


def reference_cpu_baseline(seconds: float = 12.0, pools: int = 4):
    """The reference's own CPU implementation of the step, unmodified, from its
    pip install under baseline/_ref: per layer `LayerKVCache.write_fast` (its
    CPU branch, worker/kv_cache.py:52-79) then `_paged_attention_reference`
    (layer/paged_attention.py:22-67), torch on every host core, over `pools`
    distinct layer pools (0.27 GB, more than a CPU cache) for a bounded sample
    of layers.  None when the install is absent."""
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "microinfer").is_dir():
        return None
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    import torch
    from microinfer.layer.paged_attention import _paged_attention_reference
    from microinfer.worker.kv_cache import LayerKVCache

    from tests.golden.configs import decode_bytes, store_bytes

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ctx, table, slots = make_batch(1000, "cpu")
    g = torch.Generator().manual_seed(0)
    layers = [LayerKVCache((torch.randn(NB, BS, HKV, D, generator=g) * 0.5).to(torch.bfloat16),
                           (torch.randn(NB, BS, HKV, D, generator=g) * 0.5).to(torch.bfloat16))
              for _ in range(pools)]
    q = torch.randn(NSEQ, HQ, D, generator=g).to(torch.bfloat16)
    kn = torch.randn(NSEQ, HKV, D, generator=g).to(torch.bfloat16)
    vn = torch.randn(NSEQ, HKV, D, generator=g).to(torch.bfloat16)
    sl = slots.long()
    blocks, offsets = sl // BS, sl % BS  # AttentionMetadata.slot_indices, once per step
    ctx_list, cu_q = ctx.tolist(), list(range(NSEQ + 1))
    step_b = decode_bytes(ctx_list, HQ, HKV, D, 2, BS) + store_bytes(NSEQ, HKV, D, 2)
    done = 0
    t0 = time.perf_counter()
    while True:
        layer = layers[done % pools]
        layer.write_fast(blocks, offsets, kn, vn)
        _paged_attention_reference(q, layer.keys, layer.values, table, ctx_list, cu_q,
                                   scale=1 / math.sqrt(D))
        done += 1
        el = time.perf_counter() - t0
        if el > seconds or done >= 20 * LAYERS:
            break
    return {"value": round(done * step_b / el / 1e9, 4), "unit": "GB/s", "cores": threads,
            "kind": "reference",
            "sample": f"{done} layer store+decode steps of the same workload through the "
                      f"reference's own write_fast + _paged_attention_reference (baseline/_ref, "
                      f"unmodified; torch CPU, {threads} threads, {pools} distinct layer pools), "
                      f"{el:.1f} s",
            "ms_per_28_layer_step": round(el / done * LAYERS * 1e3, 3)}


def cpu_baseline(seconds: float = 12.0):
    """The oracle port (numpy) on this host's cores over a bounded sample."""
    import numpy as np

    from oracle import paged_oracle as po
    from tests.golden import cases  # noqa: F401  (same generators as the parity tests)

    rng = np.random.default_rng(0)
    ctx = rng.integers(CTX_LO, CTX_HI + 1, size=NSEQ).astype(np.int32)
    need = [(int(c) + BS - 1) // BS for c in ctx]
    perm = rng.permutation(NB)
    table = np.full((NSEQ, max(need)), -1, np.int32)
    at = 0
    for r, k in enumerate(need):
        table[r, :k] = perm[at:at + k]
        at += k
    kc = po.f32_to_bf16(rng.standard_normal((NB, BS, HKV, D), dtype=np.float32) * 0.5)
    vc = po.f32_to_bf16(rng.standard_normal((NB, BS, HKV, D), dtype=np.float32) * 0.5)
    q = po.f32_to_bf16(rng.standard_normal((NSEQ, HQ, D), dtype=np.float32))
    kn = po.f32_to_bf16(rng.standard_normal((NSEQ, HKV, D), dtype=np.float32))
    pos = ctx - 1
    blocks = table[np.arange(NSEQ), pos // BS]
    offsets = pos % BS
    dec, st = algorithmic_bytes(ctx.tolist())
    layers_done = 0
    t0 = time.perf_counter()
    while True:
        po.store_kv(kc, vc, blocks, offsets, kn, kn)
        po.paged_decode(q, kc, vc, table, ctx, scale=1 / math.sqrt(D), dtype="bf16")
        layers_done += 1
        el = time.perf_counter() - t0
        if el > seconds or layers_done >= 4 * LAYERS:
            break
    gbs = layers_done * (dec + st) / el / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"{layers_done} layer store+decode steps of the same workload "
                      f"(numpy oracle, BLAS threads={os.cpu_count()}), {el:.1f} s",
            "ms_per_28_layer_step": round(el / layers_done * LAYERS * 1e3, 3)}


def measure_long_b1(device, reps: int = 20):
    """BASELINE configs[4] run (b): one Qwen3-8B-shaped sequence at 32768 context.

    36 distinct layer pools (36 x 134 MB), store+decode per layer, the split-K
    path with a workspace; returns decode GB/s over a 36-layer graph replay.
    """
    import torch

    import microinfer_b200 as mi

    layers, hq, hkv, ctx_len = 36, 32, 8, 32768
    nb = ctx_len // BS
    pool = mi.KVCache(layers, nb, BS, hkv, D, dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device).manual_seed(5)
    pool.keys.normal_(generator=g).mul_(0.5)
    pool.values.normal_(generator=g).mul_(0.5)
    table = torch.randperm(nb, generator=g, device=device).to(torch.int32).view(1, nb)
    ctx = torch.tensor([ctx_len], dtype=torch.int32, device=device)
    slots = (table[0, -1].long() * BS + BS - 1).to(torch.int32).view(1)
    q = torch.randn(layers, 1, hq, D, generator=g, device=device).to(torch.bfloat16)
    kn = torch.randn(layers, 1, hkv, D, generator=g, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    kernel, split, _ = mi.decode_plan(1, hq, hkv, D, torch.bfloat16, BS, 0, device, nb)
    views = [pool.layer(i) for i in range(layers)]

    def run():
        for i, view in enumerate(views):
            # as in the config-2 step: layer i's decode writes neither layer i+1's pool
            # nor the table, so layer i+1's pages may load early
            mi.paged_decode_store(q[i], view.keys, view.values, table, ctx, kn[i], kn[i], slots,
                                  split_k=None, out=out[i], early_kv=True)

    run()
    torch.cuda.synchronize(device)
    mi.check_device_status(device)
    cu = torch.tensor([0, 1], dtype=torch.int32)
    check = _check_attention(out[-1], q[-1], views[-1].keys, views[-1].values,
                             {"cu_q": cu, "table": table, "contexts": [ctx_len]}, [0],
                             "configs[4] run (b)")
    ms = _graph_ms(device, run, reps, warm=3)
    from tests.golden.configs import decode_bytes, store_bytes

    b = layers * (decode_bytes([ctx_len], hq, hkv, D, 2, BS) + store_bytes(1, hkv, D, 2))
    del pool
    peaks, src = _peaks()
    gbs = b / (ms * 1e-3) / 1e9
    return {"workload": "BASELINE configs[4] run (b): batch 1, context 32768, 32q/8kv, D128, "
                        "36 layers, bs16", "kernel": kernel, "split_k": split,
            "ms_per_step": round(ms, 4),
            "value": round(gbs, 1), "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
            "peak_source": f"hbm_gbs of {src}", "tok_per_s": round(1000.0 / ms, 1),
            "checked": check}


ATOL, RTOL = 2e-2, 1e-2  # the parity tolerance (bf16, fp32 accumulation)


def _check_attention(out, q, kc, vc, b, rows, what):
    """Whole requests `rows` of one timed layer against the reference's
    `_paged_attention_reference` restated in fp32 on the device
    (tests/golden/configs.py), before any timing.  Raises on a mismatch."""
    import torch

    from tests.golden import configs

    cu = [int(x) for x in b["cu_q"].tolist()]
    ref = configs.torch_paged_attention(q, kc, vc, b["table"], b["contexts"], cu,
                                        1.0 / math.sqrt(q.shape[-1]), rows=rows)
    worst = 0.0
    for r in rows:
        s, e = cu[r], cu[r + 1]
        a, x = out[s:e].float(), ref[s:e].float()
        err = (a - x).abs().max().item() if e > s else 0.0
        if not bool(torch.isfinite(a).all()) or not torch.allclose(a, x, atol=ATOL, rtol=RTOL):
            raise RuntimeError(f"{what}: request {r} differs from the reference restatement "
                               f"(max abs err {err:.3g}); not timed")
        worst = max(worst, err)
    return {"requests_checked": len(rows), "max_abs_err": round(worst, 5),
            "against": "fp32 restatement of _paged_attention_reference, 2e-2 abs / 1e-2 rel"}


def _graph_ms(device, run, reps, warm=2):
    """ms per replay of a CUDA graph of `run` (CUDA events on the replay stream)."""
    import torch

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    for _ in range(warm):
        graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream(device)
    e0.record(cur)
    for _ in range(reps):
        graph.replay()
    e1.record(cur)
    torch.cuda.synchronize(device)
    del graph
    return e0.elapsed_time(e1) / reps


def measure_long_batch(device, world: int = 1, rank: int = 0, layers: int = 36, reps: int = 3,
                       pool_budget_gb: float = 100.0):
    """BASELINE configs[4] run (a): 256 Qwen3-8B-shaped sequences, contexts
    U[4096, 32768], 36 layers, sharded by sequence over the ranks.

    Every rank takes the sequences `sharding.assign_sequences` gives it
    (balanced by total context, the decode bytes), owns its own pool and
    block ids, and runs store + decode for its shard, 36 layers in one CUDA
    graph; no collective is on the path.  One layer of the whole batch is
    ~19 GB, so a rank holds as many distinct layer pools as fit in
    `pool_budget_gb` (all 36 at 8 GPUs) and cycles the 36 layer launches over
    them; every pool is far larger than L2.  Throughput = bytes of all 256
    sequences x 36 layers / the slowest rank's time.
    """
    import torch
    import torch.distributed as dist

    import microinfer_b200 as mi
    from microinfer_b200.sharding import assign_sequences
    from tests.golden import configs
    from tests.golden.configs import decode_bytes, store_bytes

    hq, hkv = 32, 8
    full = configs.long_batch(256)
    shard = assign_sequences(full["contexts"], world)[rank]
    contexts = [full["contexts"][i] for i in shard]
    n = len(contexts)
    gen = torch.Generator().manual_seed(70 + rank)
    nb = sum((c + BS - 1) // BS for c in contexts) + 1
    b = configs._finish([1] * n, contexts, configs._tables(gen, contexts, nb), nb)
    layer_bytes = 2 * nb * BS * hkv * D * 2
    pools = max(1, min(layers, int(pool_budget_gb * 1e9 // layer_bytes)))
    pool = mi.KVCache(pools, nb, BS, hkv, D, dtype=torch.bfloat16, device=device)
    gd = torch.Generator(device=device).manual_seed(7 + rank)
    pool.keys.normal_(generator=gd).mul_(0.5)
    pool.values.normal_(generator=gd).mul_(0.5)
    ctx_d = torch.tensor(contexts, dtype=torch.int32, device=device)
    table_d, slots_d = b["table"].to(device), b["slots"].to(device)
    q = torch.randn(layers, n, hq, D, generator=gd, device=device).to(torch.bfloat16)
    kn = torch.randn(layers, n, hkv, D, generator=gd, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    kernel, split, _ = mi.decode_plan(n, hq, hkv, D, torch.bfloat16, BS, 0, device,
                                      table_d.shape[1])
    views = [pool.layer(i) for i in range(pools)]

    def run():
        for i in range(layers):
            v = views[i % pools]
            mi.paged_decode_store(q[i], v.keys, v.values, table_d, ctx_d, kn[i], kn[i], slots_d,
                                  split_k=None, out=out[i], early_kv=True)

    run()
    torch.cuda.synchronize(device)
    mi.check_device_status(device)
    # layer 0 was stored again by later layers sharing its pool: check the last layer
    last = views[(layers - 1) % pools]
    bd = dict(b, table=table_d)
    check = _check_attention(out[layers - 1], q[layers - 1], last.keys, last.values, bd,
                             [0, n - 1] if n > 1 else [0], "configs[4] run (a)")
    ms = _graph_ms(device, run, reps, warm=1)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    total = layers * (decode_bytes(full["contexts"], hq, hkv, D, 2, BS)
                      + store_bytes(len(full["contexts"]), hkv, D, 2))
    del pool, q, kn, out
    torch.cuda.empty_cache()
    peaks, src = _peaks()
    gbs = total / (ms * 1e-3) / 1e9
    return {"workload": "BASELINE configs[4] run (a): 256 seqs, contexts U[4096,32768], 32q/8kv, "
                        f"D128, 36 layers, bs16, sequence-sharded over {world} GPU(s) "
                        "(sharding.assign_sequences by total context)",
            "scaling": "strong (the 256 sequences are fixed as the GPU count grows)",
            "per_rank_sequences": n, "distinct_layer_pools_per_rank": pools,
            "pool_gb_per_rank": round(pools * layer_bytes / 1e9, 1),
            "kernel": kernel, "split_k": split, "ms_per_step": round(ms, 3),
            "value": round(gbs, 1), "unit": "GB/s", "frac_per_gpu": round(gbs / world / peaks["hbm_gbs"], 4),
            "peak_source": f"hbm_gbs of {src}", "tok_per_s": round(256 * 1000.0 / ms, 1),
            "checked": check}


def _prefill_batch(workload: str, device, g=None):
    """BASELINE configs[2] ("mixed") / configs[3] ("prefix") on the device
    (tests/golden/configs.py, the batches the full-size parity tests check)."""
    from tests.golden import configs

    b = configs.mixed_batch() if workload == "mixed" else configs.shared_prefix_batch()
    for k in ("table", "cu_q", "cu_k", "slots"):
        b[k] = b[k].to(device)
    return b


def prefill_kernel_name() -> str:
    """The tcgen05 prefill kernel the library launches."""
    return ("prefill_tc2_kernel (tcgen05, two 128-row query tiles per CTA sharing K/V); "
            "one-token rows of a mixed batch by paged_decode_mma_kernel launched behind it")


def measure_prefill(device, workload: str, layers: int = 28, reps: int = 10):
    """Store + paged prefill per layer (one attention launch for the whole batch).

    mixed  = BASELINE configs[2]: decode rows and prefill chunks in one launch;
    prefix = BASELINE configs[3]: suffix prefill over a shared, refcounted prefix.
    Reports prefill TFLOP/s (exact causal pairs x 2 GEMMs x 2) against the bf16
    tensor peak and, for the mixed batch, the combined bound B/BW + F/peak.
    """
    import torch

    import microinfer_b200 as mi
    from tests.golden.configs import prefill_flops

    g = torch.Generator(device=device).manual_seed(11)
    b = _prefill_batch(workload, device, g)
    pool = mi.KVCache(layers, b["nb"], BS, HKV, D, dtype=torch.bfloat16, device=device)
    pool.keys.normal_(generator=g).mul_(0.5)
    pool.values.normal_(generator=g).mul_(0.5)
    tokens = int(sum(b["q_lens"]))
    q = torch.randn(tokens, HQ, D, generator=g, device=device).to(torch.bfloat16)
    kn = torch.randn(tokens, HKV, D, generator=g, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    views = [pool.layer(i) for i in range(layers)]
    max_q = max(b["q_lens"])

    def run():
        for view in views:
            view.write_slots(b["slots"], kn, kn)
            mi.paged_prefill(q, view.keys, view.values, b["cu_q"], b["cu_k"], b["table"],
                             max_seqlen_q=max_q, out=out)

    run()
    torch.cuda.synchronize(device)
    mi.check_device_status(device)
    ctx = b["contexts"]
    if workload == "mixed":
        dec = sorted(range(24), key=ctx.__getitem__)
        rows = [dec[0], dec[-1], 24, 31]
    else:
        rows = [0, 63]
    check = _check_attention(out, q, views[-1].keys, views[-1].values, b, rows,
                             f"prefill {workload}")
    ms_layer = _graph_ms(device, run, reps, warm=1) / layers
    flops = prefill_flops(b["q_lens"], b["contexts"], HQ, D)
    kv_bytes = sum(2 * c * HKV * D * 2 for c in b["contexts"])
    if workload == "prefix":  # the shared prefix is stored once
        kv_bytes = 2 * (1024 + 64 * 128) * HKV * D * 2
    peaks, src = _peaks()
    tflops = flops / (ms_layer * 1e-3) / 1e12
    res = {"workload": ("BASELINE configs[2]: 24 decode + 8x512 prefill chunks, one launch"
                        if workload == "mixed" else
                        "BASELINE configs[3]: 64 x 128-token suffix on a shared 1024 prefix"),
           "kernel": prefill_kernel_name(), "layers": layers,
           "us_per_layer": round(ms_layer * 1e3, 2), "flops_per_layer": flops,
           "tflops": round(tflops, 1), "tensor_frac": round(tflops / peaks["bf16_tflops"], 4),
           "peak_source": f"bf16_tflops of {src}", "store_tokens": tokens, "checked": check,
           "traffic_ncu": (_profiled_traffic("prefill_tc2_shared_prefix.md")
                           if workload == "prefix" else None)}
    if workload == "mixed":
        t_min = kv_bytes / (peaks["hbm_gbs"] * 1e9) + flops / (peaks["bf16_tflops"] * 1e12)
        res["combined_bound_frac"] = round(t_min / (ms_layer * 1e-3), 4)
        res["kv_bytes_per_layer"] = kv_bytes
    del pool
    return res


def measure_shared_prefix_step(device, layers: int = LAYERS, decode_steps: int = 16, reps: int = 3):
    """BASELINE configs[3] as a whole: copy-on-write of a shared partial page,
    the suffix prefill over the shared prefix, 16 decode steps, and the
    block-table gather, each timed on its own (28 layers, one CUDA graph).

    The reference never shares a partial page, so to exercise copy-on-write
    the shared prefix here is 1016 tokens: pages 0..62 full and page 63 holding
    8 tokens, shared by all 64 sequences.  Each sequence's 128-token suffix
    starts by appending into page 63, so page 63 is first copied to a private
    page per sequence (64 (src, dst) pairs x 28 layers x K and V, one launch);
    the suffix and the 16 decoded tokens then go to the sequence's own pages.
    Decode is reported as logical GB/s (every sequence's context) and as
    unique-byte GB/s (the 63 shared pages counted once): the shared prefix
    stays in L2 across sequences, so logical GB/s can exceed the HBM peak.
    The gather is the reference's gather-plus-varlen input at the prefill
    (`_gather_paged_kv`, every sequence's 1144 rows).
    """
    import torch

    import microinfer_b200 as mi
    from tests.golden import configs
    from tests.golden.configs import (cow_bytes, decode_bytes, gather_bytes, prefill_flops,
                                      store_bytes)

    n, prefix, suffix = 64, 1016, 128
    shared_pages = (prefix + BS - 1) // BS          # 64, the last one partial
    ctx0 = prefix + suffix                           # 1144 after the prefill
    ctx_end = ctx0 + decode_steps                    # 1160 after the decode steps
    own = (ctx_end + BS - 1) // BS - (shared_pages - 1)  # private pages per sequence (incl. copy)
    nb = shared_pages + n * own + 8
    width = (ctx_end + BS - 1) // BS
    table = torch.empty(n, width, dtype=torch.int32)
    pairs = torch.empty(n, 2, dtype=torch.int32)
    for r in range(n):
        base = shared_pages + r * own
        table[r, :shared_pages - 1] = torch.arange(shared_pages - 1)
        table[r, shared_pages - 1:] = torch.arange(base, base + own)
        pairs[r] = torch.tensor([shared_pages - 1, base])
    pre = configs._finish([suffix] * n, [ctx0] * n, table, nb)
    pool = mi.KVCache(layers, nb, BS, HKV, D, dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device).manual_seed(31)
    pool.keys.normal_(generator=g).mul_(0.5)
    pool.values.normal_(generator=g).mul_(0.5)
    views = [pool.layer(i) for i in range(layers)]
    table_d, pairs_d = table.to(device), pairs.to(device)
    cu_q, cu_k, slots = pre["cu_q"].to(device), pre["cu_k"].to(device), pre["slots"].to(device)
    tokens = n * suffix
    q = torch.randn(tokens, HQ, D, generator=g, device=device).to(torch.bfloat16)
    kn = torch.randn(tokens, HKV, D, generator=g, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    qd = torch.randn(decode_steps, n, HQ, D, generator=g, device=device).to(torch.bfloat16)
    knd = torch.randn(decode_steps, n, HKV, D, generator=g, device=device).to(torch.bfloat16)
    outd = torch.empty_like(qd)
    dctx = torch.stack([torch.full((n,), ctx0 + k + 1, dtype=torch.int32)
                        for k in range(decode_steps)]).to(device)
    pos = torch.arange(ctx0, ctx_end)
    dslots = (table[:, pos // BS].long() * BS + (pos % BS)[None, :]).to(torch.int32)
    dslots = dslots.t().contiguous().to(device)  # [step, seq]
    _, split, _ = mi.decode_plan(n, HQ, HKV, D, torch.bfloat16, BS, 0, device, width)
    gk = torch.empty(n * ctx0, HKV, D, dtype=torch.bfloat16, device=device)
    gv = torch.empty_like(gk)

    def cow():
        pool.copy_blocks(pairs_d, check=False)

    def prefill():
        for v in views:
            v.write_slots(slots, kn, kn)
            mi.paged_prefill(q, v.keys, v.values, cu_q, cu_k, table_d, max_seqlen_q=suffix,
                             out=out)

    def decode():
        for k in range(decode_steps):
            for v in views:
                mi.paged_decode_store(qd[k], v.keys, v.values, table_d, dctx[k], knd[k], knd[k],
                                      dslots[k], split_k=None, out=outd[k], early_kv=True)

    def gather():
        for v in views:
            mi.gather_paged_kv(v.keys, v.values, table_d, [ctx0] * n, BS, cu_seqlens_k=cu_k,
                               out=(gk, gv))

    # --- run each phase once in order and check it before any timing -------------
    src_k = pool.keys[:, shared_pages - 1].clone()
    cow()
    torch.cuda.synchronize(device)
    for r in (0, n - 1):
        if not (torch.equal(pool.keys[:, int(pairs[r, 1])], src_k)
                and torch.equal(pool.values[:, int(pairs[r, 1])], pool.values[:, shared_pages - 1])):
            raise RuntimeError("shared-prefix step: copy-on-write page differs from its source")
    del src_k
    prefill()
    torch.cuda.synchronize(device)
    bp = dict(pre, table=table_d)
    check_p = _check_attention(out, q, views[-1].keys, views[-1].values, bp, [0, n - 1],
                               "shared-prefix suffix prefill")
    decode()
    torch.cuda.synchronize(device)
    bd = {"cu_q": torch.arange(n + 1, dtype=torch.int32), "table": table_d,
          "contexts": [ctx_end] * n}
    check_d = _check_attention(outd[-1], qd[-1], views[-1].keys, views[-1].values, bd, [0, n - 1],
                               "shared-prefix decode (last step)")
    gather()
    torch.cuda.synchronize(device)
    lk = views[-1].keys
    for r in (0, n - 1):
        rows = lk[table_d[r].long()].reshape(-1, HKV, D)[:ctx0]
        if not torch.equal(gk[r * ctx0:(r + 1) * ctx0], rows):
            raise RuntimeError("shared-prefix step: gathered rows differ from the pool")
    mi.check_device_status(device)
    ms_cow = _graph_ms(device, cow, reps * 10)
    ms_pre = _graph_ms(device, prefill, reps)
    ms_dec = _graph_ms(device, decode, reps)
    ms_gat = _graph_ms(device, gather, reps)
    mi.check_device_status(device)
    peaks, src = _peaks()
    hbm, tf = peaks["hbm_gbs"], peaks["bf16_tflops"]
    b_cow = cow_bytes(n, layers, BS, HKV, D, 2)
    f_pre = prefill_flops([suffix] * n, [ctx0] * n, HQ, D)
    st_pre = store_bytes(tokens, HKV, D, 2)
    logical = sum(decode_bytes([ctx0 + k + 1] * n, HQ, HKV, D, 2, BS) + store_bytes(n, HKV, D, 2)
                  for k in range(decode_steps))
    shared_rows = (shared_pages - 1) * BS
    unique = sum(2 * (shared_rows + n * (ctx0 + k + 1 - shared_rows)) * HKV * D * 2
                 + 2 * n * HQ * D * 2 + store_bytes(n, HKV, D, 2)
                 for k in range(decode_steps))
    b_gat = gather_bytes([ctx0] * n, HKV, D, 2)
    del pool, gk, gv
    torch.cuda.empty_cache()
    return {
        "workload": "BASELINE configs[3] whole: 64 seqs on a shared 1016-token prefix (pages 0-62 "
                    "full, page 63 shared with 8 tokens), CoW of page 63 per sequence, 128-token "
                    "suffix prefill, 16 decode steps, gather of the 1144-row contexts; 28 layers",
        "cow": {"kernel": "cow_kernel", "pairs": n, "layers": layers,
                "traffic_ncu": _profiled_traffic("cow_kernel_config4_64pairs_28layers.md"),
                "us": round(ms_cow * 1e3, 2), "bytes": b_cow,
                "gbs": round(b_cow / (ms_cow * 1e-3) / 1e9, 1),
                "hbm_frac": round(b_cow / (ms_cow * 1e-3) / 1e9 / hbm, 4)},
        "prefill": {"kernel": prefill_kernel_name(), "us_per_layer": round(ms_pre / layers * 1e3, 2),
                    "tflops": round(f_pre / (ms_pre / layers * 1e-3) / 1e12, 1),
                    "tensor_frac": round(f_pre / (ms_pre / layers * 1e-3) / 1e12 / tf, 4),
                    "includes": "store of the 8192 suffix tokens per layer",
                    "store_bytes_per_layer": st_pre, "checked": check_p},
        "decode": {"kernel": "paged_decode_mma_kernel (store fused)", "split_k": split,
                   "us_per_step": round(ms_dec / decode_steps * 1e3, 2),
                   "us_per_layer": round(ms_dec / decode_steps / layers * 1e3, 3),
                   "logical_gbs": round(layers * logical / (ms_dec * 1e-3) / 1e9, 1),
                   "unique_gbs": round(layers * unique / (ms_dec * 1e-3) / 1e9, 1),
                   "unique_hbm_frac": round(layers * unique / (ms_dec * 1e-3) / 1e9 / hbm, 4),
                   "checked": check_d},
        "gather": {"kernel": "gather_kernel", "us_per_layer": round(ms_gat / layers * 1e3, 2),
                   "traffic_ncu_1152_rows": _profiled_traffic("gather_kernel_config4_64x1152.md"),
                   "bytes_per_layer": b_gat,
                   "gbs": round(b_gat / (ms_gat / layers * 1e-3) / 1e9, 1),
                   "hbm_frac": round(b_gat / (ms_gat / layers * 1e-3) / 1e9 / hbm, 4)},
        "peak_source": f"hbm_gbs / bf16_tflops of {src}",
    }


def measure_store(device, layers: int = LAYERS, reps: int = 20):
    """Standalone store_kvcache (`store_kv_vec16_kernel`) at the prefill token
    counts of configs[2] (4120 tokens) and configs[3] (8192), 28 distinct layer
    pools per step; the written slots are checked bit for bit first."""
    import torch

    import microinfer_b200 as mi
    from tests.golden.configs import store_bytes

    peaks, src = _peaks()
    res = {}
    for label, b in (("configs[2] 4120 tokens", _prefill_batch("mixed", device)),
                     ("configs[3] 8192 tokens", _prefill_batch("prefix", device))):
        pool = mi.KVCache(layers, b["nb"], BS, HKV, D, dtype=torch.bfloat16, device=device)
        g = torch.Generator(device=device).manual_seed(41)
        t = b["tokens"]
        kn = torch.randn(layers, t, HKV, D, generator=g, device=device).to(torch.bfloat16)
        vn = torch.randn(layers, t, HKV, D, generator=g, device=device).to(torch.bfloat16)
        views = [pool.layer(i) for i in range(layers)]

        def run():
            for i, v in enumerate(views):
                v.write_slots(b["slots"], kn[i], vn[i])

        run()
        torch.cuda.synchronize(device)
        sl = b["slots"].long()
        for i in (0, layers - 1):
            if not (torch.equal(views[i].keys.view(-1, HKV, D)[sl], kn[i])
                    and torch.equal(views[i].values.view(-1, HKV, D)[sl], vn[i])):
                raise RuntimeError("store: written rows differ from the inputs")
        ms = _graph_ms(device, run, reps) / layers
        nbytes = store_bytes(t, HKV, D, 2)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[label] = {"us_per_launch": round(ms * 1e3, 2), "bytes_per_launch": nbytes,
                      "gbs": round(gbs, 1), "hbm_frac": round(gbs / peaks["hbm_gbs"], 4)}
        del pool, kn, vn
    return {"kernel": "store_kv_vec16_kernel", "checked": "written rows bit-exact",
            "traffic_ncu_8192_tokens": _profiled_traffic("store_kv_vec16_config4_8192tok.md"),
            "peak_source": f"hbm_gbs of {src}", "rows": res}


def measure_varlen(device, layers: int = LAYERS, reps: int = 10):
    """Prefix-free (direct) prefill through `varlen_prefill` on a configs[2]-sized
    batch: 8 x 512 + 24 x U[1, 64] tokens, contiguous K/V, a distinct K/V pair
    per layer (~0.5 GB over 28 layers, more than L2)."""
    import torch

    import microinfer_b200 as mi
    from tests.golden.configs import prefill_flops

    gen = torch.Generator().manual_seed(16)
    lens = [512] * 8 + torch.randint(1, 65, (24,), generator=gen).tolist()
    total = sum(lens)
    g = torch.Generator(device=device).manual_seed(16)
    q = torch.randn(total, HQ, D, generator=g, device=device).to(torch.bfloat16)
    k = torch.randn(layers, total, HKV, D, generator=g, device=device).to(torch.bfloat16)
    v = torch.randn(layers, total, HKV, D, generator=g, device=device).to(torch.bfloat16)
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0)
    cu_d = cu.to(device)
    out = torch.empty_like(q)

    def run():
        for i in range(layers):
            mi.varlen_prefill(q, k[i], v[i], cu_d, cu_d, max_seqlen_q=512, out=out)

    run()
    torch.cuda.synchronize(device)
    mi.check_device_status(device)
    # the last layer, requests 0 (512 tokens) and 31, against dense causal attention
    rows, worst = (0, len(lens) - 1), 0.0
    for r in rows:
        a, e = int(cu[r]), int(cu[r + 1])
        n = e - a
        kk = k[-1, a:e].float().repeat_interleave(HQ // HKV, 1).transpose(0, 1)
        vv = v[-1, a:e].float().repeat_interleave(HQ // HKV, 1).transpose(0, 1)
        sc = q[a:e].float().transpose(0, 1) @ kk.transpose(1, 2) / math.sqrt(D)
        sc = sc.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool, device=device), 1),
                            float("-inf"))
        ref = (sc.softmax(-1) @ vv).transpose(0, 1)
        got = out[a:e].float()
        if not torch.allclose(got, ref, atol=ATOL, rtol=RTOL):
            raise RuntimeError(f"varlen prefill: request {r} differs from dense attention")
        worst = max(worst, (got - ref).abs().max().item())
    ms = _graph_ms(device, run, reps) / layers
    flops = prefill_flops(lens, lens, HQ, D)
    peaks, src = _peaks()
    tfl = flops / (ms * 1e-3) / 1e12
    del k, v
    return {"workload": "direct prefill, 8 x 512 + 24 x U[1,64] tokens, 16q/8kv, D128, bf16",
            "kernel": "prefill_tc2_kernel (dense mode)", "us_per_layer": round(ms * 1e3, 2),
            "traffic_ncu": _profiled_traffic("prefill_tc2_direct_config3_sized.md"),
            "flops_per_layer": flops, "tflops": round(tfl, 1),
            "tensor_frac": round(tfl / peaks["bf16_tflops"], 4),
            "peak_source": f"bf16_tflops of {src}",
            "checked": {"requests_checked": len(rows), "max_abs_err": round(worst, 5),
                        "against": "fp32 dense causal attention, 2e-2 abs / 1e-2 rel"}}


def _prologue_inputs(device, layers: int, tokens: int, g):
    """Per layer: packed qkv rows [T, (Hq + 2 Hkv) * D], norm weights and a pool
    with room for every token; one RotaryCache-style fp32 table shared by all."""
    import torch

    import microinfer_b200 as mi

    nb = (tokens + BS - 1) // BS
    pool = mi.KVCache(layers, nb, BS, HKV, D, dtype=torch.bfloat16, device=device)
    qkv = torch.randn(layers, tokens, (HQ + 2 * HKV) * D, generator=g,
                      device=device).to(torch.bfloat16)
    qw = (torch.rand(layers, D, generator=g, device=device) + 0.5).to(torch.bfloat16)
    kw = (torch.rand(layers, D, generator=g, device=device) + 0.5).to(torch.bfloat16)
    max_pos = 40960
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=device).float() / D))
    ang = torch.outer(torch.arange(max_pos, device=device).float(), inv_freq)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    positions = torch.randint(0, max_pos, (tokens,), generator=g, device=device)
    slots = torch.randperm(nb * BS, generator=g, device=device)[:tokens].to(torch.int32)
    return pool, qkv, qw, kw, cos, sin, positions, slots


def prologue_bytes(tokens: int) -> int:
    """Algorithmic HBM bytes of one prologue launch (bf16): the packed qkv row read
    once, q written once, k and v written once into the pool, the token's cos/sin
    row (fp32) and its position and slot read once."""
    row = (HQ + 2 * HKV) * D * 2
    return tokens * (row + HQ * D * 2 + 2 * HKV * D * 2 + D * 4 + 8 + 4)


def measure_prologue(device, tokens: int = 8192, layers: int = 8, reps: int = 20):
    """Fused q/k RMSNorm + RoPE + k/v store (one launch per layer) against the
    reference's eager op sequence (FuseLayerNorm x2, RotaryCache.apply x2, slot
    store) written as torch ops, both over `layers` distinct layer buffers so the
    working set (layers x 128 MB) is far larger than L2."""
    import torch

    import microinfer_b200 as mi

    g = torch.Generator(device=device).manual_seed(21)
    pool, qkv, qw, kw, cos, sin, positions, slots = _prologue_inputs(device, layers, tokens, g)
    q_out = torch.empty(layers, tokens, HQ, D, dtype=torch.bfloat16, device=device)
    views = [pool.layer(i) for i in range(layers)]
    sl = slots.long()

    def fused():
        for i, view in enumerate(views):
            mi.qk_norm_rope_store(qkv[i], qw[i], kw[i], positions, cos, sin, view.keys,
                                  view.values, slots, num_q_heads=HQ, num_kv_heads=HKV, eps=1e-6,
                                  out=q_out[i])

    def eager():
        c, s_ = cos[positions].unsqueeze(1), sin[positions].unsqueeze(1)

        def norm(x, w):
            xf = x.float()
            return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).to(
                torch.bfloat16)

        def rope(x):
            a, b = x.float().chunk(2, dim=-1)
            return torch.cat((a * c - b * s_, b * c + a * s_), dim=-1).to(torch.bfloat16)

        for i, view in enumerate(views):
            x = qkv[i].view(tokens, HQ + 2 * HKV, D)
            q_out[i].copy_(rope(norm(x[:, :HQ], qw[i])))
            k = rope(norm(x[:, HQ:HQ + HKV], kw[i]))
            view.keys.view(-1, HKV, D).index_copy_(0, sl, k)
            view.values.view(-1, HKV, D).index_copy_(0, sl, x[:, HQ + HKV:])

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / reps / layers

    ms_fused = timed(fused)
    mi.check_device_status(device)
    ms_eager = timed(eager)
    peaks, src = _peaks()
    nbytes = prologue_bytes(tokens)
    gbs = nbytes / (ms_fused * 1e-3) / 1e9
    del pool, qkv, q_out
    return {"workload": f"Qwen3-0.6B attention prologue, {tokens} tokens (BASELINE configs[3] "
                        "prefill batch), bf16, split-half RoPE",
            "kernel": "qk_prologue_stream_kernel (RMSNorm q/k + RoPE + k/v store, one launch; "
                      "rows staged through shared memory by bulk copies)",
            "us_per_layer": round(ms_fused * 1e3, 2), "bytes_per_launch": nbytes,
            "gbs": round(gbs, 1), "hbm_frac": round(gbs / peaks["hbm_gbs"], 4),
            "peak_source": f"hbm_gbs of {src}",
            "torch_eager_us_per_layer": round(ms_eager * 1e3, 2),
            "speedup_vs_eager": round(ms_eager / ms_fused, 2)}


def measure_runner_metadata(device, reps: int = 200):
    """Per-step decode metadata: the device builder (worker/runner_metadata.py:
    changed page-table entries + one 6-int record per sequence, one copy, one
    launch) against the reference runner's host assembly restated
    (oracle/runner_oracle.StagedDecodeRows: host loop over sequences and whole
    block tables, five copies).  Each call is timed until its tensors are on the
    device (synchronize after it).  Contexts U[128, 512] as BASELINE configs[1],
    and a long-context batch (U[4K, 32K]) where whole tables are long."""
    import numpy as np
    import torch

    import microinfer_b200 as mi
    from oracle.runner_oracle import StagedDecodeRows

    class _Seq:
        def __init__(self, sid, n, table):
            self.seq_id, self.num_tokens, self.block_table = sid, n, table
            self.last_token, self.num_cached_tokens, self.num_scheduled_tokens = 1, n - 1, 1

        def __len__(self):
            return self.num_tokens

    res = {}
    for label, batch, lo, hi in (("b8_ctx128-512", 8, 128, 512), ("b64_ctx128-512", 64, 128, 512),
                                 ("b256_ctx128-512", 256, 128, 512),
                                 ("b64_ctx4k-32k", 64, 4096, 32768)):
        rng = np.random.default_rng(batch)
        grow = 2 * (reps + 3) // BS + 3  # pages each sequence gains over both timings
        nb = batch * (hi // BS + 2 + grow) + 16
        perm = rng.permutation(nb).tolist()
        seqs = []
        for i in range(batch):
            n = int(rng.integers(lo, hi))
            pages = (n + BS - 1) // BS + 1
            seqs.append(_Seq(i, n, [perm.pop() for _ in range(pages)]))
        width = max(len(s.block_table) for s in seqs) + grow
        ours = mi.DeviceRunnerMetadata(BS, nb, max_rows=batch, max_pages=width, device=device)
        base = StagedDecodeRows(BS, batch, width, device)

        def advance():
            for s in seqs:
                s.num_tokens += 1
                if (s.num_tokens - 1) // BS >= len(s.block_table):
                    s.block_table.append(perm.pop())

        def timed(fn):
            times = []
            for k in range(reps + 3):
                t0 = time.perf_counter()
                fn(seqs)
                torch.cuda.synchronize(device)
                if k >= 3:
                    times.append(time.perf_counter() - t0)
                advance()
            return statistics.median(times) * 1e6

        ours_us = timed(ours.prepare_decode)
        mi.check_device_status(device)
        base_us = timed(base.prepare_decode)
        res[label] = {"device_builder_us": round(ours_us, 1),
                      "host_assembly_us": round(base_us, 1),
                      "speedup": round(base_us / ours_us, 2)}

    # prefill metadata, BASELINE configs[3] shapes: 64 sequences, 128-token suffixes
    # on a cached 1024-token prefix (8192 tokens, block tables needed)
    from oracle.runner_oracle import staged_prefill

    class _PSeq:
        def __init__(self, sid, tokens, table):
            self.seq_id, self.token_ids, self.block_table = sid, tokens, table
            self.num_tokens = len(tokens)
            self.num_cached_tokens, self.num_scheduled_tokens = 1024, 128

        def __getitem__(self, key):
            return self.token_ids[key]

        def __len__(self):
            return self.num_tokens

    rng = np.random.default_rng(64)
    prefix_pages = list(range(64))
    pseqs = [_PSeq(i, [int(x) for x in rng.integers(0, 150000, 1152)],
                   prefix_pages + list(range(64 + 8 * i, 72 + 8 * i))) for i in range(64)]
    nb = 64 + 8 * 64
    times_o, times_b = [], []
    builder = mi.DeviceRunnerMetadata(BS, nb, max_rows=64, max_pages=72, device=device)
    for k in range(23):
        for sq in pseqs:  # new sequences each step: every table is sent whole
            builder.release(sq)
        t0 = time.perf_counter()
        builder.prepare_prefill(pseqs)
        torch.cuda.synchronize(device)
        t1 = time.perf_counter()
        staged_prefill(pseqs, BS, device)
        torch.cuda.synchronize(device)
        t2 = time.perf_counter()
        if k >= 3:
            times_o.append(t1 - t0)
            times_b.append(t2 - t1)
    mi.check_device_status(device)
    ours_us, base_us = statistics.median(times_o) * 1e6, statistics.median(times_b) * 1e6
    res["prefill_b64_q128_prefix1024"] = {"device_builder_us": round(ours_us, 1),
                                          "host_assembly_us": round(base_us, 1),
                                          "speedup": round(base_us / ours_us, 2)}
    return {"what": "metadata ready on the device, per step (median wall time incl. "
                    "synchronize); device builder vs the reference runner's host assembly "
                    "restated (decode rows: _fill_decode_rows + copies; prefill row: "
                    "prepare_prefill)", "rows": res}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps, warmup = args.steps, args.warmup
    budget = max(1.0, min(20.0, 150.0 / max(1, steps + warmup)))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    # The reference's own CPU path when its install is here, else the numpy port.
    run = reference_cpu_baseline if reference_cpu_baseline(seconds=0.0) else cpu_baseline
    for _ in range(warmup):
        run(seconds=budget / 4)
    vals = [run(seconds=budget) for _ in range(max(1, steps))]
    v = statistics.median([x["value"] for x in vals])
    base = vals[0]
    base["value"] = v
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
        "ms_per_step": statistics.median([x["ms_per_28_layer_step"] for x in vals]),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, BASELINE configs[1] shapes)",
        "config": bench_config(world),
        "cpu_baseline": base,
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if world > 1:
        line["note"] = ("one host: rank 0 alone times one GPU's shard (8 sequences) of the "
                        "workload on every host core; the other ranks exit without work")
    print(json.dumps(line), flush=True)


def run_reference_gpu(args):
    """The reference's own Triton kernels (baseline/_ref, unmodified) on this GPU.

    A second baseline next to the CPU arm: the same step as the default bench
    (slot split once, then per layer store_kv + triton_paged_decode, as the
    reference's CachedAttention runs them), captured in a CUDA graph, plus the
    configs[4] run (b) decode and the configs[2]/[3] prefill with
    triton_paged_prefill.  Prints one JSON line; "unavailable" when the
    reference is not installed.
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ref_dir = ROOT / "baseline" / "_ref"
    if not (ref_dir / "microinfer").is_dir():
        print(json.dumps({"impl": "reference-gpu", "unavailable": "baseline/_ref not installed"}))
        return
    sys.path.insert(0, str(ref_dir))
    import torch
    from microinfer.layer.triton_paged_attention import triton_paged_decode, triton_paged_prefill
    from microinfer.worker.triton_kv_store import store_kv

    from tests.golden.configs import decode_bytes, prefill_flops, store_bytes

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, src = _peaks()

    def timed(run, reps):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            run()
            run()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run()
        for _ in range(max(3, args.warmup)):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / reps

    # default workload
    ctx, table, slots = make_batch(1000, dev)
    ctx_d, table_d, slots_d = ctx.to(dev), table.to(dev), slots.to(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    kc = torch.empty(LAYERS, NB, BS, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    vc = torch.empty_like(kc).normal_(generator=g)
    q = torch.randn(LAYERS, NSEQ, HQ, D, generator=g, device=dev).to(torch.bfloat16)
    kn = torch.randn(LAYERS, NSEQ, HKV, D, generator=g, device=dev).to(torch.bfloat16)

    def step():
        sl = slots_d.long()
        blocks = torch.div(sl, BS, rounding_mode="floor")
        offs = sl - blocks * BS
        for i in range(LAYERS):
            store_kv(kc[i], vc[i], blocks, offs, kn[i], kn[i], BS)
            triton_paged_decode(q[i], kc[i], vc[i], table_d, ctx_d)

    ms = timed(step, args.steps)
    dec_b, st_b = algorithmic_bytes(ctx.tolist())
    value = LAYERS * (dec_b + st_b) / (ms * 1e-3) / 1e9
    del kc, vc
    # configs[4] run (b): batch 1 at 32768, Qwen3-8B heads, 36 layers
    layers, hq, ctx_len = 36, 32, 32768
    nb = ctx_len // BS
    kc = torch.empty(layers, nb, BS, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    vc = torch.empty_like(kc).normal_(generator=g)
    tb = torch.randperm(nb, generator=g, device=dev).to(torch.int32).view(1, nb)
    cl = torch.tensor([ctx_len], dtype=torch.int32, device=dev)
    sl1 = (tb[0, -1].long() * BS + BS - 1).view(1)
    q8 = torch.randn(layers, 1, hq, D, generator=g, device=dev).to(torch.bfloat16)
    k8 = torch.randn(layers, 1, HKV, D, generator=g, device=dev).to(torch.bfloat16)

    def long_step():
        blocks = torch.div(sl1, BS, rounding_mode="floor")
        offs = sl1 - blocks * BS
        for i in range(layers):
            store_kv(kc[i], vc[i], blocks, offs, k8[i], k8[i], BS)
            triton_paged_decode(q8[i], kc[i], vc[i], tb, cl)

    ms_long = timed(long_step, 5)
    long_b = layers * (decode_bytes([ctx_len], hq, HKV, D, 2, BS) + store_bytes(1, HKV, D, 2))
    del kc, vc
    extra = {"long_context_b1": {"ms_per_step": round(ms_long, 4),
                                 "value": round(long_b / (ms_long * 1e-3) / 1e9, 1), "unit": "GB/s"}}
    for workload in ("mixed", "prefix"):
        b = _prefill_batch(workload, dev, None)
        kc = torch.empty(LAYERS, b["nb"], BS, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        vc = torch.empty_like(kc).normal_(generator=g)
        tokens = int(sum(b["q_lens"]))
        qp = torch.randn(tokens, HQ, D, generator=g, device=dev).to(torch.bfloat16)
        kp = torch.randn(tokens, HKV, D, generator=g, device=dev).to(torch.bfloat16)

        def prefill_step():
            sl = b["slots"].long()
            blocks = torch.div(sl, BS, rounding_mode="floor")
            offs = sl - blocks * BS
            for i in range(LAYERS):
                store_kv(kc[i], vc[i], blocks, offs, kp, kp, BS)
                triton_paged_prefill(qp, kc[i], vc[i], b["cu_q"], b["cu_k"], b["table"],
                                     max_seqlen_q=max(b["q_lens"]))

        ms_p = timed(prefill_step, 3)
        flops = prefill_flops(b["q_lens"], b["contexts"], HQ, D)
        tf = flops / (ms_p / LAYERS * 1e-3) / 1e12
        extra[f"prefill_{'mixed' if workload == 'mixed' else 'shared_prefix'}"] = {
            "us_per_layer": round(ms_p / LAYERS * 1e3, 2), "tflops": round(tf, 1),
            "tensor_frac": round(tf / peaks["bf16_tflops"], 4)}
        del kc, vc
    print(json.dumps({
        "impl": "reference-gpu", "metric": METRIC, "value": round(value, 2), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(ms, 5), "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (seeded torch, BASELINE configs[1] shapes)",
        "config": {"workload": WORKLOAD, "kernels": "reference Triton store_kv + triton_paged_decode "
                   "(baseline/_ref, unmodified), CUDA graph"},
        "frac": round(value / peaks["hbm_gbs"], 4), "peak_source": f"hbm_gbs of {src}",
        "extra": extra}), flush=True)


_CUDART = None


def _copy_async(dst, src, stream):
    """cudaMemcpyAsync of one whole contiguous tensor on `stream`.

    Raw runtime call (the libcudart torch has loaded), so that a copy from pinned host
    memory can be captured in a CUDA graph without torch's host-allocator bookkeeping.
    Direction from the pointers (cudaMemcpyDefault)."""
    global _CUDART
    if _CUDART is None:
        import ctypes
        lib = ctypes.CDLL("libcudart.so.12")
        lib.cudaMemcpyAsync.restype = ctypes.c_int
        lib.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                        ctypes.c_int, ctypes.c_void_p]
        _CUDART = lib
    nbytes = src.numel() * src.element_size()
    if not (dst.is_contiguous() and src.is_contiguous()) or dst.numel() * dst.element_size() != nbytes:
        raise RuntimeError("_copy_async: tensors must be contiguous and of equal byte size")
    rc = _CUDART.cudaMemcpyAsync(dst.data_ptr(), src.data_ptr(), nbytes, 4, stream.cuda_stream)
    if rc != 0:
        raise RuntimeError(f"cudaMemcpyAsync returned {rc}")


def _e2e_whole_step_graph(device, cur, in_ends, out_ends, attention_layers, sample, meta_d,
                          h_meta, pk_d, h_pk, out, h_out, tokens, tok_all, h_tok, steps):
    """End-to-end decode step captured whole (1 GPU): ms per step by CUDA events.

    One graph launch per step holds the step's input copies from pinned host memory, the 28
    store+decode launches, the sampler and the read-back of every layer's output and of the
    token ids.  Inputs go in as runs of consecutive layers ending at `in_ends`, outputs come
    back as runs ending at `out_ends`: a layer starts once its input run is on the device, an
    output run goes back while later layers compute, and the next replay (the next step)
    starts only once this step's results are on the host.  Only the first input run and the
    last output run are not hidden behind compute.  The read-back is checked against the
    device results before timing."""
    import torch

    cuts = sorted(set(in_ends) | set(out_ends))
    assert cuts[-1] == LAYERS and in_ends[-1] == LAYERS and out_ends[-1] == LAYERS
    h2d_s, d2h_s = torch.cuda.Stream(device), torch.cuda.Stream(device)
    # the step's metadata and the token read-back each get a copy stream of their own,
    # so they run beside the first input run and the last output run, not after them
    meta_s, tok_s = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = {e: torch.cuda.Event() for e in in_ends}
    ev_done = {e: torch.cuda.Event() for e in out_ends}
    ev_meta, ev_tok = torch.cuda.Event(), torch.cuda.Event()
    sg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(sg):
        cs = torch.cuda.current_stream(device)
        h2d_s.wait_stream(cs)
        meta_s.wait_stream(cs)
        _copy_async(meta_d, h_meta, meta_s)
        ev_meta.record(meta_s)
        lo = 0
        for e in in_ends:
            _copy_async(pk_d[lo:e], h_pk[lo:e], h2d_s)
            ev_in[e].record(h2d_s)
            lo = e
        cs.wait_event(ev_meta)
        lo, out_lo = 0, 0
        for hi in cuts:
            starts = [e for e in in_ends if e > lo]
            if lo == 0 or lo in in_ends:  # first layer of an input run
                cs.wait_event(ev_in[starts[0]])
            attention_layers(range(lo, hi))
            if hi == LAYERS:
                sample()  # one GPU: the gathered token ids are this GPU's own
                ev_tok.record(cs)
                tok_s.wait_event(ev_tok)
                _copy_async(h_tok, tokens, tok_s)
            if hi in out_ends:
                ev_done[hi].record(cs)
                d2h_s.wait_event(ev_done[hi])
                _copy_async(h_out[out_lo:hi], out[out_lo:hi], d2h_s)
                out_lo = hi
            lo = hi
        cs.wait_stream(d2h_s)
        cs.wait_stream(tok_s)
    for _ in range(3):
        sg.replay()
    torch.cuda.synchronize(device)
    if not (torch.equal(h_out, out.cpu()) and torch.equal(h_tok, tokens.cpu())):
        raise RuntimeError("whole-step graph read-back differs from the device results")
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(cur)
    for _ in range(steps):
        sg.replay()
    x1.record(cur)
    torch.cuda.synchronize(device)
    del sg
    return x0.elapsed_time(x1) / steps


def run_ours(args):
    import torch
    import torch.distributed as dist

    import microinfer_b200 as mi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    # --- per-rank shard: own pool, own 8 sequences -------------------------
    ctx, table, slots = make_batch(1000 + rank, device)
    # The step's int32 inputs (lengths, tables, slots) share one device buffer so the
    # end-to-end path moves them in one copy.
    meta_d = torch.empty(ctx.numel() + table.numel() + slots.numel(), dtype=torch.int32,
                         device=device)
    ctx_d = meta_d[: ctx.numel()]
    table_d = meta_d[ctx.numel(): ctx.numel() + table.numel()].view(table.shape)
    slots_d = meta_d[ctx.numel() + table.numel():]
    ctx_d.copy_(ctx)
    table_d.copy_(table)
    slots_d.copy_(slots)
    pool = mi.KVCache(LAYERS, NB, BS, HKV, D, dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device).manual_seed(rank)
    pool.keys.normal_(generator=g).mul_(0.5)
    pool.values.normal_(generator=g).mul_(0.5)
    q_all = torch.randn(LAYERS, NSEQ, HQ, D, generator=g, device=device).to(torch.bfloat16)
    kn_all = torch.randn(LAYERS, NSEQ, HKV, D, generator=g, device=device).to(torch.bfloat16)
    vn_all = torch.randn(LAYERS, NSEQ, HKV, D, generator=g, device=device).to(torch.bfloat16)
    # Per-layer inputs packed [q | k_new | v_new] layer after layer, so the end-to-end path
    # moves any run of consecutive layers (a group, or one layer) in one copy.
    qn, kvn = NSEQ * HQ * D, NSEQ * HKV * D
    pk_d = torch.empty(LAYERS, qn + 2 * kvn, dtype=torch.bfloat16, device=device)
    pk_d[:, :qn].copy_(q_all.reshape(LAYERS, -1))
    pk_d[:, qn:qn + kvn].copy_(kn_all.reshape(LAYERS, -1))
    pk_d[:, qn + kvn:].copy_(vn_all.reshape(LAYERS, -1))
    q = list(pk_d[:, :qn].unflatten(1, (NSEQ, HQ, D)).unbind(0))
    kn = list(pk_d[:, qn:qn + kvn].unflatten(1, (NSEQ, HKV, D)).unbind(0))
    vn = list(pk_d[:, qn + kvn:].unflatten(1, (NSEQ, HKV, D)).unbind(0))
    del q_all, kn_all, vn_all
    out = torch.empty(LAYERS, NSEQ, HQ, D, dtype=torch.bfloat16, device=device)
    # Sampled token ids in a ring of n_slots buffers: step k writes buffer
    # k % n_slots while the all_gathers of the steps before it (off the attention
    # path, on their own stream) read the others.
    n_slots = TOKEN_SLOTS if world > 1 else 2
    tokens_buf = torch.empty(n_slots, NSEQ, dtype=torch.int32, device=device)
    tokens = tokens_buf[0]
    decode_kernel, split, _ = mi.decode_plan(NSEQ, HQ, HKV, D, torch.bfloat16, BS, 0, device,
                                             table_d.shape[1])
    views = [pool.layer(i) for i in range(LAYERS)]

    def attention_layers(layers=range(LAYERS)):
        # store_kvcache fused into paged decode: one launch per layer
        for i in layers:
            view = views[i]
            # Layer i+1's launch only follows layer i's decode, which writes neither
            # layer i+1's pool nor the tables: its pages may load early (PDL).
            mi.paged_decode_store(q[i], view.keys, view.values, table_d, ctx_d, kn[i], vn[i],
                                  slots_d, split_k=None, out=out[i], early_kv=True)

    def sample(slot=0):
        # stand-in sampler: one int32 token id per sequence from the last layer
        tokens_buf[slot].copy_(out[-1, :, 0, :].float().argmax(-1))

    def layer_loop(slot=0):
        attention_layers()
        sample(slot)

    decode_only = attention_layers

    # warm up + capture
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for _ in range(2):
            layer_loop()
            decode_only()
    torch.cuda.current_stream(device).wait_stream(stream)
    torch.cuda.synchronize(device)
    cur = torch.cuda.current_stream(device)
    gathered = torch.empty(n_slots, world * NSEQ, dtype=torch.int32, device=device)
    ag_stream = torch.cuda.Stream(device)
    if world > 1:  # communicators exist before any capture
        dist.all_gather_into_tensor(gathered[0], tokens_buf[0])
        torch.cuda.synchronize(device)
    # One CUDA graph per token slot: graph `slot` runs the 28 layers and the sampler into
    # tokens_buf[slot].  With N > 1 the NCCL all_gather of those token ids (for the
    # scheduler; the attention never waits on it) is a second captured graph, replayed on
    # its own stream once the step's graph is done, so it overlaps the next steps' layers;
    # step k + n_slots reuses the slot only after that gather.
    # The host issues two graph launches and three event operations per step.  (Measured
    # at N = 2: 0.1604 ms per step this way, 0.1648 with the gather as a side branch inside
    # the step's graph, 0.1734 with it at the end of the graph, 0.1592 with no gather.)
    graphs, ag_graphs = [], []
    for slot in range(n_slots):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            layer_loop(slot)
        graphs.append(gr)
        if world > 1:
            ag_cap = torch.cuda.Stream(device)
            with torch.cuda.stream(ag_cap):
                agr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(agr, stream=ag_cap):
                    dist.all_gather_into_tensor(gathered[slot], tokens_buf[slot])
            ag_graphs.append(agr)
            del agr
        del gr
    dgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(dgraph):
        decode_only()
    ag_ready = [torch.cuda.Event() for _ in range(n_slots)]
    ag_done = [torch.cuda.Event() for _ in range(n_slots)]

    def step(k):
        slot = k % n_slots
        if world > 1:
            cur.wait_event(ag_done[slot])
        graphs[slot].replay()
        if world > 1:
            ag_ready[slot].record(cur)
            ag_stream.wait_event(ag_ready[slot])
            with torch.cuda.stream(ag_stream):
                ag_graphs[slot].replay()
            ag_done[slot].record(ag_stream)

    def last_gather(k_last):
        if world > 1:
            cur.wait_stream(ag_stream)

    warm = max(3, args.warmup, n_slots)  # every slot's graphs replayed before timing
    for k in range(warm):
        step(k)
    last_gather(warm - 1)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()

    # --- timed region: exactly K steps ---------------------------------------
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_all0, t_all1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index if device.index is not None else 0) as clocks:
        torch.cuda.synchronize(device)
        t_all0.record(cur)
        for k in range(args.steps):
            starts[k].record(cur)
            step(k)
            ends[k].record(cur)
        last_gather(args.steps - 1)  # the last step's gather ends inside the timed region
        t_all1.record(cur)
        torch.cuda.synchronize(device)
        # keep sampling clocks over ~1 s of the decode layers (not timed; no collective,
        # so the ranks need not replay it equally often)
        if len(clocks.samples) < 20:
            t_end = time.time() + 1.0
            while time.time() < t_end:
                for _ in range(50):
                    dgraph.replay()
                torch.cuda.synchronize(device)
    total_ms = t_all0.elapsed_time(t_all1)
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    # device idle time between consecutive steps (host issue gaps)
    gaps = [ends[k].elapsed_time(starts[k + 1]) for k in range(args.steps - 1)]
    ms_step = total_ms / args.steps
    gap_stats = [statistics.median(gaps) * 1e3 if gaps else 0.0, max(gaps) * 1e3 if gaps else 0.0]
    ordered = sorted(per_step)
    step_dist = [ordered[len(ordered) // 2], ordered[(9 * len(ordered)) // 10], ordered[-1]]
    if world > 1:
        t = torch.tensor([ms_step, gap_stats[0], gap_stats[1], *step_dist], device=device)
        every = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(every, t)
        ms_step = max(float(x[0]) for x in every)
        gap_stats = [max(float(x[1]) for x in every), max(float(x[2]) for x in every)]
        step_dist = [max(float(x[3 + i]) for x in every) for i in range(3)]
        rank_ms = [round(float(x[0]), 5) for x in every]
    else:
        rank_ms = [round(ms_step, 5)]

    dec_b, st_b = algorithmic_bytes(ctx.tolist())
    step_bytes = LAYERS * (dec_b + st_b)
    value = world * step_bytes / (ms_step * 1e-3) / 1e9

    # --- dominant kernel: decode-only graph over the 28 distinct layer pools --
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dgraph.replay()
    torch.cuda.synchronize(device)
    e0.record(cur)
    for _ in range(reps):
        dgraph.replay()
    e1.record(cur)
    torch.cuda.synchronize(device)
    decode_launch_ms = e0.elapsed_time(e1) / (reps * LAYERS)
    peaks, peak_src = _peaks()
    achieved = (dec_b + st_b) / (decode_launch_ms * 1e-3) / 1e9

    # --- the same launches isolated, as the model runs them: each layer's decode follows
    # a GEMM (the 1024 x 4096 x 3072 bf16 product standing in for a layer's projections)
    # that occupies every SM, so no page load starts early.  Per-layer decode cost =
    # (graph of 28 x [GEMM, decode]) - (graph of 28 x [GEMM]), both by CUDA events.
    ga = torch.randn(1024, 4096, device=device, dtype=torch.bfloat16)
    gb = torch.randn(4096, 3072, device=device, dtype=torch.bfloat16)
    gc = torch.empty(1024, 3072, device=device, dtype=torch.bfloat16)

    def gemm_layers(with_decode):
        for i in range(LAYERS):
            torch.mm(ga, gb, out=gc)
            if with_decode:
                view = views[i]
                mi.paged_decode_store(q[i], view.keys, view.values, table_d, ctx_d, kn[i], vn[i],
                                      slots_d, split_k=None, out=out[i], early_kv=True)

    gemm_layers(True)
    torch.cuda.synchronize(device)
    iso_both = _graph_ms(device, lambda: gemm_layers(True), 20, warm=3)
    iso_gemm = _graph_ms(device, lambda: gemm_layers(False), 20, warm=3)
    iso_avg_us = (iso_both - iso_gemm) / LAYERS * 1e3
    iso_gbs = (dec_b + st_b) / (iso_avg_us * 1e-6) / 1e9
    del ga, gb, gc

    # --- e2e: host buffers through the public API ----------------------------
    # Every step copies its inputs in from pinned host memory and its results (the
    # attention outputs of all layers and the gathered token ids) back, inside the
    # timed region.  Each group of E2E_GROUP layers has one packed input buffer, copied
    # on a side stream while the previous group computes; a group's outputs go back on
    # a third stream as soon as it finishes.
    groups = LAYERS // E2E_GROUP
    h_pk = pk_d.cpu().pin_memory()
    h_meta = meta_d.cpu().pin_memory()
    h_out = torch.empty_like(out, device="cpu").pin_memory()
    tok_all = torch.empty(world * NSEQ, dtype=torch.int32, device=device)
    h_tok = torch.empty(world * NSEQ, dtype=torch.int32).pin_memory()
    h2d = h_pk.numel() * h_pk.element_size() + h_meta.numel() * h_meta.element_size()
    d2h = h_out.numel() * h_out.element_size() + h_tok.numel() * h_tok.element_size()
    gstream = torch.cuda.Stream(device)
    gstream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(gstream):
        for gi in range(groups):
            attention_layers(range(gi * E2E_GROUP, (gi + 1) * E2E_GROUP))
        sample()
    torch.cuda.current_stream(device).wait_stream(gstream)
    torch.cuda.synchronize(device)
    ggraphs = []
    for gi in range(groups):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            attention_layers(range(gi * E2E_GROUP, (gi + 1) * E2E_GROUP))
            if gi == groups - 1:
                sample()
        ggraphs.append(gr)
    h2d_stream, d2h_stream = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(groups)]
    ev_done = [torch.cuda.Event() for _ in range(groups)]

    def e2e_step():
        h2d_stream.wait_stream(cur)  # the previous step no longer reads the inputs
        with torch.cuda.stream(h2d_stream):
            meta_d.copy_(h_meta, non_blocking=True)
            for gi in range(groups):
                lo, hi = gi * E2E_GROUP, (gi + 1) * E2E_GROUP
                pk_d[lo:hi].copy_(h_pk[lo:hi], non_blocking=True)
                ev_in[gi].record(h2d_stream)
        for gi in range(groups):
            cur.wait_event(ev_in[gi])
            ggraphs[gi].replay()
            ev_done[gi].record(cur)
            d2h_stream.wait_event(ev_done[gi])
            with torch.cuda.stream(d2h_stream):
                lo, hi = gi * E2E_GROUP, (gi + 1) * E2E_GROUP
                h_out[lo:hi].copy_(out[lo:hi], non_blocking=True)
        if world > 1:
            dist.all_gather_into_tensor(tok_all, tokens)
        else:
            tok_all.copy_(tokens)
        d2h_stream.wait_stream(cur)
        with torch.cuda.stream(d2h_stream):
            h_tok.copy_(tok_all, non_blocking=True)
        cur.wait_stream(d2h_stream)  # the step ends with its results on the host

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record(cur)
    for _ in range(args.steps):
        e2e_step()
    x1.record(cur)
    torch.cuda.synchronize(device)
    e2e_ms = x0.elapsed_time(x1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * step_bytes / (e2e_ms * 1e-3) / 1e9
    mi.check_device_status(device)
    e2e_eager_ms = e2e_ms
    e2e_graph_note = None
    e2e_graph_ms = None
    if world == 1:
        try:
            e2e_graph_ms = _e2e_whole_step_graph(
                device, cur, E2E_IN_ENDS, E2E_OUT_ENDS, attention_layers, sample, meta_d, h_meta,
                pk_d, h_pk, out, h_out, tokens, tok_all, h_tok, args.steps)
        except (RuntimeError, OSError) as exc:  # capture refused: keep the eager number
            e2e_graph_note = f"whole-step graph not used: {str(exc).splitlines()[0][:160]}"
        if e2e_graph_ms is not None and e2e_graph_ms < e2e_ms:
            e2e_ms = e2e_graph_ms
            e2e_value = world * step_bytes / (e2e_ms * 1e-3) / 1e9
            e2e_graph_note = "graph"
        mi.check_device_status(device)

    # one launch per layer (store and split merge are inside the decode kernel)
    launches_per_step = LAYERS
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": warm, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded torch, BASELINE configs[1] shapes), random-init pool",
            "config": bench_config(world),
            "plan": {"split_k": split, "decode_kernel": decode_kernel,
                     "bytes_per_step_per_gpu": step_bytes,
                     "graph": "one CUDA graph per step: 28 store+decode launches and the "
                              "sampler; with N > 1 the step's token all_gather is a second "
                              "captured graph replayed on a side stream after it, overlapping "
                              "the next step's layers"},
            "tok_per_s": round(world * NSEQ / (ms_step * 1e-3), 1),
            "median_step_ms": round(statistics.median(per_step), 5),
            "rank_ms_per_step": rank_ms,
            "step_ms": {"median": round(step_dist[0], 5), "p90": round(step_dist[1], 5),
                        "max": round(step_dist[2], 5),
                        "what": "device time of single steps (a step's event pair), max over ranks"},
            "step_gap_us": {"median": round(gap_stats[0], 2), "max": round(gap_stats[1], 2),
                            "what": "device idle time between one step's end and the next "
                                    "step's start, max over ranks"},
            "roofline": {"bound": "hbm",
                         "kernel": DECODE_KERNEL_NAMES.get(decode_kernel, decode_kernel)
                                   + " (store fused, split merge)",
                         "achieved": round(achieved, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_source": f"hbm_gbs of {peak_src}",
                         "avg_launch_us": round(decode_launch_ms * 1e3, 3),
                         "algorithmic_bytes_per_launch": dec_b + st_b,
                         "traffic": _profiled_traffic(DECODE_PROFILES.get(decode_kernel, "")),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                           "profiles/ summary of the same kernel and shapes",
                         "step_frac": round(value / world / peaks["hbm_gbs"], 4),
                         "timing": "average launch in a 28-layer decode-only graph replay "
                                   "(back to back: a layer's page loads may start under the "
                                   "previous layer's tail)",
                         "isolated": {"avg_launch_us": round(iso_avg_us, 3),
                                      "achieved": round(iso_gbs, 1),
                                      "frac": round(iso_gbs / peaks["hbm_gbs"], 4),
                                      "what": "per-layer decode cost behind a GEMM that fills "
                                              "every SM (28 x [GEMM, decode] graph minus 28 x "
                                              "[GEMM] graph); no early start"}},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 5),
                    "path": ("pinned host inputs -> microinfer_b200 API (C ABI) -> host outputs; "
                             f"inputs copied per group of {E2E_GROUP} layers on a side stream while "
                             "the previous group computes, outputs copied back per group"
                             if e2e_graph_note != "graph" else
                             "pinned host inputs -> microinfer_b200 API (C ABI) -> host outputs; "
                             "the whole step (copies, 28 layers, sampler, read-back) is one CUDA "
                             f"graph launch; inputs in as runs of layers ending at {E2E_IN_ENDS}, "
                             f"outputs back as runs ending at {E2E_OUT_ENDS}, while other layers "
                             "compute"),
                    "eager_ms_per_step": round(e2e_eager_ms, 5),
                    "graph_ms_per_step": (None if e2e_graph_ms is None
                                          else round(e2e_graph_ms, 5)),
                    **({"note": e2e_graph_note}
                       if e2e_graph_note not in (None, "graph") else {})},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
        }
    torch.cuda.synchronize(device)
    del graphs, ag_graphs, dgraph  # graphs holding NCCL calls go before the process group
    del pool, pk_d, out
    torch.cuda.empty_cache()
    # configs[4] run (a), sequence-sharded over every rank (each rank times its shard)
    extra = {"long_context_batch256": measure_long_batch(device, world, rank)}
    if rank == 0:
        if world == 1:
            extra.update({"long_context_b1": measure_long_b1(device),
                          "prefill_mixed": measure_prefill(device, "mixed"),
                          "prefill_shared_prefix": measure_prefill(device, "prefix"),
                          "shared_prefix_step": measure_shared_prefix_step(device),
                          "store_kv": measure_store(device),
                          "direct_prefill": measure_varlen(device),
                          "attention_prologue": measure_prologue(device),
                          "runner_metadata": measure_runner_metadata(device)})
        line["extra"] = extra
        if world == 1 and not args.no_cpu_baseline:
            ref_cpu = reference_cpu_baseline()
            line["cpu_baseline"] = ref_cpu if ref_cpu is not None else cpu_baseline()
            if ref_cpu is not None:
                line["cpu_baseline_port"] = cpu_baseline(seconds=6.0)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_profile(args):
    """Small fixed case for ncu: config-2 shapes on 4 layer pools (256 MB > L2).

    Eager launches (no graph), `--steps` iterations of store + decode per
    layer, so an ncu capture with -k/-s/-c stays small and ends by itself.
    """
    import torch

    import microinfer_b200 as mi

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    if args.profile == "long":
        # BASELINE configs[4] run (b) shape on 4 layer pools (4 x 134 MB > L2)
        layers, hq, hkv, ctx_len = 4, 32, 8, 32768
        nb = ctx_len // BS
        pool = mi.KVCache(layers, nb, BS, hkv, D, dtype=torch.bfloat16, device=device)
        g = torch.Generator(device=device).manual_seed(5)
        pool.keys.normal_(generator=g).mul_(0.5)
        pool.values.normal_(generator=g).mul_(0.5)
        table = torch.randperm(nb, generator=g, device=device).to(torch.int32).view(1, nb)
        ctx = torch.tensor([ctx_len], dtype=torch.int32, device=device)
        slots = (table[0, -1].long() * BS + BS - 1).to(torch.int32).view(1)
        q = torch.randn(layers, 1, hq, D, generator=g, device=device).to(torch.bfloat16)
        kn = torch.randn(layers, 1, hkv, D, generator=g, device=device).to(torch.bfloat16)
        kernel, split, _ = mi.decode_plan(1, hq, hkv, D, torch.bfloat16, BS, args.split_k, device,
                                          nb)
        for _ in range(args.steps):
            for i in range(layers):
                view = pool.layer(i)
                mi.paged_decode_store(q[i], view.keys, view.values, table, ctx, kn[i], kn[i],
                                      slots, split_k=args.split_k or None, early_kv=True)
        torch.cuda.synchronize(device)
        mi.check_device_status(device)
        from tests.golden.configs import decode_bytes

        print(json.dumps({"profile": "long", "kernel": kernel, "split_k": split,
                          "decode_bytes_per_launch": decode_bytes([ctx_len], hq, hkv, D, 2, BS)}))
        return
    if args.profile == "metadata":
        # decode metadata for 256 sequences (contexts U[128, 512]) over `--steps` steps
        import numpy as np

        class _Seq:
            def __init__(self, sid, n, table):
                self.seq_id, self.num_tokens, self.block_table = sid, n, table
                self.last_token, self.num_cached_tokens, self.num_scheduled_tokens = 1, n - 1, 1

        rng = np.random.default_rng(256)
        nb = 256 * 40
        perm = rng.permutation(nb).tolist()
        seqs = []
        for i in range(256):
            n = int(rng.integers(128, 512))
            seqs.append(_Seq(i, n, [perm.pop() for _ in range((n + BS - 1) // BS + 1)]))
        meta = mi.DeviceRunnerMetadata(BS, nb, max_rows=256, max_pages=40, device=device)
        for _ in range(args.steps):
            meta.prepare_decode(seqs)
            for s_ in seqs:
                s_.num_tokens += 1
                if (s_.num_tokens - 1) // BS >= len(s_.block_table):
                    s_.block_table.append(perm.pop())
        torch.cuda.synchronize(device)
        mi.check_device_status(device)
        print(json.dumps({"profile": "metadata", "sequences": 256, "steps": args.steps}))
        return
    if args.profile == "prologue":
        g = torch.Generator(device=device).manual_seed(21)
        layers, tokens = 2, 8192
        pool, qkv, qw, kw, cos, sin, positions, slots = _prologue_inputs(device, layers, tokens,
                                                                         g)
        for _ in range(args.steps):
            for i in range(layers):
                view = pool.layer(i)
                mi.qk_norm_rope_store(qkv[i], qw[i], kw[i], positions, cos, sin, view.keys,
                                      view.values, slots, num_q_heads=HQ, num_kv_heads=HKV,
                                      eps=1e-6)
        torch.cuda.synchronize(device)
        mi.check_device_status(device)
        print(json.dumps({"profile": "prologue", "layers": layers, "iterations": args.steps,
                          "bytes_per_launch": prologue_bytes(tokens)}))
        return
    if args.profile in ("store", "gather", "cow", "varlen"):
        # configs[3] shapes on 2 layer pools: store of the 8192 suffix tokens, gather of the
        # 64 x 1152-row contexts, copy-on-write of 64 pages (every layer of a 28-layer pool),
        # direct prefill of 8 x 512 + 24 short sequences
        from tests.golden.configs import cow_bytes, gather_bytes, prefill_flops, store_bytes

        g = torch.Generator(device=device).manual_seed(41)
        b = _prefill_batch("prefix", device)
        layers = 28 if args.profile == "cow" else 2
        pool = mi.KVCache(layers, b["nb"], BS, HKV, D, dtype=torch.bfloat16, device=device)
        pool.keys.normal_(generator=g)
        pool.values.normal_(generator=g)
        kn = torch.randn(b["tokens"], HKV, D, generator=g, device=device).to(torch.bfloat16)
        info = {"profile": args.profile, "iterations": args.steps}
        if args.profile == "store":
            for _ in range(args.steps):
                for i in range(layers):
                    pool.layer(i).write_slots(b["slots"], kn, kn)
            info["bytes_per_launch"] = store_bytes(b["tokens"], HKV, D, 2)
        elif args.profile == "gather":
            total = sum(b["contexts"])
            gk = torch.empty(total, HKV, D, dtype=torch.bfloat16, device=device)
            gv = torch.empty_like(gk)
            for _ in range(args.steps):
                for i in range(layers):
                    v = pool.layer(i)
                    mi.gather_paged_kv(v.keys, v.values, b["table"], b["contexts"], BS,
                                       cu_seqlens_k=b["cu_k"], out=(gk, gv))
            info["bytes_per_launch"] = gather_bytes(b["contexts"], HKV, D, 2)
        elif args.profile == "cow":
            # the 64 shared prefix pages -> the last 64 pages of the pool
            pairs = torch.stack([torch.arange(64), torch.arange(b["nb"] - 64, b["nb"])],
                                dim=1).to(torch.int32)
            for _ in range(args.steps):
                pool.copy_blocks(pairs.to(device), check=False)
            info["bytes_per_launch"] = cow_bytes(64, layers, BS, HKV, D, 2)
        else:
            gen = torch.Generator().manual_seed(16)
            lens = [512] * 8 + torch.randint(1, 65, (24,), generator=gen).tolist()
            total = sum(lens)
            q = torch.randn(total, HQ, D, generator=g, device=device).to(torch.bfloat16)
            k = torch.randn(layers, total, HKV, D, generator=g, device=device).to(torch.bfloat16)
            cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
            cu[1:] = torch.cumsum(torch.tensor(lens), 0)
            cu = cu.to(device)
            for _ in range(args.steps):
                for i in range(layers):
                    mi.varlen_prefill(q, k[i], k[i], cu, cu, max_seqlen_q=512)
            info["flops_per_launch"] = prefill_flops(lens, lens, HQ, D)
        torch.cuda.synchronize(device)
        mi.check_device_status(device)
        print(json.dumps(info))
        return
    if args.profile in ("prefill", "mixed"):
        workload = "prefix" if args.profile == "prefill" else "mixed"
        g = torch.Generator(device=device).manual_seed(11)
        b = _prefill_batch(workload, device, g)
        layers = 2
        pool = mi.KVCache(layers, b["nb"], BS, HKV, D, dtype=torch.bfloat16, device=device)
        pool.keys.normal_(generator=g).mul_(0.5)
        pool.values.normal_(generator=g).mul_(0.5)
        tokens = int(sum(b["q_lens"]))
        q = torch.randn(tokens, HQ, D, generator=g, device=device).to(torch.bfloat16)
        for _ in range(args.steps):
            for i in range(layers):
                view = pool.layer(i)
                mi.paged_prefill(q, view.keys, view.values, b["cu_q"], b["cu_k"], b["table"],
                                 max_seqlen_q=max(b["q_lens"]))
        torch.cuda.synchronize(device)
        mi.check_device_status(device)
        from tests.golden.configs import prefill_flops

        print(json.dumps({"profile": args.profile, "layers": layers, "iterations": args.steps,
                          "flops_per_launch": prefill_flops(b["q_lens"], b["contexts"], HQ, D)}))
        return
    layers = 4
    ctx, table, slots = make_batch(1000, device)
    ctx_d, table_d, slots_d = ctx.to(device), table.to(device), slots.to(device)
    pool = mi.KVCache(layers, NB, BS, HKV, D, dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device).manual_seed(0)
    pool.keys.normal_(generator=g).mul_(0.5)
    pool.values.normal_(generator=g).mul_(0.5)
    q = torch.randn(layers, NSEQ, HQ, D, generator=g, device=device).to(torch.bfloat16)
    kn = torch.randn(layers, NSEQ, HKV, D, generator=g, device=device).to(torch.bfloat16)
    _, split, _ = mi.decode_plan(NSEQ, HQ, HKV, D, torch.bfloat16, BS, args.split_k, device,
                                 table_d.shape[1])
    for _ in range(args.steps):
        for i in range(layers):
            view = pool.layer(i)
            mi.paged_decode_store(q[i], view.keys, view.values, table_d, ctx_d, kn[i], kn[i],
                                  slots_d, split_k=args.split_k or None)
    torch.cuda.synchronize(device)
    mi.check_device_status(device)
    dec_b, _ = algorithmic_bytes(ctx.tolist())
    print(json.dumps({"profile": args.profile, "layers": layers, "iterations": args.steps,
                      "split_k": split, "decode_bytes_per_launch": dec_b}))


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-gpu"], default="ours",
                    help="reference = the reference's CPU path (oracle port); reference-gpu = "
                         "its Triton kernels on this GPU (needs baseline/_ref)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", choices=["decode", "long", "prefill", "mixed", "prologue", "metadata",
                                          "store", "gather", "cow", "varlen"], default=None,
                    help="run a small eager case for ncu instead of the benchmark")
    ap.add_argument("--split-k", type=int, default=0)
    args = ap.parse_args()
    if args.profile:
        run_profile(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference-gpu":
        run_reference_gpu(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
