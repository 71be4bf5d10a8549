"""Generate the golden fixtures from the reference implementation itself.

Run in a container where the reference MicroInfer source tree is available
(pass its path, default ``$MICROINFER_REFERENCE``):

    python tests/golden/make_golden.py /path/to/MicroInfer

For every case in ``cases.CASES`` it rebuilds the seeded inputs, runs the
reference's own CPU functions on them and writes ``<case>.npz`` with:

* the reference outputs (raw element bits for bf16),
* SHA-256 digests of every input (so a test can prove it regenerated the
  exact same bytes), and of bulky bit-exact outputs (the gathered K/V).

Reference functions used (paths inside the reference project):
  LayerKVCache.write_checked      microinfer/worker/kv_cache.py:30-50
  _paged_attention_reference      microinfer/layer/paged_attention.py:22-67
  _gather_paged_kv                microinfer/layer/paged_attention.py:76-101
  _direct_prefill_sdpa            microinfer/layer/cached_attention.py:47-55
The copy-on-write fixture uses the torch restatement ``pool[:, dst] = pool[:, src]``
(the reference has no copy-on-write).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden import cases  # noqa: E402

TORCH_DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def to_torch(a: np.ndarray, dtype: str | None = None) -> torch.Tensor:
    if dtype == "bf16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a))


def to_numpy(t: torch.Tensor, dtype: str) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if dtype == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from microinfer.layer.cached_attention import _direct_prefill_sdpa
    from microinfer.layer.paged_attention import _gather_paged_kv, _paged_attention_reference
    from microinfer.worker.kv_cache import LayerKVCache

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    force = "--force" in sys.argv
    for name in cases.CASES:
        if (HERE / f"{name}.npz").exists() and not force:
            continue  # fixtures are deterministic; keep committed bytes unchanged
        case = cases.build(name)
        dt = case["dtype"]
        out = {"digest_" + k: np.array(cases.digest(case[k])) for k in cases.INPUT_KEYS if k in case}
        kind = case["kind"]
        if kind in ("decode", "prefill"):
            layer = LayerKVCache(to_torch(case["key_cache"], dt).clone(),
                                 to_torch(case["value_cache"], dt).clone())
            layer.write_checked(torch.from_numpy(case["slots"].astype(np.int64)),
                                to_torch(case["k_new"], dt), to_torch(case["v_new"], dt))
            contexts = [int(c) for c in case["contexts"]]
            if kind == "decode":
                cu_q = list(range(len(contexts) + 1))
            else:
                cu_q = [int(x) for x in case["cu_seqlens_q"]]
            table = torch.from_numpy(case["block_tables"].astype(np.int64))
            result = _paged_attention_reference(
                to_torch(case["query"], dt), layer.keys, layer.values, table, contexts, cu_q,
                scale=case["scale"])
            out["out"] = to_numpy(result, dt)
            slots = case["slots"].astype(np.int64)
            bs = case["block_size"]
            # stored rows are bit-exact: their digests pin them
            out["stored_k_digest"] = np.array(cases.digest(to_numpy(layer.keys[slots // bs, slots % bs], dt)))
            out["stored_v_digest"] = np.array(cases.digest(to_numpy(layer.values[slots // bs, slots % bs], dt)))
            gk, gv = _gather_paged_kv(layer.keys, layer.values, table, contexts, bs)
            out["gather_k_digest"] = np.array(cases.digest(to_numpy(gk, dt)))
            out["gather_v_digest"] = np.array(cases.digest(to_numpy(gv, dt)))
            out["gather_rows"] = np.array(gk.shape[0])
        elif kind == "direct":
            q, k, v = (to_torch(case[x], dt) for x in ("query", "keys", "values"))
            cu = [int(x) for x in case["cu_seqlens"]]
            result = torch.empty_like(q)
            for s, e in zip(cu[:-1], cu[1:]):
                if e > s:
                    result[s:e] = _direct_prefill_sdpa(q[s:e], k[s:e], v[s:e])
            out["out"] = to_numpy(result, dt)
        elif kind == "cow":
            kp = to_torch(case["key_pool"], dt).clone()
            vp = to_torch(case["value_pool"], dt).clone()
            pairs = torch.from_numpy(case["pairs"].astype(np.int64))
            kp[:, pairs[:, 1]] = kp[:, pairs[:, 0]]
            vp[:, pairs[:, 1]] = vp[:, pairs[:, 0]]
            out["key_pool_digest"] = np.array(cases.digest(to_numpy(kp, dt)))
            out["value_pool_digest"] = np.array(cases.digest(to_numpy(vp, dt)))
        elif kind == "write_checked":
            layer = LayerKVCache(to_torch(case["key_cache"], dt).clone(),
                                 to_torch(case["value_cache"], dt).clone())
            layer.write_checked(torch.from_numpy(case["slots"]), to_torch(case["keys"], dt),
                                to_torch(case["values"], dt))
            out["key_cache"] = to_numpy(layer.keys, dt)
            out["value_cache"] = to_numpy(layer.values, dt)
        np.savez_compressed(HERE / f"{name}.npz", **out)
        print(f"wrote {name}.npz ({(HERE / f'{name}.npz').stat().st_size} bytes)")


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    root = args[0] if args else os.environ.get("MICROINFER_REFERENCE", "")
    if not root:
        raise SystemExit("usage: make_golden.py /path/to/MicroInfer")
    main(root)
