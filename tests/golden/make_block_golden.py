"""Record the reference BlockManager on the seeded engine trace (block_trace.py).

Imports the reference from its source tree (path as the first argument, default
the repository's baseline/_ref install), runs ``run_trace`` on its
``BlockManager`` and ``Sequence`` (block size 4, 24 pages) and writes
``tests/golden/block_manager_trace.json``.  The fixture is committed; the test
replays the same trace on CowBlockManager without the reference.
"""
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
ref = sys.argv[1] if len(sys.argv) > 1 else str(HERE.parent.parent / "baseline" / "_ref")
sys.path.append(ref)  # after this repository: its own tests package must not shadow ours

from microinfer.engine.blockmanager import BlockManager  # noqa: E402
from microinfer.engine.sequence import Sequence  # noqa: E402

from tests.golden.block_trace import run_trace  # noqa: E402

Sequence.block_size = 4
out = {}
for seed, (pages, steps) in {0: (24, 400), 1: (12, 400), 2: (40, 600)}.items():
    out[str(seed)] = {"pages": pages, "steps": steps,
                      "records": run_trace(BlockManager(pages, 4), Sequence, seed, steps)}
(HERE / "block_manager_trace.json").write_text(json.dumps(out, separators=(",", ":")))
print({s: len(v["records"]) for s, v in out.items()})
