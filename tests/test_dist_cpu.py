"""The N>1 plumbing of bench.py on CPU: two ranks over gloo (127.0.0.1).

The cache path has no collective -- each tensor-parallel rank runs its own replica -- so
what is shared is the benchmark's barrier and its max/sum over ranks; the reference arm
must run on rank 0 only and let the other ranks exit cleanly.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

CHILD = """
import sys
sys.path.insert(0, {root!r})
import bench
d = bench.Dist()
d.init("gloo")
d.barrier()
m = d.max(float(d.rank + 1))
s = d.sum(10.0)
assert m == d.world == 2 and s == 20.0, (m, s)
d.barrier()
print("RANK_OK", d.rank)
d.close()
"""


def torchrun(args, port, timeout=180):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node",
           "2", "--master-addr", "127.0.0.1", "--master-port", str(port), *args]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, cwd=ROOT)


def test_two_rank_barrier_and_reductions(tmp_path):
    script = tmp_path / "child.py"
    script.write_text(CHILD.format(root=str(ROOT)))
    r = torchrun([str(script)], 29631)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.count("RANK_OK") == 2


def test_reference_arm_rank0_only():
    r = torchrun([str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2", "--steps",
                  "4", "--warmup", "3"], 29632, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["cores"] >= 1
    assert line["n_gpus"] == 2 and line["steps"] == 4 and line["warmup"] == 3
