"""The N>1 plumbing of bench.py on CPU: two ranks over gloo (127.0.0.1).

The cache path has no collective -- each tensor-parallel rank runs its own replica -- so
what is shared is the benchmark's barrier and its max/sum over ranks; the reference arm
must run on rank 0 only and let the other ranks exit cleanly.  Under expert parallelism
each rank caches its own experts; the two-rank test checks, through the oracle, that the
ranks' composed maps together serve every routed expert exactly once.
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
lo = d.min(float(d.rank + 1))
assert m == d.world == 2 and s == 20.0 and lo == 1.0, (m, s, lo)
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


CHILD_EP = """
import sys
sys.path.insert(0, {root!r})
import numpy as np
import torch
import torch.distributed as dist
from oracle import policy

dist.init_process_group("gloo")
rank, world = dist.get_rank(), dist.get_world_size()
Eg, S, k = 32, 4, 4
emap = np.full(Eg, -1, dtype=np.int32)           # round-robin: global g lives on g % world
emap[rank::world] = np.arange(Eg // world, dtype=np.int32)
st = policy.CacheState(Eg // world, S)
rng = np.random.default_rng(99)                  # the same routing on every rank
for step in range(60):
    ids = rng.choice(Eg, k, replace=False).astype(np.int32)
    _, cmap = policy.manage_ep(st, ids, emap, ids.size, S, step % 2, 8)
    maps = [torch.zeros(Eg, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(maps, torch.from_numpy(cmap))
    maps = torch.stack(maps).numpy()
    for g in range(Eg):
        owners = [r for r in range(world) if maps[r, g] >= 0]
        assert owners in ([], [g % world]), (step, g, owners)
    for g in ids:                                 # every routed expert served exactly once
        assert maps[g % world, g] >= 0, (step, g)
    mine = cmap[cmap >= 0]
    assert len(set(mine.tolist())) == mine.size   # one expert per slot
    assert not policy.check_invariants(st)
dist.barrier()
print("EP_OK", rank)
dist.destroy_process_group()
"""


def test_two_rank_expert_parallel_maps_partition_the_routing(tmp_path):
    """Two EP ranks over gloo, each composing its local cache with vLLM's expert map for
    the same global routing: the gathered global id -> slot maps give every routed expert
    exactly one slot, on the rank that owns it, and no rank ever maps another's expert."""
    script = tmp_path / "child_ep.py"
    script.write_text(CHILD_EP.format(root=str(ROOT)))
    r = torchrun([str(script)], 29633)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.count("EP_OK") == 2
