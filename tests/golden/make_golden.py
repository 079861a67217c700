"""Generate the golden fixtures from the reference's own Python policy model.

Run in the build container, where the reference checkout is readable:

    python tests/golden/make_golden.py --ref PATH        (PATH: the reference checkout)

What it runs from the reference, extracted by ``ast`` so the modules' import-time side
effects (a ``ctypes.CDLL`` of the HIP library, tests/test_policy.py:20-22) never execute:

* ``ref_step`` -- the reference's independent numpy model of ``expert_cache_manage_k``
  (tests/test_policy.py:83-132);
* ``zipf_trace`` / ``interleaved_trace`` -- the seeded routing generators behind the
  published miss counts (tests/compare_policies.py:51-73, driven as in :77-93).

What it writes (``tests/golden/golden.npz``), per case: the routing trace, the initial
state, the call parameters, the per-step ``n_miss`` and installed (expert, slot) pairs, a
chained digest of the full state after every step (oracle/hashing.py) and the final
state.  The GPU box has no reference checkout; the tests read only this file.
"""

from __future__ import annotations

import argparse
import ast
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "vllm-expert-cache_b200"))

from oracle import hashing  # noqa: E402
from synthetic import sticky_zipf_trace  # noqa: E402

OUT = Path(__file__).resolve().parent / "golden.npz"


def extract(path: Path, names: list[str], env: dict) -> dict:
    """Exec only the named top-level function definitions of ``path``."""
    tree = ast.parse(path.read_text())
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    missing = set(names) - {n.name for n in keep}
    if missing:
        raise SystemExit(f"{path}: functions not found: {sorted(missing)}")
    mod = ast.Module(body=keep, type_ignores=[])
    ns = dict(env)
    exec(compile(mod, str(path), "exec"), ns)
    return {n: ns[n] for n in names}


def ref_state(E, S, hot):
    """The state object ``ref_step`` mutates (field names from tests/test_policy.py:71-76)."""
    table = np.full(E, -1, dtype=np.int32)
    cold = np.arange(E, dtype=np.int32)
    se = np.full(S, -1, dtype=np.int32)
    hot = np.asarray(hot, dtype=np.int64)
    table[hot] = np.arange(len(hot), dtype=np.int32)
    cold[hot] = -1
    se[: len(hot)] = hot.astype(np.int32)
    return SimpleNamespace(E=E, S=S, r_table=table, r_cold=cold, r_se=se,
                           r_st=np.zeros(S, dtype=np.int64), r_step=0)


def trace_digest(trace) -> int:
    import hashlib
    a = np.ascontiguousarray(np.asarray(trace), dtype="<i4")
    return int.from_bytes(hashlib.blake2b(a.tobytes(), digest_size=8).digest(), "little")


def run_case(ref_step, name, E, S, trace, hot, md, mi, policy, decay, keep_pairs,
             store_trace=True):
    s = ref_state(E, S, hot)
    chain = hashing.start()
    nmiss = np.zeros(len(trace), dtype=np.int32)
    pairs = []
    for t, ids in enumerate(trace):
        out = ref_step(s, np.asarray(ids).ravel(), md, mi, policy=policy, decay=decay)
        nmiss[t] = len(out)
        if keep_pairs:
            pairs.extend(out)
        chain = hashing.fold(chain, s.r_table, s.r_cold, s.r_se, s.r_st,
                             np.array([s.r_step], dtype=np.int64))
    rec = {
        "E": E, "S": S, "md": md, "mi": mi, "policy": policy, "decay": decay,
        "trace_digest": np.array([trace_digest(trace)], dtype=np.uint64),
        "hot": np.asarray(hot, dtype=np.int32),
        "nmiss": nmiss,
        "pairs": np.asarray(pairs, dtype=np.int16).reshape(-1, 2),
        "chain": np.array([hashing.as_u64(chain)], dtype=np.uint64),
        "final_table": s.r_table.copy(), "final_cold": s.r_cold.copy(),
        "final_se": s.r_se.copy(), "final_st": s.r_st.copy(),
        "final_step": np.array([s.r_step], dtype=np.int64),
    }
    if store_trace:
        rec["trace"] = np.asarray(trace, dtype=np.int16)
    return {f"{name}/{k}": np.asarray(v) for k, v in rec.items()}


def suite_traces():
    """Routing suites with the shapes of tests/test_policy.py:202-221 (own seeded draws).

    Each yields (name, E, S, steps, max_distinct, max_inserts, hot, trace).
    """
    out = []
    rng = np.random.default_rng(20240611)

    def warm(E, S):
        return sorted(rng.choice(E, S, replace=False).tolist())

    # tiny high-churn: E32 S8, 2 tokens x 5 ids with replacement
    E, S = 32, 8
    hot = warm(E, S)
    out.append(("tiny-churn", E, S, 8, 8, hot,
                np.stack([rng.choice(E, size=10, replace=True) for _ in range(200)])))
    # skewed E512 S257: 5 tokens x top-10 drawn from Zipf(1.1) without replacement
    E, S = 512, 257
    p = np.arange(1, E + 1, dtype=float) ** -1.1
    p /= p.sum()
    hot = warm(E, S)
    out.append(("skewed-512", E, S, 128, 64, hot,
                np.stack([np.concatenate([rng.choice(E, 10, replace=False, p=p)
                                          for _ in range(5)]) for _ in range(300)])))
    # insert-capped: more distinct misses than max_inserts
    E, S = 128, 32
    hot = warm(E, S)
    out.append(("insert-capped", E, S, 128, 4, hot,
                np.stack([rng.choice(E, size=80, replace=True) for _ in range(150)])))
    # read-through gate: distinct > max_distinct changes nothing but the step counter
    hot = warm(E, S)
    out.append(("read-through", E, S, 8, 16, hot,
                np.stack([rng.choice(E, size=160, replace=True) for _ in range(60)])))
    # padded rows: -1 sentinels ignored
    E, S = 64, 16
    hot = warm(E, S)
    tr = np.stack([rng.choice(E, size=40, replace=True) for _ in range(120)])
    tr[:, 20:] = -1
    out.append(("padded-rows", E, S, 64, 16, hot, tr))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the reference checkout")
    args = ap.parse_args()
    ref = Path(args.ref)
    env = {"np": np, "POLICY": 0, "DECAY": 64}
    ref_step = extract(ref / "tests" / "test_policy.py", ["ref_step"], env)["ref_step"]
    gens = extract(ref / "tests" / "compare_policies.py",
                   ["zipf_trace", "interleaved_trace"], {"np": np})

    rec: dict[str, np.ndarray] = {}
    cases = []

    # 1. the routing suites, both policies, plus LFU with a short decay period
    for name, E, S, md, mi, hot, trace in suite_traces():
        for pol, dec in ((0, 64), (1, 64), (1, 8)):
            key = f"suite:{name}:p{pol}d{dec}"
            rec.update(run_case(ref_step, key, E, S, trace, hot, md, mi, pol, dec, True))
            cases.append(key)

    # 2. the published miss counts: rng seed 1234, E128 top-8, 600 steps, cold start
    for gname, fn in (("zipf", gens["zipf_trace"]), ("interleaved", gens["interleaved_trace"])):
        for S in (16, 32, 64):
            trace = fn(np.random.default_rng(1234), 600, 128, 8)
            for pol in (0, 1):
                key = f"kat:{gname}:S{S}:p{pol}"
                rec.update(run_case(ref_step, key, 128, S, trace, [], 8, S, pol, 64, False))
                cases.append(key)

    # 3. the policy-simulation benchmark configuration: E128 top-8 S64, 4096 steps
    for seed in range(4):
        trace = sticky_zipf_trace(seed, steps=4096)
        for pol in (1, 0):
            key = f"cfg1:seed{seed}:p{pol}"
            rec.update(run_case(ref_step, key, 128, 64, trace, [], 8, 64, pol, 64, False,
                                store_trace=False))
            cases.append(key)

    rec["cases"] = np.array(cases)
    np.savez_compressed(OUT, **rec)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(cases)} cases)")
    for k in cases:
        if k.startswith("kat:"):
            print(f"  {k}: {int(rec[k + '/nmiss'].sum())} misses")


if __name__ == "__main__":
    main()
