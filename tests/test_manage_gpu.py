"""Parity of the sm_100a manage kernel (through the C-ABI) with the reference's policy.

* Every golden case -- the five routing suites under three policy settings, the twelve
  published miss-count traces, and the four 4096-step policy-simulation traces under
  both policies -- replayed on the GPU: per-step n_miss, installed pairs, the chained
  digest of the full state after every step, and the final state must equal the
  reference model's (tests/golden/golden.npz).
* Randomised cases over E, S, mk, caps, ids outside [0, E), both policies and several
  decay periods, compared field by field after every step with the CPU oracle, including
  the fields the reference model does not track (``routed``, the miss-list entries past
  n_miss) and the fused remap in int32 and int64.
* The sequence recorded in a CUDA graph and replayed.
All comparisons are bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_cases import cases
from gpu_util import DEV, DeviceState, compare_state, lib, manage
from oracle import hashing, policy

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h():
    return lib()


def replay_golden(h, case, remap_dtype=torch.int32):
    st = policy.CacheState.warm(case.E, case.S, case.hot, miss_cap=case.mi)
    ds = DeviceState(st)
    steps, mk = case.trace.shape
    trace = torch.from_numpy(case.trace.astype(np.int32)).to(DEV)
    hist = {f: torch.empty((steps,) + tuple(getattr(ds, f).shape),
                           dtype=getattr(ds, f).dtype, device=DEV)
            for f in ("table", "map_cold", "slot_expert", "slot_stamp", "step", "n_miss",
                      "miss")}
    out = torch.empty((steps, mk), dtype=remap_dtype, device=DEV)
    for t in range(steps):
        manage(h, ds, trace[t], case.md, case.mi, case.policy, case.decay, out=out[t])
        for f, buf in hist.items():
            buf[t].copy_(getattr(ds, f))
    torch.cuda.synchronize()
    hist = {f: v.cpu().numpy() for f, v in hist.items()}
    chain = hashing.start()
    pairs = []
    for t in range(steps):
        chain = hashing.fold(chain, hist["table"][t], hist["map_cold"][t],
                             hist["slot_expert"][t], hist["slot_stamp"][t], hist["step"][t])
        n = int(hist["n_miss"][t][0])
        pairs.extend(hist["miss"][t][:2 * n].reshape(-1, 2).tolist())
    np.testing.assert_array_equal(hist["n_miss"][:, 0], case.nmiss, err_msg=case.key)
    if len(case.pairs):
        np.testing.assert_array_equal(np.array(pairs).reshape(-1, 2), case.pairs,
                                      err_msg=case.key)
    assert hashing.as_u64(chain) == case.chain, case.key
    for k, v in case.final.items():
        np.testing.assert_array_equal(getattr(ds, k).cpu().numpy(), v, err_msg=case.key)
    return ds, out.cpu().numpy()


def test_golden_suites(h, golden):
    for case in cases(golden, "suite:"):
        replay_golden(h, case)


def test_golden_published_miss_counts(h, golden):
    for case in cases(golden, "kat:"):
        replay_golden(h, case)


def test_golden_policy_simulation_config(h, golden):
    """E128 top-8 S64, 4096 steps, LFU decay 64 and LRU, seeds 0-3 (bit-exact)."""
    for case in cases(golden, "cfg1:"):
        ds, out = replay_golden(h, case, remap_dtype=torch.int64)
        # the remap of the last step against the oracle on the final table
        want = policy.remap(case.final["table"], case.trace[-1], np.int64)
        np.testing.assert_array_equal(out[-1], want)


def _random_case(rng):
    E = int(rng.choice([1, 3, 8, 32, 128, 129, 300, 512, 1024, 3000]))
    S = int(rng.integers(1, min(1024, 2 * E + 8) + 1))
    mk = int(rng.choice([0, 1, 2, 8, 32, 50, 255, 256, 257, 700]))
    mi = int(rng.choice([0, 1, 4, S, min(1024, 2 * S)]))
    mi = max(0, min(mi, 1024))
    md = int(rng.choice([-1, 0, 4, 8, E, 10 ** 6]))
    pol = int(rng.integers(0, 2))
    decay = int(rng.choice([0, 1, 3, 64]))
    return E, S, mk, mi, md, pol, decay


def _ids(rng, E, mk):
    ids = rng.integers(-2, E + 2, size=mk).astype(np.int32)
    hot = rng.integers(0, max(1, E // 4 + 1), size=mk).astype(np.int32)   # some locality
    return np.where(rng.random(mk) < 0.6, hot, ids)


def oracle_step_nins(st, ids, md, mi, E):
    valid = np.unique(ids[(ids >= 0) & (ids < E)])
    if len(valid) > md:
        return 0
    return min(int(np.count_nonzero(st.table[valid] < 0)), mi)


def run_case(h, E, S, mk, mi, md, pol, decay, steps, rng, out_dtype=None):
    cap = max(mi, 1)
    if S <= E and rng.random() < 0.7:
        st = policy.CacheState.warm(E, S, rng.choice(E, size=S, replace=False), miss_cap=cap)
    else:
        st = policy.CacheState(E, S, miss_cap=cap)
    ds = DeviceState(st)
    out = torch.empty(max(mk, 1), dtype=out_dtype or torch.int32, device=DEV)
    tag = f"E{E} S{S} mk{mk} mi{mi} md{md} p{pol} d{decay}"
    for t in range(steps):
        ids = _ids(rng, E, mk)
        nins = oracle_step_nins(st, ids, md, mi, E)
        policy.manage(st, ids, md, mi, pol, decay)
        ids_t = torch.from_numpy(ids).to(DEV)
        manage(h, ds, ids_t, md, mi, pol, decay, out=out[:mk])
        compare_state(ds.host(), st, nins, f"{tag} t{t}")
        if mk:
            want = policy.remap(st.table, ids, np.int64)
            np.testing.assert_array_equal(out[:mk].cpu().numpy().astype(np.int64), want,
                                          err_msg=f"{tag} t{t}: remap")
        assert not policy.check_invariants(st), tag


def test_random_cases_vs_oracle(h):
    rng = np.random.default_rng(7)
    for i in range(60):
        E, S, mk, mi, md, pol, decay = _random_case(rng)
        run_case(h, E, S, mk, mi, md, pol, decay, steps=12, rng=rng,
                 out_dtype=torch.int64 if i % 2 else torch.int32)


def test_decode_shapes_many_steps(h):
    """The benchmark shapes (E128 top-8, tokens 1 and 4, S 16..96), long enough to churn."""
    rng = np.random.default_rng(11)
    for S in (16, 32, 64, 96):
        for mk in (8, 32):
            for pol in (0, 1):
                run_case(h, 128, S, mk, S, min(128, mk), pol, 64, steps=40, rng=rng)


def test_largest_sizes(h):
    """E at its bound (shared-memory opt-in path) and S = max_inserts = 1024."""
    rng = np.random.default_rng(3)
    run_case(h, 32768, 1024, 2048, 1024, 10 ** 6, 1, 4, steps=6, rng=rng)
    run_case(h, 1024, 1024, 1024, 1024, 1024, 0, 64, steps=6, rng=rng)
    run_case(h, 2000, 700, 900, 1000, 10 ** 6, 1, 2, steps=6, rng=rng)


def test_remap_torch_semantics_on_device(h):
    """Negative ids count from the end, like ``table[topk_ids.long()]`` in torch."""
    E, S = 16, 8
    st = policy.CacheState.warm(E, S, list(range(8)))
    ds = DeviceState(st)
    ids = torch.tensor([3, -1, 15, 9, -16, 0, 20, -17], dtype=torch.int32, device=DEV)
    out = torch.empty(8, dtype=torch.int64, device=DEV)
    manage(h, ds, ids, 10 ** 6, S, 0, 64, out=out)
    policy.manage(st, ids.cpu().numpy(), 10 ** 6, S, 0, 64)
    want = policy.remap(st.table, ids.cpu().numpy(), np.int64)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    table = torch.from_numpy(st.table)
    in_range = ids.cpu().long()[(ids.cpu() >= -E) & (ids.cpu() < E)]
    np.testing.assert_array_equal(out.cpu()[(ids.cpu() >= -E) & (ids.cpu() < E)].numpy(),
                                  table[in_range].long().numpy())


def test_cuda_graph_replay(h):
    """manage+remap captured once, replayed with new ids copied into the captured input."""
    E, S, mk = 128, 32, 8
    st = policy.CacheState(E, S)
    ds = DeviceState(st)
    ids_buf = torch.zeros(mk, dtype=torch.int32, device=DEV)
    out = torch.empty(mk, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            manage(h, ds, ids_buf, E, S, 1, 64, out=out)
    # capture does not execute: the state is still the initial one
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ds.step.cpu().numpy(), [0])
    from synthetic import sticky_zipf_trace
    trace = sticky_zipf_trace(9, steps=200, E=E)
    for t in range(200):
        ids_buf.copy_(torch.from_numpy(trace[t]))
        g.replay()
        nins = oracle_step_nins(st, trace[t], E, S, E)
        policy.manage(st, trace[t], E, S, 1, 64)
        if t % 20 == 19:
            torch.cuda.synchronize()
            compare_state(ds.host(), st, nins, f"graph t{t}")
            np.testing.assert_array_equal(out.cpu().numpy(), policy.remap(st.table, trace[t]))


def test_two_replicas_evolve_identically(h):
    """Tensor-parallel ranks see the same routing: their caches must stay identical."""
    E, S = 128, 64
    a, b = DeviceState(policy.CacheState(E, S)), DeviceState(policy.CacheState(E, S))
    from synthetic import sticky_zipf_trace
    tr = torch.from_numpy(sticky_zipf_trace(2, steps=300)).to(DEV)
    side = torch.cuda.Stream()
    for t in range(300):
        manage(h, a, tr[t], E, S, 1, 64)
        with torch.cuda.stream(side):
            side.wait_stream(torch.cuda.current_stream())
            manage(h, b, tr[t], E, S, 1, 64)
        torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    ha, hb = a.host(), b.host()
    for f in ("table", "map_cold", "slot_expert", "slot_stamp", "step"):
        np.testing.assert_array_equal(ha[f], hb[f])
