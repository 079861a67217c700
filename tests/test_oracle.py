"""The CPU oracle against the reference's golden vectors (no GPU).

Both restatements -- oracle/policy.py and oracle/policy.c -- must reproduce, on every
fixture case, the reference model's per-step miss counts, installed (expert, slot) pairs,
the chained digest of the full state after every step, and the final state; plus the
twelve published miss counts.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from golden_cases import PUBLISHED, cases, load
from oracle import hashing, policy, policy_c


def replay(case, impl):
    st = policy.CacheState.warm(case.E, case.S, case.hot, miss_cap=case.mi)
    chain = hashing.start()
    nmiss, pairs = [], []
    for ids in case.trace:
        if impl == "py":
            out = policy.manage(st, ids, case.md, case.mi, case.policy, case.decay)
        else:
            assert policy_c.manage(st, ids, case.md, case.mi, case.policy, case.decay) == 0
            n = int(st.n_miss[0])
            out = [(int(st.miss[2 * j]), int(st.miss[2 * j + 1])) for j in range(n)]
        assert int(st.n_miss[0]) == len(out)
        nmiss.append(len(out))
        pairs.extend(out)
        assert not policy.check_invariants(st)
        chain = hashing.fold(chain, st.table, st.map_cold, st.slot_expert, st.slot_stamp,
                             st.step)
    return st, np.array(nmiss), pairs, hashing.as_u64(chain)


def _check(case, impl):
    st, nmiss, pairs, chain = replay(case, impl)
    np.testing.assert_array_equal(nmiss, case.nmiss)
    if len(case.pairs):
        np.testing.assert_array_equal(np.array(pairs).reshape(-1, 2), case.pairs)
    assert chain == case.chain
    for k, v in case.final.items():
        np.testing.assert_array_equal(getattr(st, k), v, err_msg=k)


def test_fixture_has_all_cases(golden):
    keys = golden["cases"].tolist()
    assert sum(k.startswith("suite:") for k in keys) == 15
    assert sum(k.startswith("kat:") for k in keys) == 12
    assert sum(k.startswith("cfg1:") for k in keys) == 8


@pytest.mark.parametrize("impl", ["py", "c"])
def test_suites_match_reference(golden, impl):
    for case in cases(golden, "suite:"):
        _check(case, impl)


@pytest.mark.parametrize("impl", ["py", "c"])
def test_published_miss_counts(golden, impl):
    for (gen, S), (lru, lfu) in PUBLISHED.items():
        for pol, want in ((0, lru), (1, lfu)):
            case = load(golden, f"kat:{gen}:S{S}:p{pol}")
            assert int(case.nmiss.sum()) == want
            _check(case, impl)


def test_cfg1_traces_are_the_fixture_traces(golden):
    for case in cases(golden, "cfg1:"):
        a = np.ascontiguousarray(case.trace, dtype="<i4")
        d = int.from_bytes(hashlib.blake2b(a.tobytes(), digest_size=8).digest(), "little")
        assert d == int(golden[f"{case.key}/trace_digest"][0])
        assert case.trace.shape == (4096, 8)
        assert all(len(set(r.tolist())) == 8 for r in case.trace[:256])


def test_cfg1_policy_sim_c(golden):
    for case in cases(golden, "cfg1:"):
        _check(case, "c")


def test_cfg1_policy_sim_py_one_seed(golden):
    _check(load(golden, "cfg1:seed0:p1"), "py")


def test_run_matches_stepwise(golden):
    case = load(golden, "cfg1:seed1:p1")
    st = policy.CacheState(case.E, case.S)
    nm = policy_c.run(st, case.trace, case.md, case.mi, case.policy, case.decay)
    np.testing.assert_array_equal(nm, case.nmiss)


def test_arg_checks_match_launcher_rule():
    st = policy.CacheState(8, 4)
    for E, S, mi, pol in ((0, 4, 4, 0), (8, 0, 4, 0), (8, 1025, 4, 0), (8, 4, -1, 0),
                          (8, 4, 1025, 0), (8, 4, 4, 2), (8, 4, 4, -1)):
        assert policy.check_args(E, S, mi, pol) == -1
        bad = policy.CacheState(max(E, 1), max(min(S, 1024), 1))
        bad.E, bad.S = E, S
        assert policy_c.manage(bad, [0], 8, mi, pol, 64) == -1
    assert policy.check_args(8, 4, 4, 1) == 0
    assert policy_c.manage(st, [0, 1], 8, 4, 1, 64) == 0


def test_remap_torch_semantics():
    import torch
    table = np.array([3, -1, 0, 2], dtype=np.int32)
    ids = np.array([[0, 2, -1, 3], [1, 0, -4, 2]], dtype=np.int32)
    want = torch.from_numpy(table)[torch.from_numpy(ids).long()].int().numpy()
    np.testing.assert_array_equal(policy.remap(table, ids), want)
    np.testing.assert_array_equal(policy_c.remap(table, ids).reshape(ids.shape), want)
    np.testing.assert_array_equal(policy.remap(table, np.array([4, -5])), [-1, -1])


def test_gather_oracle_bytes():
    rng = np.random.default_rng(0)
    E, S, sizes = 6, 3, [32, 48, 16]
    srcs = [rng.integers(0, 256, E * b, dtype=np.uint8) for b in sizes]
    d1 = [np.zeros(S * b, np.uint8) for b in sizes]
    d2 = [np.zeros(S * b, np.uint8) for b in sizes]
    miss = np.array([4, 2, 1, 0, 5, 1], dtype=np.int32)
    n = np.array([3], dtype=np.int32)
    policy.gather(d1, srcs, sizes, miss, n)
    policy_c.gather(d2, srcs, sizes, miss, n)
    for a, b, s, sz in zip(d1, d2, srcs, sizes):
        np.testing.assert_array_equal(a, b)
        np.testing.assert_array_equal(a[2 * sz:3 * sz], s[4 * sz:5 * sz])


def _random_case(rng):
    E = int(rng.choice([1, 3, 8, 32, 128, 129, 300, 512, 1024]))
    S = int(rng.integers(1, min(1024, 2 * E + 8) + 1))
    mk = int(rng.choice([0, 1, 8, 32, 257]))
    mi = int(min(1024, rng.choice([0, 1, 4, S])))
    md = int(rng.choice([-1, 0, 4, 8, E, 10 ** 6]))
    return E, S, mk, mi, md, int(rng.integers(0, 2)), int(rng.choice([0, 1, 3, 64]))


def test_c_oracle_agrees_with_python_oracle_on_random_cases():
    rng = np.random.default_rng(1)
    for _ in range(40):
        E, S, mk, mi, md, pol, decay = _random_case(rng)
        a = policy.CacheState(E, S, miss_cap=max(mi, 1))
        b = a.copy()
        for _ in range(6):
            ids = rng.integers(-2, E + 2, size=mk).astype(np.int32)
            policy.manage(a, ids, md, mi, pol, decay)
            assert policy_c.manage(b, ids, md, mi, pol, decay) == 0
            for k, v in a.fields().items():
                np.testing.assert_array_equal(v, getattr(b, k), err_msg=k)
            nins = int(a.n_miss[0])
            np.testing.assert_array_equal(a.miss[:2 * nins], b.miss[:2 * nins])


def test_align_oracle_small_known_answer():
    """vLLM's documented example (moe_align_block_size.py:59-72), all experts cold: the
    cold side must reproduce it; the hot side is then empty."""
    table = np.full(5, -1, dtype=np.int32)            # experts 0..4, none resident
    ids = np.array([2, 3, 4, 1, 2, 4, 1, 3, 4, 1, 2, 3], dtype=np.int32)
    L, NB = policy.align_lengths(12, 5, 4)
    sh, eh, nh, sc, ec, nc = policy.align(table, ids, 4, 4, L, NB)
    assert nh[0] == 0 and (eh == -1).all() and (sh == 12).all()
    assert nc[0] == 16
    np.testing.assert_array_equal(sc[:16], [3, 6, 9, 12, 0, 4, 10, 12, 1, 7, 11, 12,
                                            2, 5, 8, 12])
    np.testing.assert_array_equal(ec[:4], [1, 2, 3, 4])


def test_align_oracle_hot_cold_split():
    table = np.array([-1, 2, -1, 0, -1, 1], dtype=np.int32)   # experts 1,3,5 resident
    ids = np.array([[1, 0], [3, 5], [0, 1], [-1, 4]], dtype=np.int32)
    L, NB = policy.align_lengths(8, 6, 2)
    sh, eh, nh, sc, ec, nc = policy.align(table, ids, 3, 2, L, NB)
    # hot buckets by slot: slot0 <- expert3 (token 2), slot1 <- expert5 (3), slot2 <- 1 (0,5)
    assert nh[0] == 6
    np.testing.assert_array_equal(sh[:6], [2, 8, 3, 8, 0, 5])
    np.testing.assert_array_equal(eh[:3], [0, 1, 2])
    # cold buckets by expert: 0 (tokens 1, 4), 4 (token 7)
    assert nc[0] == 4
    np.testing.assert_array_equal(sc[:4], [1, 4, 7, 8])
    np.testing.assert_array_equal(ec[:2], [0, 4])
    assert (ec[2:] == -1).all()


def test_manage_ep_known_answer():
    """Rank 1 of 2, linear placement: global 4..7 are local 0..3.  Routing [5, 1, 6, -1,
    9]: global 1 is another rank's expert, -1 padding, 9 outside the map; the local step
    installs locals 1 and 2 into the two empty slots (ascending id, slots by (stamp,
    slot)), and the composed map sends globals 5, 6 to slots 0, 1."""
    emap = np.array([-1, -1, -1, -1, 0, 1, 2, 3], dtype=np.int32)
    st = policy.CacheState(4, 2)
    pairs, cmap = policy.manage_ep(st, [5, 1, 6, -1, 9], emap, 4, 2, policy.LRU, 0)
    assert pairs == [(1, 0), (2, 1)]
    assert st.table.tolist() == [-1, 0, 1, -1]
    assert cmap.tolist() == [-1, -1, -1, -1, -1, 0, 1, -1]
    assert st.routed.tolist() == [0, 1, 1, 0]
    # next step: global 7 (local 3) evicts the older of the two unrouted slots
    pairs, cmap = policy.manage_ep(st, [7, 6], emap, 4, 2, policy.LRU, 0)
    assert pairs == [(3, 0)]
    assert cmap.tolist() == [-1, -1, -1, -1, -1, -1, 1, 0]


def test_prefetch_known_answer():
    """Prefetch installs missing predicted experts without the step's bookkeeping: step
    stays, the resident predicted expert keeps its priority, new slots take priority
    ``step`` (LRU)."""
    st = policy.CacheState(8, 3)
    policy.manage(st, [1, 2], 8, 3, policy.LRU, 0)            # step 1: 1->s0, 2->s1
    policy.manage(st, [3], 8, 3, policy.LRU, 0)               # step 2: 3->s2
    assert st.slot_stamp.tolist() == [1, 1, 2]
    pairs = policy.prefetch(st, [2, 5, 6], 8, 3, policy.LRU)
    # slot 1 holds predicted expert 2 and slot 2 the last step's expert 3: both parked,
    # so only slot 0 (expert 1) can take a prediction -- 5, the lower missing id
    assert pairs == [(5, 0)]
    assert int(st.step[0]) == 2
    assert st.slot_stamp.tolist() == [2, 1, 2]
    assert st.table[1] == -1 and st.map_cold[1] == 1 and st.table[2] == 1
    assert int(st.n_miss[0]) == 1 and st.miss[2] == 6          # 6 listed, not installed
    assert st.routed.tolist() == [0, 0, 1, 0, 0, 1, 1, 0]     # the predicted flags
    # a real step afterwards sees the prefetched expert as a hit
    assert policy.manage(st, [5, 3], 8, 3, policy.LRU, 0) == []


def test_prefetch_lfu_keeps_counts_and_skips_ageing():
    st = policy.CacheState(6, 2)
    for _ in range(4):
        policy.manage(st, [0], 6, 2, policy.LFU, 2)
    before = st.slot_stamp.copy()
    policy.prefetch(st, [0, 3], 6, 2, policy.LFU)
    s0 = int(st.table[0])
    assert st.slot_stamp[s0] == before[s0]                    # no refresh, no halving
    assert st.slot_stamp[int(st.table[3])] == 1


def test_pregate_oracle_ties_and_nan():
    x = np.array([[1.0, 0.0], [0.0, 0.0]])
    w = np.array([[1.0, 0.0], [1.0, 0.0], [np.nan, 0.0], [2.0, 0.0]])
    got = policy.pregate(x, w, 3)
    assert got[0].tolist() == [3, 0, 1]                       # tie 0/1 -> lower id first
    assert got[1].tolist() == [0, 1, 3]                       # all zero: ascending ids
    got = policy.pregate(x, w, 4)
    assert got[0].tolist() == [3, 0, 1, -1]                   # NaN never chosen
