"""Property tests of the oracle's extension rules (CPU, hypothesis).

The GPU tests compare the kernels with ``oracle.policy`` field by field, so these pin the
oracle itself on arbitrary call sequences:

* a prefetch never advances ``step``, never changes a resident expert's priority, never
  evicts an expert the previous call routed, and installs only predicted experts;
* after any mix of manage and prefetch calls the state invariants hold (table and
  slot_expert inverse, map_cold the complement);
* ``manage_ep`` equals translating the ids, calling ``manage`` on a copy of the state and
  composing the map; the composed map sends an expert to a slot exactly when the expert
  is local and resident.
"""

from __future__ import annotations

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import policy

E, S = 12, 4

ids_st = st.lists(st.integers(min_value=-2, max_value=E + 1), min_size=0, max_size=10)
calls_st = st.lists(st.tuples(st.sampled_from(["manage", "prefetch"]), ids_st),
                    min_size=1, max_size=25)


def _md(ids):
    return max(0, min(E, len(ids)))


@settings(max_examples=200, deadline=None)
@given(calls=calls_st, pol=st.sampled_from([policy.LRU, 1]))
def test_prefetch_rules_hold_on_any_call_sequence(calls, pol):
    cs = policy.CacheState(E, S)
    for kind, ids in calls:
        ids = np.asarray(ids, dtype=np.int32)
        if kind == "manage":
            policy.manage(cs, ids, _md(ids), S, pol, 3)
        else:
            before = cs.copy()
            pairs = policy.prefetch(cs, ids, _md(ids), S, pol)
            assert int(cs.step[0]) == int(before.step[0])
            predicted = {int(e) for e in ids if 0 <= e < E}
            for e, sl in pairs:
                assert e in predicted and int(before.table[e]) < 0
                old = int(before.slot_expert[sl])
                assert old < 0 or not before.routed[old]      # last step's set is parked
                assert old not in predicted
            installed = {sl for _, sl in pairs}
            for sl in range(S):
                if sl not in installed:
                    assert cs.slot_stamp[sl] == before.slot_stamp[sl]
                    assert cs.slot_expert[sl] == before.slot_expert[sl]
            assert int(cs.n_miss[0]) == len(pairs)
        assert not policy.check_invariants(cs)


emap_st = st.lists(st.integers(min_value=-1, max_value=E + 2), min_size=1, max_size=24)


@settings(max_examples=200, deadline=None)
@given(emap=emap_st, steps=st.lists(ids_st, min_size=1, max_size=12),
       pol=st.sampled_from([policy.LRU, 1]))
def test_manage_ep_is_translate_manage_compose(emap, steps, pol):
    emap = np.asarray(emap, dtype=np.int32)
    Eg = emap.size
    a, b = policy.CacheState(E, S), policy.CacheState(E, S)
    for ids in steps:
        ids = np.asarray([g % (Eg + 2) - 1 for g in ids], dtype=np.int32)   # -1..Eg
        pairs, cmap = policy.manage_ep(a, ids, emap, _md(ids), S, pol, 2)
        local = policy.local_ids(ids, emap)
        assert pairs == policy.manage(b, local, _md(ids), S, pol, 2)
        for f in ("table", "map_cold", "slot_expert", "slot_stamp", "routed", "step"):
            np.testing.assert_array_equal(getattr(a, f), getattr(b, f))
        for g in range(Eg):
            e = int(emap[g])
            want = int(a.table[e]) if 0 <= e < E else -1
            assert int(cmap[g]) == want
            if cmap[g] >= 0:
                assert int(a.slot_expert[cmap[g]]) == e
