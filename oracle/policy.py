"""Pure-Python/numpy restatement of the expert-cache step.  TEST INFRASTRUCTURE ONLY.

One call of :func:`manage` is one ``expert_cache_manage`` launch on the same state
arrays the C-ABI takes (``include/expert_cache.h``).  The rules, each with the reference
line it restates:

* ``step += 1`` on every call, read-through included
  (kernels/expert_cache.hip:214-217; tests/test_policy.py:92).
* ``routed[e] = 1`` for every id with ``0 <= id < E``, all others cleared
  (expert_cache.hip:218-226).  Negative ids are padding; ids ``>= E`` are ignored
  (the kernel's bounds guard, expert_cache.hip:224).
* More distinct routed experts than ``max_distinct``: nothing else changes
  (expert_cache.hip:228-232; test_policy.py:93-95).
* In ascending expert id: a resident expert's priority becomes ``step`` (LRU, policy 0)
  or ``priority + 1`` (LFU, policy 1); a non-resident one is a miss
  (expert_cache.hip:236-246; test_policy.py:97-106).
* ``nins = min(#misses, max_inserts)``; ``miss[2j] = e`` for the first ``nins`` misses.
  ``nins == 0`` ends the call before the ageing pass (expert_cache.hip:247-259;
  test_policy.py:107-111).
* LFU ageing: when ``decay > 0`` and ``step % decay == 0`` every slot's priority is
  halved (arithmetic shift) (expert_cache.hip:261-267; test_policy.py:112-114).
* Victims: among slots whose expert is empty (-1) or not routed this step, the ``nins``
  smallest ``(priority, slot)`` pairs in ascending order; the r-th miss goes to the r-th
  victim.  Fewer evictable slots than misses installs only as many as there are
  (expert_cache.hip:83-97, 123-189; test_policy.py:115-121).
* Install: the evicted expert (if any) gets ``table = -1`` / ``map_cold = itself``; the
  new one gets ``table = slot`` / ``map_cold = -1``; the slot's priority becomes
  ``step`` (LRU) or 1 (LFU); ``miss[2r+1] = slot`` (expert_cache.hip:106-121;
  test_policy.py:122-131).
* ``n_miss`` = number installed (0 on every early exit) (expert_cache.hip:216, 281).

:func:`remap` is ``table[ids]`` with torch indexing semantics (vllm_expert_cache/
cache.py:108-110): a negative index counts from the end.  :func:`gather` is the byte copy
``dst[slot] = src[expert]`` for every installed miss (expert_cache.hip:286-314).
"""

from __future__ import annotations

import numpy as np

LRU, LFU = 0, 1
MAX_SLOTS = 1024          # expert_cache.hip:80 (MAXS); launcher check :596
MAX_INSERTS = 1024        # expert_cache.hip:81 (MAXINS); launcher check :597
SLOT_BITS = 20            # expert_cache.hip:33; S must also fit the key's slot field


class CacheState:
    """Host copy of one layer's cache state, laid out exactly like the device arrays.

    Field names and dtypes follow vllm_expert_cache/cache.py:84-92.
    """

    def __init__(self, E: int, S: int, miss_cap: int | None = None):
        self.E, self.S = int(E), int(S)
        cap = self.S if miss_cap is None else int(miss_cap)
        self.table = np.full(self.E, -1, dtype=np.int32)
        self.map_cold = np.arange(self.E, dtype=np.int32)
        self.slot_expert = np.full(self.S, -1, dtype=np.int32)
        self.slot_stamp = np.zeros(self.S, dtype=np.int64)
        self.routed = np.zeros(self.E, dtype=np.uint8)
        self.step = np.zeros(1, dtype=np.int64)
        self.miss = np.zeros(2 * cap, dtype=np.int32)
        self.n_miss = np.zeros(1, dtype=np.int32)

    @classmethod
    def warm(cls, E: int, S: int, hot, miss_cap: int | None = None) -> "CacheState":
        """Experts ``hot[i]`` pre-installed in slot ``i`` (tests/test_policy.py:57-76)."""
        st = cls(E, S, miss_cap)
        hot = np.asarray(hot, dtype=np.int64)
        st.table[hot] = np.arange(len(hot), dtype=np.int32)
        st.map_cold[hot] = -1
        st.slot_expert[: len(hot)] = hot.astype(np.int32)
        return st

    def copy(self) -> "CacheState":
        c = CacheState.__new__(CacheState)
        c.E, c.S = self.E, self.S
        for k in ("table", "map_cold", "slot_expert", "slot_stamp", "routed", "step",
                  "miss", "n_miss"):
            setattr(c, k, getattr(self, k).copy())
        return c

    def fields(self) -> dict:
        return {k: getattr(self, k) for k in
                ("table", "map_cold", "slot_expert", "slot_stamp", "routed", "step",
                 "n_miss")}


def check_args(E, S, max_inserts, policy) -> int:
    """The launcher's argument rule (expert_cache.hip:596-598): 0 = ok, -1 = refused."""
    if E <= 0 or S <= 0 or S > MAX_SLOTS or S > (1 << SLOT_BITS) - 1:
        return -1
    if max_inserts < 0 or max_inserts > MAX_INSERTS:
        return -1
    if policy not in (LRU, LFU):
        return -1
    return 0


def manage(st: CacheState, ids, max_distinct: int, max_inserts: int, policy: int,
           decay: int) -> list[tuple[int, int]]:
    """Apply one manage call to ``st`` in place; return the installed (expert, slot) list."""
    E, S = st.E, st.S
    ids = np.asarray(ids).reshape(-1).astype(np.int64)
    st.step[0] += 1
    now = int(st.step[0])
    st.n_miss[0] = 0

    valid = ids[(ids >= 0) & (ids < E)]
    st.routed[:] = 0
    st.routed[valid] = 1
    routed = np.flatnonzero(st.routed)          # ascending expert id
    if routed.size > max_distinct:
        return []

    stamp = st.slot_stamp                       # updated in place, like the kernel
    missing = []
    for e in routed.tolist():
        s = int(st.table[e])
        if s >= 0:
            stamp[s] = now if policy == LRU else stamp[s] + 1
        else:
            missing.append(e)
    nins = min(len(missing), max_inserts)
    if nins <= 0:
        return []
    for j in range(nins):
        st.miss[2 * j] = missing[j]

    if policy != LRU and decay > 0 and now % decay == 0:
        stamp >>= 1

    # evictable slots, sorted by (priority, slot); the kernel's (stamp<<20 | slot) key
    # orders them identically for any priority below 2**43
    se = st.slot_expert
    evictable = [i for i in range(S)
                 if se[i] < 0 or se[i] >= E or not st.routed[se[i]]]
    evictable.sort(key=lambda i: (int(stamp[i]), i))
    fresh = now if policy == LRU else 1
    out = []
    for r, sl in enumerate(evictable[:nins]):
        e = missing[r]
        old = int(se[sl])
        if old >= 0:
            st.table[old] = -1
            st.map_cold[old] = old
        se[sl] = e
        stamp[sl] = fresh
        st.table[e] = sl
        st.map_cold[e] = -1
        st.miss[2 * r + 1] = sl
        out.append((e, sl))
    st.n_miss[0] = len(out)
    return out


def remap(table: np.ndarray, ids, out_dtype=None) -> np.ndarray:
    """``table[ids]`` with torch's negative-index wrap (vllm_expert_cache/cache.py:110).

    Ids outside ``[-E, E)`` have no torch answer (it raises); the fused CUDA remap writes
    -1 for them and so does this oracle.
    """
    ids = np.asarray(ids)
    E = table.shape[0]
    flat = ids.reshape(-1).astype(np.int64)
    ok = (flat >= -E) & (flat < E)
    out = np.full(flat.shape, -1, dtype=np.int64)
    out[ok] = table[np.where(flat[ok] < 0, flat[ok] + E, flat[ok])]
    return out.astype(out_dtype or ids.dtype).reshape(ids.shape)


def local_ids(ids, expert_map) -> np.ndarray:
    """Global routing ids -> this rank's local experts through vLLM's expert map
    (vllm/model_executor/layers/fused_moe/expert_map_manager.py:22-113: ``map[g]`` is
    the local index, -1 for another rank's expert).  Ids outside the map are -1."""
    ids = np.asarray(ids).reshape(-1).astype(np.int64)
    emap = np.asarray(expert_map).astype(np.int64)
    ok = (ids >= 0) & (ids < emap.shape[0])
    out = np.full(ids.shape, -1, dtype=np.int64)
    out[ok] = emap[ids[ok]]
    return out


def compose_map(table: np.ndarray, expert_map) -> np.ndarray:
    """Global id -> slot: ``table[map[g]]`` where ``map[g]`` names a local expert, else -1."""
    emap = np.asarray(expert_map).astype(np.int64)
    E = table.shape[0]
    ok = (emap >= 0) & (emap < E)
    out = np.full(emap.shape, -1, dtype=np.int32)
    out[ok] = table[emap[ok]]
    return out


def manage_ep(st: CacheState, ids, expert_map, max_distinct: int, max_inserts: int,
              policy: int, decay: int) -> tuple[list[tuple[int, int]], np.ndarray]:
    """``expert_cache_manage_ep``: the reference manage step on the local ids, then the
    composed global-id -> slot map.  The reference has no expert-parallel path (it
    refuses such layers, vllm_expert_cache/backends/generic.py:145-149); this composes
    its manage rules above with vLLM's expert map.  Map entries outside ``[0, E)`` are
    treated like -1, as the kernel's bounds guard does."""
    pairs = manage(st, local_ids(ids, expert_map), max_distinct, max_inserts, policy, decay)
    return pairs, compose_map(st.table, expert_map)


def prefetch(st: CacheState, ids, max_distinct: int, max_inserts: int,
             policy: int) -> list[tuple[int, int]]:
    """``expert_cache_prefetch``: install the predicted experts that are missing, with the
    victim order and install rules of :func:`manage`, and change nothing else -- ``step``
    does not advance, hits keep their priority, no ageing.  New slots take priority
    ``step`` (LRU) or 1 (LFU).  Slots holding an expert the previous call routed (the
    ``routed`` flags on entry) are parked like the predicted ones: a speculative install
    never evicts the last step's working set.  ``routed`` is left holding the predicted
    flags.  The reference has no prefetch (its README.md:392-394 names it as
    unexplored); the rules are the manage rules above minus the step's own bookkeeping."""
    E, S = st.E, st.S
    ids = np.asarray(ids).reshape(-1).astype(np.int64)
    now = int(st.step[0])
    st.n_miss[0] = 0
    previous = st.routed.copy()
    st.routed[:] = 0
    st.routed[ids[(ids >= 0) & (ids < E)]] = 1
    routed = np.flatnonzero(st.routed)
    if routed.size > max_distinct:
        return []
    missing = [e for e in routed.tolist() if st.table[e] < 0]
    nins = min(len(missing), max_inserts)
    if nins <= 0:
        return []
    for j in range(nins):
        st.miss[2 * j] = missing[j]
    se, stamp = st.slot_expert, st.slot_stamp
    evictable = [i for i in range(S)
                 if se[i] < 0 or se[i] >= E or not (st.routed[se[i]] or previous[se[i]])]
    evictable.sort(key=lambda i: (int(stamp[i]), i))
    fresh = now if policy == LRU else 1
    out = []
    for r, sl in enumerate(evictable[:nins]):
        e = missing[r]
        old = int(se[sl])
        if old >= 0:
            st.table[old] = -1
            st.map_cold[old] = old
        se[sl] = e
        stamp[sl] = fresh
        st.table[e] = sl
        st.map_cold[e] = -1
        st.miss[2 * r + 1] = sl
        out.append((e, sl))
    st.n_miss[0] = len(out)
    return out


def pregate_scores(x, gate_w) -> np.ndarray:
    """``x[t] . gate_w[e]`` in float64 from the bf16 values (given as float arrays)."""
    return np.asarray(x, dtype=np.float64) @ np.asarray(gate_w, dtype=np.float64).T


def pregate(x, gate_w, k: int) -> np.ndarray:
    """``expert_cache_pregate``: per token, the k highest scores' expert ids, ties to the
    lower id, NaN never chosen, -1 where fewer than k scores are finite."""
    sc = pregate_scores(x, gate_w)
    T, E = sc.shape
    out = np.full((T, k), -1, dtype=np.int32)
    for t in range(T):
        order = sorted((e for e in range(E) if not np.isnan(sc[t, e])),
                       key=lambda e: (-sc[t, e], e))
        take = order[:k]
        out[t, :len(take)] = take
    return out


def gather(dsts, srcs, nbytes, miss, n_miss) -> None:
    """Byte copy of every installed miss: ``dst_k[slot] = src_k[expert]``.

    ``dsts``/``srcs`` are flat uint8 arrays; ``nbytes[k]`` is buffer k's bytes per expert.
    """
    n = int(np.asarray(n_miss).reshape(-1)[0])
    for j in range(n):
        e, sl = int(miss[2 * j]), int(miss[2 * j + 1])
        for d, s, b in zip(dsts, srcs, nbytes):
            d[sl * b:(sl + 1) * b] = s[e * b:(e + 1) * b]


def check_invariants(st: CacheState) -> list[str]:
    """The structural checks of tests/test_policy.py:162-169, as a list of failures."""
    bad = []
    t, c = st.table, st.map_cold
    ok = ((t >= 0) & (c == -1)) | ((t < 0) & (c == np.arange(st.E)))
    if not ok.all():
        bad.append("table/map_cold not complementary")
    se = st.slot_expert
    live_slots = np.flatnonzero(se >= 0)
    live = se[live_slots]
    if len(np.unique(live)) != len(live):
        bad.append("duplicate expert in slots")
    if len(live) and not (t[live] == live_slots).all():
        bad.append("table/slot mismatch")
    return bad


def align_lengths(mk: int, E: int, bs: int) -> tuple[int, int]:
    """(L, NB): the buffer lengths vLLM's moe_align_block_size wrapper allocates for mk
    routing ids over E experts (vllm/model_executor/layers/fused_moe/
    moe_align_block_size.py:74-84; the reference's fused launcher comment,
    kernels/expert_cache.hip:606-609)."""
    L = mk + E * (bs - 1)
    if mk < E:
        L = min(mk * bs, L)
    return L, (L + bs - 1) // bs


def align(table: np.ndarray, ids, S: int, bs: int, L: int, NB: int):
    """Both moe_align_block_size outputs of the fused step, on the UPDATED table.

    Token i with a valid expert e goes to the hot side in bucket table[e] when
    0 <= table[e] < S, else to the cold side in bucket e (map_cold's value for a
    non-resident expert).  Per side: buckets in ascending order, each padded to a multiple
    of ``bs`` with the sentinel mk; tokens inside a bucket in ascending index; block ->
    bucket ids, -1 for unused blocks; the padded total.  Restates the reference's fused
    kernel phases 1-5 (kernels/expert_cache.hip:515-587) with deterministic placement.
    Returns (sorted_hot, eids_hot, npad_hot, sorted_cold, eids_cold, npad_cold).
    """
    ids = np.asarray(ids).reshape(-1).astype(np.int64)
    E = table.shape[0]
    mk = ids.size
    hot = [[] for _ in range(S)]
    cold = [[] for _ in range(E)]
    for i, e in enumerate(ids.tolist()):
        if e < 0 or e >= E:
            continue
        s = int(table[e])
        (hot[s] if 0 <= s < S else cold[e]).append(i)
    out = []
    for buckets in (hot, cold):
        sorted_ids = np.full(L, mk, dtype=np.int32)
        eids = np.full(NB, -1, dtype=np.int32)
        pos = 0
        for b, toks in enumerate(buckets):
            padded = -(-len(toks) // bs) * bs
            for k, tok in enumerate(toks):
                if pos + k < L:
                    sorted_ids[pos + k] = tok
            for blk in range(pos // bs, (pos + padded) // bs):
                if blk < NB:
                    eids[blk] = b
            pos += padded
        out += [sorted_ids, eids, np.array([pos], dtype=np.int32)]
    return tuple(out)
