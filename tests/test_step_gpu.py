"""The single-launch step (``expert_cache_step``: manage + remap + gather) on the GPU.

* Randomised cases over E (up to the shared-memory opt-in bound), S up to 256, mk, the
  caps, ids outside [0, E) and both policies, compared field by field after every step
  with the CPU oracle -- state, miss list, remap -- and every installed slot byte for byte
  against its expert's pinned host bytes.
* The same drive through ``expert_cache_step`` and through the two launches it replaces
  (``expert_cache_manage_remap`` then ``expert_cache_gather``) at the Qwen3-30B-A3B W8A8
  slab: identical state, slot ids and slot bytes.
* A CUDA graph of many step nodes replayed once, and a graph of one step node replayed
  many times (each replay is a new epoch of the same node); no wait ever runs out and
  the install count is exact.
* The wait bound: with a 1 us bound and a policy step that takes far longer (E = 32768,
  2048 routing ids), the other CTAs' waits run out and are counted in sync[5]; the policy
  CTA then copies every tile alone, so state, remap and slot bytes are still exact.  No
  GPU fault is involved: the wait is a bounded poll that returns.
All comparisons are bit-exact.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gpu_util import DEV, DeviceState, compare_state, device_ptr_of_pinned, lib, p, stream_ptr
from oracle import policy

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h():
    return lib()


def pinned_random(nbytes, seed):
    g = torch.Generator().manual_seed(seed)
    t = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    t.copy_(torch.randint(0, 256, (nbytes,), dtype=torch.uint8, generator=g))
    return t


class Slabs:
    """Pinned host experts (one tensor per size) and their device slot buffers."""

    def __init__(self, E, S, sizes, seed=0):
        self.sizes = list(sizes)
        self.hosts = [pinned_random(E * b, seed + i) for i, b in enumerate(self.sizes)]
        self.srcs = [device_ptr_of_pinned(x) for x in self.hosts]
        self.dsts = [torch.zeros(S * b, dtype=torch.uint8, device=DEV) for b in self.sizes]

    def triples(self):
        t = [(d.data_ptr(), s, b) for d, s, b in zip(self.dsts, self.srcs, self.sizes)]
        t += [t[-1]] * (6 - len(t))
        args = []
        for d, s, b in t:
            args += [ctypes.c_void_p(d), ctypes.c_void_p(s), ctypes.c_long(b)]
        return args

    def check(self, pairs, tag=""):
        for e, sl in pairs:
            for d, hs, b in zip(self.dsts, self.hosts, self.sizes):
                assert torch.equal(d[sl * b:(sl + 1) * b].cpu(), hs[e * b:(e + 1) * b]), \
                    f"{tag}: expert {e} slot {sl} ({b} B)"


def step(h, ds, ids_t, md, mi, pol, decay, out, slabs, sync, chunks=16, lanes=64, wait_us=0):
    rc = h.expert_cache_step(p(ids_t), ids_t.numel(), ds.E, ds.S, md, mi, *ds.ptrs(), pol,
                             decay, p(out), out.element_size(), *slabs.triples(), chunks,
                             lanes, p(sync), wait_us, stream_ptr())
    assert rc == 0, f"step rc={rc}"


def _ids(rng, E, mk):
    ids = rng.integers(-2, E + 2, size=mk).astype(np.int32)
    hot = rng.integers(0, max(1, E // 4 + 1), size=mk).astype(np.int32)
    return np.where(rng.random(mk) < 0.6, hot, ids)


def nins_of(st, ids, md, mi, E):
    valid = np.unique(ids[(ids >= 0) & (ids < E)])
    if len(valid) > md:
        return 0
    return min(int(np.count_nonzero(st.table[valid] < 0)), mi)


def counters(sync):
    """(timed-out waits, installs) from a step's sync array."""
    c = sync.cpu()
    return int(c[5]), int(c[6:8].view(torch.int64)[0])


def drive(h, E, S, mk, mi, md, pol, decay, steps, rng, sizes=(48, 32, 16), chunks=16,
          lanes=64, out_dtype=torch.int32):
    cap = max(mi, 1)
    if S <= E and rng.random() < 0.6:
        st = policy.CacheState.warm(E, S, rng.choice(E, size=S, replace=False), miss_cap=cap)
    else:
        st = policy.CacheState(E, S, miss_cap=cap)
    ds = DeviceState(st)
    slabs = Slabs(E, S, sizes, seed=int(rng.integers(1 << 20)))
    # slots already occupied by the warm start hold their experts' bytes
    for sl, e in enumerate(st.slot_expert):
        if e >= 0:
            for d, hs, b in zip(slabs.dsts, slabs.hosts, slabs.sizes):
                d[sl * b:(sl + 1) * b].copy_(hs[e * b:(e + 1) * b])
    sync = torch.zeros(8, dtype=torch.int32, device=DEV)
    out = torch.empty(max(mk, 1), dtype=out_dtype, device=DEV)
    tag = f"E{E} S{S} mk{mk} mi{mi} md{md} p{pol} d{decay}"
    installs = 0
    for t in range(steps):
        ids = _ids(rng, E, mk)
        nins = nins_of(st, ids, md, mi, E)
        pairs = policy.manage(st, ids, md, mi, pol, decay)
        step(h, ds, torch.from_numpy(ids).to(DEV), md, mi, pol, decay, out[:max(mk, 1)],
             slabs, sync, chunks, lanes)
        torch.cuda.synchronize()
        compare_state(ds.host(), st, nins, f"{tag} t{t}")
        if mk:
            np.testing.assert_array_equal(out[:mk].cpu().numpy().astype(np.int64),
                                          policy.remap(st.table, ids, np.int64),
                                          err_msg=f"{tag} t{t}: remap")
        slabs.check(pairs, f"{tag} t{t}")
        installs += len(pairs)
        assert counters(sync) == (0, installs), tag
    # every occupied slot holds its expert at the end
    slabs.check([(int(e), s) for s, e in enumerate(ds.slot_expert.cpu().numpy()) if e >= 0],
                tag)


def test_random_cases_vs_oracle(h):
    rng = np.random.default_rng(21)
    for i in range(40):
        E = int(rng.choice([1, 3, 8, 32, 128, 129, 300, 512, 1024, 3000]))
        S = int(rng.integers(1, min(256, 2 * E + 8) + 1))
        mk = int(rng.choice([0, 1, 2, 8, 32, 50, 255, 256, 257, 700]))
        mi = max(0, min(int(rng.choice([0, 1, 4, S, 2 * S])), 1024))
        md = int(rng.choice([-1, 0, 4, 8, E, 10 ** 6]))
        pol = int(rng.integers(0, 2))
        decay = int(rng.choice([0, 1, 3, 64]))
        chunks, lanes = [(16, 64), (1, 1), (3, 5), (148, 2)][i % 4]
        drive(h, E, S, mk, mi, md, pol, decay, steps=10, rng=rng, chunks=chunks, lanes=lanes,
              out_dtype=torch.int64 if i % 2 else torch.int32)


def test_decode_shapes_many_steps(h):
    """E128 top-8, tokens 1 and 4, S 16..256, long enough to churn."""
    rng = np.random.default_rng(5)
    for S in (16, 64, 96, 256):
        for mk in (8, 32):
            for pol in (0, 1):
                drive(h, 128, S, mk, S, min(128, mk), pol, 64, steps=30, rng=rng)


def test_largest_experts_and_slots(h):
    """E at the shared-memory opt-in bound with S = max_inserts = 256."""
    rng = np.random.default_rng(9)
    drive(h, 32768, 256, 300, 256, 10 ** 6, 1, 4, steps=4, rng=rng, sizes=(16,))
    drive(h, 256, 256, 256, 256, 256, 0, 64, steps=6, rng=rng)


def test_equals_two_launch_path_at_qwen_shape(h):
    """expert_cache_step vs expert_cache_manage_remap + expert_cache_gather."""
    from gpu_util import gather, manage
    from synthetic import bytes_per_expert, qwen3_30b_a3b_experts, sticky_zipf_trace
    E, S = 128, 64
    ex = qwen3_30b_a3b_experts(E=E, seed=2)
    names = list(ex)
    sizes = [bytes_per_expert(ex[n]) for n in names]
    srcs = [device_ptr_of_pinned(ex[n]) for n in names]
    one, two = DeviceState(policy.CacheState(E, S)), DeviceState(policy.CacheState(E, S))
    slabs = Slabs.__new__(Slabs)
    slabs.sizes, slabs.srcs = sizes, srcs
    slabs.hosts = [ex[n].view(torch.uint8).reshape(-1) for n in names]
    slabs.dsts = [torch.zeros(S * b, dtype=torch.uint8, device=DEV) for b in sizes]
    dst2 = [torch.zeros(S * b, dtype=torch.uint8, device=DEV) for b in sizes]
    sync = torch.zeros(8, dtype=torch.int32, device=DEV)
    trace = sticky_zipf_trace(3, steps=60, E=E, tokens=4)
    out1 = torch.empty(32, dtype=torch.int32, device=DEV)
    out2 = torch.empty(32, dtype=torch.int32, device=DEV)
    for t in range(len(trace)):
        ids = torch.from_numpy(trace[t]).to(DEV)
        step(h, one, ids, 32, S, 1, 64, out1, slabs, sync)
        manage(h, two, ids, 32, S, 1, 64, out=out2)
        assert gather(h, [(d.data_ptr(), s, b) for d, s, b in zip(dst2, srcs, sizes)],
                      two.miss, two.n_miss) == 0
        if t % 6 == 5:
            torch.cuda.synchronize()
            assert torch.equal(out1, out2), t
            h1, h2 = one.host(), two.host()
            for f in ("table", "map_cold", "slot_expert", "slot_stamp", "routed", "step",
                      "n_miss"):
                np.testing.assert_array_equal(h1[f], h2[f], err_msg=f"t{t} {f}")
    torch.cuda.synchronize()
    for a, b in zip(slabs.dsts, dst2):
        assert torch.equal(a, b)


def test_graph_of_many_steps(h):
    """4096-step-style replay: 200 step nodes in one CUDA graph."""
    from synthetic import sticky_zipf_trace
    E, S, steps = 128, 32, 200
    st = policy.CacheState(E, S)
    ds = DeviceState(st)
    slabs = Slabs(E, S, (4096, 1024, 32), seed=4)
    sync = torch.zeros(8, dtype=torch.int32, device=DEV)
    trace = sticky_zipf_trace(6, steps=steps, E=E)
    ids = torch.from_numpy(trace).to(DEV)
    out = torch.empty_like(ids)
    nm = torch.zeros(steps, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for t in range(steps):
            step(h, ds, ids[t], 8, S, 1, 64, out[t], slabs, sync)
            nm[t:t + 1].copy_(ds.n_miss)
    torch.cuda.synchronize()
    assert int(ds.step.item()) == 0           # capture recorded, did not run
    g.replay()
    torch.cuda.synchronize()
    got_nm = nm.cpu().numpy()
    got_out = out.cpu().numpy()
    for t in range(steps):
        pairs = policy.manage(st, trace[t], 8, S, 1, 64)
        assert got_nm[t] == len(pairs), t
        np.testing.assert_array_equal(got_out[t], policy.remap(st.table, trace[t]))
    compare_state(ds.host(), st, 0, "after graph")
    slabs.check([(int(e), s) for s, e in enumerate(st.slot_expert) if e >= 0], "graph")
    assert counters(sync) == (0, int(got_nm.sum()))


def test_wait_bound_runs_out_and_no_bytes_are_lost(h):
    """1 us wait bound against a slow policy step: waits run out, the result is exact."""
    rng = np.random.default_rng(17)
    E, S, mk = 32768, 256, 2048
    st = policy.CacheState(E, S, miss_cap=S)
    ds = DeviceState(st)
    slabs = Slabs(E, S, (4096, 48), seed=12)
    sync = torch.zeros(8, dtype=torch.int32, device=DEV)
    out = torch.empty(mk, dtype=torch.int32, device=DEV)
    timed_out = installs = 0
    for t in range(4):
        ids = rng.choice(E, size=mk, replace=False).astype(np.int32)
        nins = nins_of(st, ids, 10 ** 6, S, E)
        pairs = policy.manage(st, ids, 10 ** 6, S, 1, 64)
        step(h, ds, torch.from_numpy(ids).to(DEV), 10 ** 6, S, 1, 64, out, slabs, sync,
             wait_us=1)
        torch.cuda.synchronize()
        compare_state(ds.host(), st, nins, f"t{t}")
        np.testing.assert_array_equal(out.cpu().numpy(), policy.remap(st.table, ids))
        slabs.check(pairs, f"t{t}")
        installs += len(pairs)
        timed_out, got_installs = counters(sync)
        assert got_installs == installs
    assert timed_out > 0, "no wait ran out: the bound was not exercised"


def test_one_node_replayed_many_times(h):
    """One captured step node replayed 300 times with new ids each time: every replay must
    elect its own policy CTA and never take an earlier replay's published word."""
    from synthetic import sticky_zipf_trace
    E, S = 128, 16
    st = policy.CacheState(E, S)
    ds = DeviceState(st)
    slabs = Slabs(E, S, (1024, 64), seed=13)
    sync = torch.zeros(8, dtype=torch.int32, device=DEV)
    ids = torch.zeros(8, dtype=torch.int32, device=DEV)
    out = torch.empty(8, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        step(h, ds, ids, 8, S, 0, 0, out, slabs, sync)
    torch.cuda.synchronize()
    trace = sticky_zipf_trace(11, steps=300, E=E)
    installs = 0
    for t in range(len(trace)):
        ids.copy_(torch.from_numpy(trace[t]))
        g.replay()
        nins = nins_of(st, trace[t], 8, S, E)
        pairs = policy.manage(st, trace[t], 8, S, 0, 0)
        installs += len(pairs)
        if pairs or t % 25 == 24:
            torch.cuda.synchronize()
            compare_state(ds.host(), st, nins, f"t{t}")
            np.testing.assert_array_equal(out.cpu().numpy(), policy.remap(st.table, trace[t]))
            slabs.check(pairs, f"t{t}")
    torch.cuda.synchronize()
    assert counters(sync) == (0, installs)


def test_refresh_beyond_step_slots_uses_two_launches(monkeypatch):
    """S > 256: ExpertSlotCache.refresh falls back to manage_remap + gather."""
    from synthetic import qwen3_30b_a3b_experts, sticky_zipf_trace
    from test_cache_gpu import OffloadedLayer, check_slots
    from vllm_expert_cache.cache import ExpertSlotCache
    monkeypatch.setenv("EXPERT_CACHE_POLICY", "lru")
    E, S = 512, 300
    host = qwen3_30b_a3b_experts(E=E, seed=4, hidden=32, inter=16)
    layer = OffloadedLayer(host)
    cache = ExpertSlotCache(layer, list(host), E, S, DEV, required={"w13_weight", "w2_weight"})
    st = policy.CacheState(E, S)
    trace = sticky_zipf_trace(2, steps=60, E=E, k=8, tokens=4)
    for t in range(len(trace)):
        out = cache.refresh(torch.from_numpy(trace[t]).view(4, 8).to(DEV))
        pairs = policy.manage(st, trace[t], 32, S, 0, 64)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().ravel(), policy.remap(st.table, trace[t]))
        check_slots(cache, layer, pairs)
    np.testing.assert_array_equal(cache.slot_expert.cpu().numpy(), st.slot_expert)
    assert cache.step_timeouts() == 0
