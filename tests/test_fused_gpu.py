"""expert_cache_fused on the GPU: the LRU manage step plus both moe_align_block_size
outputs in one launch, against the CPU oracle (bit-exact, every step) and, order-
insensitively, against vLLM's own moe_align_block_size run on the updated table."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gpu_util import DEV, DeviceState, compare_state, lib, p, stream_ptr
from oracle import policy

pytestmark = pytest.mark.gpu


def bind(h):
    P, I = ctypes.c_void_p, ctypes.c_int
    fn = h.expert_cache_fused
    fn.restype = I
    fn.argtypes = [P] + [I] * 5 + [P] * 8 + [I, I, I] + [P] * 6 + [P]
    return fn


class AlignBufs:
    def __init__(self, mk, E, bs):
        self.L, self.NB = policy.align_lengths(mk, E, bs)
        z = lambda n: torch.full((n,), -99, dtype=torch.int32, device=DEV)  # noqa: E731
        self.sh, self.eh, self.nh = z(self.L), z(self.NB), z(1)
        self.sc, self.ec, self.nc = z(self.L), z(self.NB), z(1)

    def ptrs(self):
        return [p(self.sh), p(self.eh), p(self.nh), p(self.sc), p(self.ec), p(self.nc)]

    def host(self):
        return [t.cpu().numpy() for t in (self.sh, self.eh, self.nh, self.sc, self.ec, self.nc)]


def fused(fn, ds, ids, md, mi, bs, bufs):
    rc = fn(p(ids), ids.numel(), ds.E, ds.S, md, mi, *ds.ptrs(), bs, bufs.L, bufs.NB,
            *bufs.ptrs(), stream_ptr())
    assert rc == 0, f"expert_cache_fused rc={rc}"


def nins_of(st, ids, md, mi):
    valid = np.unique(ids[(ids >= 0) & (ids < st.E)])
    if len(valid) > md:
        return 0
    return min(int(np.count_nonzero(st.table[valid] < 0)), mi)


def run(fn, E, S, mk, bs, md, mi, steps, rng):
    cap = max(mi, 1)
    st = (policy.CacheState.warm(E, S, rng.choice(E, size=S, replace=False), miss_cap=cap)
          if S <= E else policy.CacheState(E, S, miss_cap=cap))
    ds = DeviceState(st)
    bufs = AlignBufs(mk, E, bs)
    tag = f"E{E} S{S} mk{mk} bs{bs} md{md} mi{mi}"
    for t in range(steps):
        ids = np.where(rng.random(mk) < 0.7, rng.integers(0, max(1, E // 3), size=mk),
                       rng.integers(-1, E + 1, size=mk)).astype(np.int32)
        nins = nins_of(st, ids, md, mi)
        policy.manage(st, ids, md, mi, 0, 0)
        fused(fn, ds, torch.from_numpy(ids).to(DEV), md, mi, bs, bufs)
        compare_state(ds.host(), st, nins, f"{tag} t{t}")
        want = policy.align(st.table, ids, S, bs, bufs.L, bufs.NB)
        for name, g, w in zip(("sorted_hot", "eids_hot", "npad_hot", "sorted_cold",
                               "eids_cold", "npad_cold"), bufs.host(), want):
            np.testing.assert_array_equal(g, w, err_msg=f"{tag} t{t} {name}")
    return st, ds, bufs


def test_fused_matches_oracle_random():
    fn = bind(lib())
    rng = np.random.default_rng(21)
    for E, S, mk, bs in [(128, 64, 8, 16), (128, 64, 32, 64), (128, 16, 8, 1),
                         (512, 257, 50, 16), (64, 16, 40, 4), (1024, 1024, 700, 16),
                         (1024, 300, 257, 128), (32, 8, 10, 3), (1, 1, 4, 2)]:
        for md, mi in ((10 ** 6, S), (8, 4)):
            run(fn, E, S, mk, bs, md, min(mi, 1024), steps=6, rng=rng)


def test_fused_decode_shape_many_steps():
    fn = bind(lib())
    rng = np.random.default_rng(5)
    run(fn, 128, 64, 8, 16, 8, 64, steps=150, rng=rng)


def _blocks(sorted_ids, eids, npad, bs, mk):
    out = []
    for b in range(int(npad) // bs):
        toks = tuple(sorted(int(x) for x in sorted_ids[b * bs:(b + 1) * bs] if x < mk))
        out.append((int(eids[b]), toks))
    return sorted(out)


def test_fused_align_agrees_with_vllm():
    """The hot side is vLLM's moe_align_block_size with expert_map = the updated table, the
    cold side with expert_map = map_cold (invalid experts ignored); compared per block."""
    try:
        from vllm.model_executor.layers.fused_moe.moe_align_block_size import (
            moe_align_block_size)
    except Exception as e:  # vLLM is part of this image; say so if it cannot load
        pytest.skip(f"vLLM's moe_align_block_size unavailable: {e!r}")
    fn = bind(lib())
    rng = np.random.default_rng(8)
    for E, S, mk, bs in [(128, 64, 8, 16), (128, 64, 32, 16), (256, 96, 64, 64)]:
        st, ds, bufs = run(fn, E, S, mk, bs, 10 ** 6, S, steps=3, rng=rng)
        ids = torch.from_numpy(rng.integers(0, E, size=mk).astype(np.int32)).to(DEV)
        fused(fn, ds, ids, 10 ** 6, S, bs, bufs)
        torch.cuda.synchronize()
        sh, eh, nh, sc, ec, nc = bufs.host()
        for mapping, (s_, e_, n_) in ((ds.table, (sh, eh, nh)), (ds.map_cold, (sc, ec, nc))):
            v_sorted, v_eids, v_n = moe_align_block_size(
                ids.view(-1, 1), bs, E, expert_map=mapping, ignore_invalid_experts=True)
            v_n = int(v_n.item())
            assert int(n_[0]) == v_n
            assert _blocks(s_, e_, n_[0], bs, mk) == _blocks(
                v_sorted.cpu().numpy(), v_eids.cpu().numpy(), v_n, bs, mk)
