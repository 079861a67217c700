"""The allocation-free manage entry point against the existing one (GPU).

``expert_cache_manage_remap_noalloc`` serves callers that cannot call cudaMalloc -- a
serving engine that already gave all free HBM to its own pool, a host runtime whose device
memory only comes from a foreign allocator, a loop that must not take cudaMalloc's
implicit device-wide synchronisation.  It takes no ``routed`` scratch array and writes
those flags into an array the library owns.  Its results must be exactly those of
``expert_cache_manage_remap`` given the same inputs, call after call (the same bit-exact
tolerance as every other test of this integer path).

This file is named to be collected last, so a run that stops at the first failure has
already run every other test; it passes on its own in a fresh process as well.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gpu_util import DEV, DeviceState, lib, manage, p, stream_ptr
from oracle import policy

pytestmark = pytest.mark.gpu

NOALLOC_MAX_EXPERTS = 8192     # EXPERT_CACHE_NOALLOC_MAX_EXPERTS in include/expert_cache.h


def bind_noalloc(h):
    P, I = ctypes.c_void_p, ctypes.c_int
    fn = h.expert_cache_manage_remap_noalloc
    fn.restype = I
    fn.argtypes = [P] + [I] * 5 + [P] * 7 + [I, I, P, I, P]
    return fn


def call_noalloc(fn, ds, ids, md, mi, pol, decay, out):
    return fn(p(ids), ids.numel(), ds.E, ds.S, md, mi, p(ds.table), p(ds.map_cold),
              p(ds.slot_expert), p(ds.slot_stamp), p(ds.step), p(ds.miss), p(ds.n_miss),
              pol, decay, p(out), out.element_size(), stream_ptr())


@pytest.mark.parametrize("E,S,pol,out_dtype", [(128, 16, 1, torch.int32),
                                               (512, 64, 0, torch.int64),
                                               (NOALLOC_MAX_EXPERTS, 1024, 1, torch.int32)])
def test_noalloc_matches_existing_entry_point_two_calls(E, S, pol, out_dtype):
    h = lib()
    noalloc = bind_noalloc(h)
    rng = np.random.default_rng(E + S)
    start = policy.CacheState.warm(E, S, rng.choice(E, size=S, replace=False), miss_cap=S)
    a, b = DeviceState(start), DeviceState(start)   # existing / allocation-free
    mk, md, mi = 64, 10 ** 6, S
    out_a = torch.full((mk,), -7, dtype=out_dtype, device=DEV)
    out_b = torch.full((mk,), -9, dtype=out_dtype, device=DEV)
    for call in range(2):
        ids = torch.from_numpy(rng.integers(-1, E, size=mk).astype(np.int32)).to(DEV)
        manage(h, a, ids, md, mi, pol, 64, out=out_a)
        assert call_noalloc(noalloc, b, ids, md, mi, pol, 64, out_b) == 0
        torch.cuda.synchronize()
        for f in ("table", "map_cold", "slot_expert", "slot_stamp", "step", "n_miss"):
            assert torch.equal(getattr(a, f), getattr(b, f)), (call, f)
        n = int(a.n_miss.item())
        assert n > 0 or call == 1
        assert torch.equal(a.miss[:2 * n], b.miss[:2 * n]), call
        assert torch.equal(out_a, out_b), call


def test_noalloc_refuses_more_experts_than_its_array():
    h = lib()
    noalloc = bind_noalloc(h)
    null = ctypes.c_void_p(0)
    rc = noalloc(null, 8, NOALLOC_MAX_EXPERTS + 1, 64, 8, 64, *([null] * 7), 1, 64, null, 4,
                 null)
    assert rc == -2
    rc = noalloc(null, 8, 0, 64, 8, 64, *([null] * 7), 1, 64, null, 4, null)
    assert rc == -1
