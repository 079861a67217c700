"""The sm_100a gather kernel through the C-ABI: slot bytes must equal the host bytes.

Sources are pinned host buffers read through their UVA device pointers, as vLLM's expert
offload provides them.  Cases: the reference's six-buffer byte-identity drive
(tests/test_policy.py:234-282 shapes: E512 S257, 819200/409600/51200/640/25600/2560 B),
the Qwen3-30B-A3B W8A8 slab, padded triples, an empty miss list, a slab of a few hundred
MB (64-bit offsets), device-resident sources, and several CTA budgets.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import (DEV, DeviceState, compare_state, device_ptr_of_pinned, gather, lib,
                      manage)
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


def check_slots(dsts, hosts, sizes, pairs):
    for e, sl in pairs:
        for d, hsrc, b in zip(dsts, hosts, sizes):
            got = d[sl * b:(sl + 1) * b].cpu()
            assert torch.equal(got, hsrc[e * b:(e + 1) * b]), f"expert {e} slot {sl} {b}B"


def test_six_buffer_byte_identity_drive(h):
    E, S = 512, 257
    sizes = [819200, 409600, 51200, 640, 25600, 2560]
    hosts = [pinned_random(E * b, i) for i, b in enumerate(sizes)]
    srcs = [device_ptr_of_pinned(x) for x in hosts]
    dsts = [torch.zeros(S * b, dtype=torch.uint8, device=DEV) for b in sizes]
    rng = np.random.default_rng(3)
    st = policy.CacheState.warm(E, S, sorted(rng.choice(E, S, replace=False)), miss_cap=64)
    ds = DeviceState(st)
    rng = np.random.default_rng(11)
    written = {}
    for step in range(40):
        ids = np.concatenate([rng.choice(E, 10, replace=False) for _ in range(5)]).astype(np.int32)
        nins = min(64, int(np.count_nonzero(st.table[np.unique(ids)] < 0)))
        pairs = policy.manage(st, ids, 128, 64, 1, 64)
        manage(h, ds, torch.from_numpy(ids).to(DEV), 128, 64, 1, 64)
        rc = gather(h, [(d.data_ptr(), s, b) for d, s, b in zip(dsts, srcs, sizes)],
                    ds.miss, ds.n_miss)
        assert rc == 0
        torch.cuda.synchronize()
        compare_state(ds.host(), st, nins, f"step {step}")
        check_slots(dsts, hosts, sizes, pairs)
        for e, sl in pairs:
            written[sl] = e
    # every slot filled during the drive still holds its expert's bytes
    se = ds.slot_expert.cpu().numpy()
    for sl, e in written.items():
        if se[sl] == e:
            check_slots(dsts, hosts, sizes, [(e, sl)])


@pytest.mark.parametrize("chunks,lanes", [(16, 64), (1, 1), (3, 5), (148, 2), (64, 64)])
def test_qwen3_w8a8_slab_any_grid(h, chunks, lanes):
    from synthetic import bytes_per_expert, qwen3_30b_a3b_experts
    E, S = 12, 8
    ex = qwen3_30b_a3b_experts(E=E, seed=5)
    names = list(ex)
    sizes = [bytes_per_expert(ex[n]) for n in names]
    hosts = [ex[n].view(torch.uint8).reshape(-1) for n in names]
    srcs = [device_ptr_of_pinned(ex[n]) for n in names]
    dsts = [torch.zeros(S * b, dtype=torch.uint8, device=DEV) for b in sizes]
    miss = torch.tensor([7, 3, 0, 5, 11, 0, 2, 7, 9, 1, 4, 6], dtype=torch.int32, device=DEV)
    n_miss = torch.tensor([6], dtype=torch.int32, device=DEV)
    rc = gather(h, [(d.data_ptr(), s, b) for d, s, b in zip(dsts, srcs, sizes)], miss, n_miss,
                chunks, lanes)
    assert rc == 0
    torch.cuda.synchronize()
    pairs = miss.cpu().numpy().reshape(-1, 2)[:6].tolist()
    check_slots(dsts, hosts, sizes, pairs)
    # slots never named in the miss list stay untouched
    for d, b in zip(dsts, sizes):
        for sl in (2, 4):
            assert int(d[sl * b:(sl + 1) * b].count_nonzero()) == 0


def test_padding_triples_and_empty_list(h):
    E, S, b = 6, 4, 4096
    host = pinned_random(E * b, 9)
    src = device_ptr_of_pinned(host)
    dst = torch.zeros(S * b, dtype=torch.uint8, device=DEV)
    miss = torch.tensor([4, 2, 1, 0], dtype=torch.int32, device=DEV)
    n0 = torch.tensor([0], dtype=torch.int32, device=DEV)
    assert gather(h, [(dst.data_ptr(), src, b)], miss, n0) == 0
    torch.cuda.synchronize()
    assert int(dst.count_nonzero()) == 0
    n2 = torch.tensor([2], dtype=torch.int32, device=DEV)
    assert gather(h, [(dst.data_ptr(), src, b)] * 6, miss, n2) == 0
    torch.cuda.synchronize()
    check_slots([dst], [host], [b], [(4, 2), (1, 0)])


def test_large_slab_64bit_offsets(h):
    """A Mixtral-sized w13 slab (234,881,024 B) at expert index 2: offsets above 2**31."""
    E, S, b = 3, 2, 234_881_024
    host = torch.empty(E * b, dtype=torch.uint8, pin_memory=True)
    host.view(torch.int64)[:] = torch.arange(E * b // 8, dtype=torch.int64)
    src = device_ptr_of_pinned(host)
    dst = torch.zeros(S * b, dtype=torch.uint8, device=DEV)
    miss = torch.tensor([2, 1, 0, 0], dtype=torch.int32, device=DEV)
    n = torch.tensor([2], dtype=torch.int32, device=DEV)
    assert gather(h, [(dst.data_ptr(), src, b)], miss, n) == 0
    torch.cuda.synchronize()
    for e, sl in ((2, 1), (0, 0)):
        want = host[e * b:(e + 1) * b].view(torch.int64)
        got = dst[sl * b:(sl + 1) * b].view(torch.int64).cpu()
        assert torch.equal(got, want)


def test_device_resident_sources(h):
    E, S, b = 10, 5, 48
    src = torch.randint(0, 256, (E * b,), dtype=torch.uint8, device=DEV)
    dst = torch.zeros(S * b, dtype=torch.uint8, device=DEV)
    miss = torch.tensor([9, 4, 0, 0, 3, 1], dtype=torch.int32, device=DEV)
    n = torch.tensor([3], dtype=torch.int32, device=DEV)
    assert gather(h, [(dst.data_ptr(), src.data_ptr(), b)], miss, n, 2, 2) == 0
    torch.cuda.synchronize()
    check_slots([dst], [src.cpu()], [b], [(9, 4), (0, 0), (3, 1)])
