"""ExpertSlotCache.refresh -- the step vLLM's wrapped ``apply`` runs -- end to end on the GPU.

The owner is a stand-in MoE layer whose expert tensors are CUDA views of pinned host
memory (what ``--cpu-offload-params experts`` leaves behind).  After every step: the
returned slot ids equal the oracle's remap, the state equals the oracle's, and every
installed slot holds exactly its expert's bytes.  Also: a CUDA-graph capture of the whole
step replayed over a trace, int64 routing ids, and the W8A8 Qwen3-30B-A3B layer shape.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import DEV, uva_view
from oracle import policy
from vllm_expert_cache.cache import ExpertSlotCache
from synthetic import qwen3_30b_a3b_experts, sticky_zipf_trace

pytestmark = pytest.mark.gpu


class OffloadedLayer(torch.nn.Module):
    def __init__(self, host: dict):
        super().__init__()
        self.host = host
        for name, t in host.items():
            self.register_parameter(name, torch.nn.Parameter(uva_view(t), requires_grad=False))


def make_cache(monkeypatch, E, S, policy_name="lfu", **shape):
    monkeypatch.setenv("EXPERT_CACHE_POLICY", policy_name)
    host = qwen3_30b_a3b_experts(E=E, seed=1, **shape)
    layer = OffloadedLayer(host)
    cache = ExpertSlotCache(layer, list(host), E, S, DEV, required={"w13_weight", "w2_weight"})
    return layer, cache


def check_slots(cache, layer, pairs):
    for name in cache.names:
        host = layer.host[name]
        for e, sl in pairs:
            assert torch.equal(cache.slots[name][sl].cpu(), host[e]), (name, e, sl)


@pytest.mark.parametrize("pol,code", [("lfu", 1), ("lru", 0)])
def test_refresh_matches_oracle_every_step(monkeypatch, pol, code):
    E, S = 32, 12
    layer, cache = make_cache(monkeypatch, E, S, pol, hidden=64, inter=32)
    st = policy.CacheState(E, S)
    trace = sticky_zipf_trace(4, steps=120, E=E, k=4, tokens=2)
    for t in range(len(trace)):
        ids = torch.from_numpy(trace[t].reshape(2, 4)).to(DEV)
        out = cache.refresh(ids)
        pairs = policy.manage(st, trace[t], min(E, 8), S, code, 64)
        torch.cuda.synchronize()
        assert out.dtype == ids.dtype and out.shape == ids.shape
        np.testing.assert_array_equal(out.cpu().numpy().ravel(),
                                      policy.remap(st.table, trace[t]))
        for f in ("table", "map_cold", "slot_expert", "slot_stamp", "step", "n_miss"):
            np.testing.assert_array_equal(getattr(cache, f).cpu().numpy(), getattr(st, f), f)
        check_slots(cache, layer, pairs)
    # at the end every occupied slot holds its expert
    se = cache.slot_expert.cpu().numpy()
    check_slots(cache, layer, [(int(e), s) for s, e in enumerate(se) if e >= 0])


def test_int64_routing_ids(monkeypatch):
    E, S = 16, 8
    layer, cache = make_cache(monkeypatch, E, S, hidden=32, inter=16)
    st = policy.CacheState(E, S)
    ids = torch.tensor([[3, 9, 1, 12]], dtype=torch.int64, device=DEV)
    out = cache.refresh(ids)
    policy.manage(st, ids.cpu().numpy().ravel(), 4, S, 1, 64)
    assert out.dtype == torch.int64
    np.testing.assert_array_equal(out.cpu().numpy().ravel(),
                                  policy.remap(st.table, ids.cpu().numpy().ravel()))
    assert torch.equal(cache.remap(ids), out)     # the torch remap agrees


def test_graph_captured_step(monkeypatch):
    E, S = 64, 16
    layer, cache = make_cache(monkeypatch, E, S, hidden=128, inter=64)
    st = policy.CacheState(E, S)
    static_ids = torch.zeros((1, 8), dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        static_out = cache.refresh(static_ids)
    torch.cuda.synchronize()
    assert int(cache.step.item()) == 0          # capture recorded, did not run
    trace = sticky_zipf_trace(8, steps=150, E=E)
    for t in range(len(trace)):
        static_ids.copy_(torch.from_numpy(trace[t]).view(1, 8))
        g.replay()
        pairs = policy.manage(st, trace[t], 8, S, 1, 64)
        if t % 10 == 9 or pairs:
            torch.cuda.synchronize()
            np.testing.assert_array_equal(static_out.cpu().numpy().ravel(),
                                          policy.remap(st.table, trace[t]))
            np.testing.assert_array_equal(cache.table.cpu().numpy(), st.table)
            check_slots(cache, layer, pairs)


def test_qwen3_w8a8_layer_shape(monkeypatch):
    """Full W8A8 expert slabs (4,732,928 B per expert), E128 S64, decode steps of 1 and 4
    tokens."""
    E, S = 128, 64
    layer, cache = make_cache(monkeypatch, E, S)
    assert sum(cache.slots[n][0].numel() * cache.slots[n].element_size()
               for n in cache.names) == 4_732_928
    st = policy.CacheState(E, S)
    trace = sticky_zipf_trace(1, steps=24, E=E, tokens=4)
    for t in range(len(trace)):
        rows = 1 if t % 2 else 4
        ids_np = trace[t][: rows * 8]
        out = cache.refresh(torch.from_numpy(ids_np).view(rows, 8).to(DEV))
        pairs = policy.manage(st, ids_np, min(E, rows * 8), S, 1, 64)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().ravel(), policy.remap(st.table, ids_np))
        check_slots(cache, layer, pairs[:3])
    np.testing.assert_array_equal(cache.slot_expert.cpu().numpy(), st.slot_expert)
