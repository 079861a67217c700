"""Next-layer prefetch on a B200: the prefetch step and the pregate top-k against the
oracle, and two chained layers through vLLM's own fused-MoE kernel.

* ``expert_cache_prefetch`` interleaved with ordinary manage steps, both policies: state,
  miss list and n_miss equal the oracle's after every call.
* ``expert_cache_pregate``: per-token top-k ids of x . gate_w equal the oracle's, except
  where two scores are within fp32 summation-order noise of each other.
* Two armed W8A8 int8 layers (vLLM's Triton ``fused_experts``), the second's router on
  ``layer.runner.gate``: with prefetch on, every output equals the stock kernel's bit for
  bit, eagerly and replayed from a captured CUDA graph (the side-stream fork and join are
  recorded in the graph); the prefetch installs experts (never over the previous step's
  working set) and the second layer's own steps install fewer than without it.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from gpu_util import DEV, DeviceState, compare_state, lib, p, stream_ptr
from oracle import policy
from test_generic import Log

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h():
    return lib()


@pytest.mark.parametrize("pol", [0, 1])
def test_prefetch_matches_oracle(h, pol):
    E, S = 40, 9
    st = policy.CacheState(E, S)
    ds = DeviceState(st)
    rng = np.random.default_rng(23 + pol)
    for step in range(120):
        ids = rng.choice(E, int(rng.integers(1, 9)), replace=False).astype(np.int32)
        if step % 5 == 2:
            ids = np.concatenate([ids, [-1, E + 2]]).astype(np.int32)
        uniq = np.unique(ids[(ids >= 0) & (ids < E)])
        md = min(E, ids.size)
        nins = min(S, int(np.count_nonzero(st.table[uniq] < 0)))
        ids_t = torch.from_numpy(ids).to(DEV)
        if rng.random() < 0.5:
            policy.prefetch(st, ids, md, S, pol)
            rc = h.expert_cache_prefetch(p(ids_t), ids.size, E, S, md, S, *ds.ptrs(), pol,
                                         stream_ptr())
            what = "prefetch"
        else:
            policy.manage(st, ids, md, S, pol, 4)
            rc = h.expert_cache_manage(p(ids_t), ids.size, E, S, md, S, *ds.ptrs(), pol, 4,
                                       stream_ptr())
            what = "manage"
        assert rc == 0
        torch.cuda.synchronize()
        compare_state(ds.host(), st, nins, f"step {step} ({what})")
        assert not policy.check_invariants(st)


def _pregate(h, x, w, k):
    out = torch.full((x.size(0) * k,), -9, dtype=torch.int32, device=DEV)
    rc = h.expert_cache_pregate(p(x), x.size(0), x.stride(0), x.size(1), p(w), w.size(0), k,
                                p(out), stream_ptr())
    assert rc == 0
    torch.cuda.synchronize()
    return out.view(x.size(0), k).cpu().numpy()


@pytest.mark.parametrize("T,E,H,k", [(1, 128, 2048, 8), (3, 128, 2048, 8), (8, 64, 4096, 4),
                                     (2, 256, 7168, 8), (5, 8, 64, 8)])
def test_pregate_matches_oracle(h, T, E, H, k):
    g = torch.Generator().manual_seed(T * 1000 + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    got = _pregate(h, x.to(DEV), w.to(DEV), k)
    xf, wf = x.float().numpy(), w.float().numpy()
    want = policy.pregate(xf, wf, k)
    sc = policy.pregate_scores(xf, wf)
    for t in range(T):
        for r in range(k):
            if got[t, r] != want[t, r]:
                # only a near-tie may differ (fp32 accumulation order vs float64)
                gap = abs(sc[t, got[t, r]] - sc[t, want[t, r]])
                assert gap <= 1e-4 * (1 + abs(sc[t, want[t, r]])), (t, r, got[t], want[t])


def test_pregate_ties_nan_and_short_rows(h):
    x = torch.zeros(2, 8, dtype=torch.bfloat16)
    x[0, 0] = 1.0
    w = torch.zeros(4, 8, dtype=torch.bfloat16)
    w[:, 0] = torch.tensor([1.0, 1.0, float("nan"), 2.0])
    got = _pregate(h, x.to(DEV), w.to(DEV), 4)
    assert got[0].tolist() == [3, 0, 1, -1]
    assert got[1].tolist() == [0, 1, 3, -1]
    # padded row stride: ldx = 16 elements, only the first 8 read
    xp = torch.zeros(2, 16, dtype=torch.bfloat16)
    xp[:, :8] = x
    xp[:, 8:] = 100.0
    out = torch.full((8,), -9, dtype=torch.int32, device=DEV)
    xd = xp.to(DEV)
    rc = h.expert_cache_pregate(p(xd), 2, 16, 8, p(w.to(DEV).contiguous()), 4, 4, p(out),
                                stream_ptr())
    assert rc == 0
    torch.cuda.synchronize()
    assert out.view(2, 4).cpu().tolist() == got.tolist()


# --- two chained layers through vLLM's kernel -------------------------------------------

E2, S2, H2, N2, K2 = 16, 8, 256, 128, 4


@pytest.fixture(scope="module")
def vllm_moe():
    fm = pytest.importorskip("vllm.model_executor.layers.fused_moe.fused_moe")
    cfg = pytest.importorskip("vllm.model_executor.layers.fused_moe.config")
    return fm.fused_experts, cfg.int8_w8a8_moe_quant_config


class GatedLayer(torch.nn.Module):
    def __init__(self, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        prm = lambda t: torch.nn.Parameter(t.cuda(), requires_grad=False)  # noqa: E731
        self.w13_weight = prm(torch.randint(-128, 128, (E2, 2 * N2, H2), dtype=torch.int8,
                                            generator=g))
        self.w2_weight = prm(torch.randint(-128, 128, (E2, H2, N2), dtype=torch.int8,
                                           generator=g))
        self.w13_weight_scale = prm(torch.rand(E2, 2 * N2, 1, generator=g) * 1e-3 + 1e-4)
        self.w2_weight_scale = prm(torch.rand(E2, H2, 1, generator=g) * 1e-3 + 1e-4)
        self.global_num_experts = E2
        self.expert_map = None
        gate = torch.randn(E2, H2, generator=g).to(torch.bfloat16).cuda()
        self.runner = SimpleNamespace(gate=SimpleNamespace(weight=gate))


class Int8Method:
    is_monolithic = False

    def __init__(self, layer, fused_experts, make_cfg):
        self._fused, self._make = fused_experts, make_cfg
        self.moe_quant_config = self.get_fused_moe_quant_config(layer)
        self.moe_kernel = SimpleNamespace(
            fused_experts=SimpleNamespace(quant_config=self.moe_quant_config))

    def get_fused_moe_quant_config(self, layer):
        return self._make(layer.w13_weight_scale, layer.w2_weight_scale, None, None,
                          per_act_token_quant=True)

    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None,
              shared_experts_input=None):
        return self._fused(x, layer.w13_weight, layer.w2_weight, topk_weights, topk_ids,
                           quant_config=self.moe_kernel.fused_experts.quant_config,
                           global_num_experts=layer.global_num_experts)


def route(layer, x):
    logits = x.float() @ layer.runner.gate.weight.float().T
    w, ids = torch.topk(torch.softmax(logits, 1), K2, dim=1)
    return w, ids.to(torch.int32)


def build_pair(vllm_moe, monkeypatch, prefetch: bool):
    monkeypatch.setenv("EXPERT_CACHE_SLOTS", str(S2))
    monkeypatch.setenv("EXPERT_CACHE_STATS", "1")
    monkeypatch.setenv("EXPERT_CACHE_PREFETCH", str(K2) if prefetch else "0")
    from vllm_expert_cache.backends import generic
    layers = [GatedLayer(seed=11), GatedLayer(seed=12)]
    methods = [Int8Method(ly, *vllm_moe) for ly in layers]
    stocks = [m.apply for m in methods]
    log = Log()
    for ly, m in zip(layers, methods):
        assert generic.arm(ly, m, log), log.msgs
    if prefetch:
        chain = [(ly, ly._expert_cache) for ly in layers]
        assert generic._link_prefetch(chain, log) == 1
    return layers, methods, stocks


def drive(layers, methods, stocks, steps, seed):
    rng = torch.Generator().manual_seed(seed)
    for step in range(steps):
        x = torch.randn(1, H2, generator=rng).to(torch.bfloat16).cuda()   # 4 ids of 8 slots
        for i, (ly, m, stock) in enumerate(zip(layers, methods, stocks)):
            w, ids = route(ly, x)
            got = m.apply(ly, x, w, ids)
            want = stock(ly, x, w, ids)
            torch.cuda.synchronize()
            assert torch.equal(got, want), f"step {step} layer {i}"


def test_prefetch_keeps_outputs_exact_and_saves_installs(vllm_moe, monkeypatch):
    layers, methods, stocks = build_pair(vllm_moe, monkeypatch, prefetch=True)
    drive(layers, methods, stocks, 30, seed=1)
    b = layers[1]._expert_cache
    on = b.stats()
    assert on["prefetch_installs"] > 0
    assert not layers[1]._expert_cache.pending

    layers0, methods0, stocks0 = build_pair(vllm_moe, monkeypatch, prefetch=False)
    drive(layers0, methods0, stocks0, 30, seed=1)
    off = layers0[1]._expert_cache.stats()
    assert off["prefetch_installs"] == 0
    # the second layer's input is the first's, so the prediction is its true routing up
    # to near-ties: its own steps find the prefetched experts resident
    assert on["installs"] < off["installs"], (on, off)


def test_prefetch_inside_a_captured_graph(vllm_moe, monkeypatch):
    layers, methods, stocks = build_pair(vllm_moe, monkeypatch, prefetch=True)
    drive(layers, methods, stocks, 3, seed=2)          # warm: Triton JIT, events, streams
    x = torch.zeros(1, H2, dtype=torch.bfloat16, device=DEV)
    routes = [[torch.zeros(1, K2, device=DEV), torch.zeros(1, K2, dtype=torch.int32,
                                                           device=DEV)] for _ in layers]
    outs = [None, None]

    def forward():
        for i, (ly, m) in enumerate(zip(layers, methods)):
            outs[i] = m.apply(ly, x, routes[i][0], routes[i][1])

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        forward()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        forward()
    rng = torch.Generator().manual_seed(9)
    for step in range(12):
        xn = torch.randn(1, H2, generator=rng).to(torch.bfloat16).cuda()
        x.copy_(xn)
        for i, ly in enumerate(layers):
            w, ids = route(ly, xn)
            routes[i][0].copy_(w)
            routes[i][1].copy_(ids)
        graph.replay()
        torch.cuda.synchronize()
        for i, ly in enumerate(layers):
            want = stocks[i](ly, xn, routes[i][0], routes[i][1])
            torch.cuda.synchronize()
            assert torch.equal(outs[i], want), f"replay {step} layer {i}"
    assert layers[1]._expert_cache.stats()["prefetch_installs"] > 0
