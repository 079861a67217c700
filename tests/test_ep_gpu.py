"""Expert-parallel composition on a B200: ``expert_cache_manage_ep`` against the oracle,
and an EP layer served through vLLM's own fused-MoE kernel with the composed map.

The kernel drive runs linear and round-robin placements (vLLM's two, expert_map_manager.py
:22-113) and a map with corrupt entries, under both policies.  Routing carries padding,
out-of-range ids and other ranks' experts.  After every step the state, the miss list and
the composed global id -> slot map must equal the oracle's.

The layer test arms a stand-in W8A8 int8 method whose ``apply`` is vLLM's Triton
``fused_experts`` with ``expert_map=layer.expert_map``, rank 0 of 2 (round-robin).  The
cached step, with slot weights and the composed map bound, must equal the stock call on
the full local weights and vLLM's own map, bit for bit.
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


def expert_map(Eg: int, ep: int, rank: int, kind: str) -> np.ndarray:
    El = Eg // ep
    m = np.full(Eg, -1, dtype=np.int32)
    if kind == "round_robin":
        g = np.arange(rank, Eg, ep)
    else:
        g = np.arange(rank * El, (rank + 1) * El)
    m[g] = np.arange(g.size, dtype=np.int32)
    if kind == "corrupt":                   # entries naming no local expert count as -1
        m[(rank * El + El) % Eg] = El + 5
        m[(rank * El + El + 1) % Eg] = 1 << 30
    return m


@pytest.mark.parametrize("kind", ["linear", "round_robin", "corrupt"])
@pytest.mark.parametrize("pol", [0, 1])
def test_manage_ep_matches_oracle(h, kind, pol):
    Eg, ep, rank, S = 64, 4, 1, 6
    El = Eg // ep
    emap_np = expert_map(Eg, ep, rank, kind)
    emap = torch.from_numpy(emap_np).to(DEV)
    st = policy.CacheState(El, S)
    ds = DeviceState(st)
    rng = np.random.default_rng(17 + pol)
    local_ids = np.flatnonzero((emap_np >= 0) & (emap_np < El))
    for step in range(80):
        tokens = int(rng.integers(1, 3))
        rows = []
        for _ in range(tokens):
            # bias towards this rank's experts so the slots churn
            pick = rng.choice(local_ids, 2, replace=False).tolist()
            pick += rng.choice(Eg, 2, replace=False).tolist()
            rows += pick
        if step % 7 == 3:
            rows += [-1, Eg + 3]                 # padding and an id outside the map
        ids = np.asarray(rows, dtype=np.int32)
        loc = policy.local_ids(ids, emap_np)
        uniq = np.unique(loc[(loc >= 0) & (loc < El)])
        md = min(El, ids.size)
        nins = 0 if uniq.size > md else min(S, int(np.count_nonzero(st.table[uniq] < 0)))
        _, want_map = policy.manage_ep(st, ids, emap_np, md, S, pol, 8)
        ids_t = torch.from_numpy(ids).to(DEV)
        out = torch.full((Eg,), -7, dtype=torch.int32, device=DEV)
        rc = h.expert_cache_manage_ep(p(ids_t), ids.size, p(emap), Eg, El, S, md, S,
                                      *ds.ptrs(), pol, 8, p(out), stream_ptr())
        assert rc == 0
        torch.cuda.synchronize()
        compare_state(ds.host(), st, nins, f"{kind} step {step}")
        np.testing.assert_array_equal(out.cpu().numpy(), want_map,
                                      err_msg=f"{kind} step {step}: composed map")
        assert not policy.check_invariants(st)


def test_manage_ep_empty_step_still_writes_the_map(h):
    Eg, El, S = 16, 8, 4
    emap_np = expert_map(Eg, 2, 0, "linear")
    st = policy.CacheState.warm(El, S, [1, 3, 5, 6])
    ds = DeviceState(st)
    ids_t = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.full((Eg,), -7, dtype=torch.int32, device=DEV)
    rc = h.expert_cache_manage_ep(p(ids_t), 0, p(torch.from_numpy(emap_np).to(DEV)), Eg,
                                  El, S, 0, S, *ds.ptrs(), 0, 0, p(out), stream_ptr())
    assert rc == 0
    torch.cuda.synchronize()
    _, want = policy.manage_ep(st, np.zeros(0, np.int32), emap_np, 0, S, 0, 0)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    assert int(ds.step.item()) == 1


# --- an EP layer through vLLM's Triton fused_experts ------------------------------------

EG, EL, S_L, H, N, K = 24, 12, 6, 256, 128, 4


@pytest.fixture(scope="module")
def vllm_moe():
    fm = pytest.importorskip("vllm.model_executor.layers.fused_moe.fused_moe")
    cfg = pytest.importorskip("vllm.model_executor.layers.fused_moe.config")
    return fm.fused_experts, cfg.int8_w8a8_moe_quant_config


class EPLayer(torch.nn.Module):
    """Rank 0 of 2, round-robin: global expert 2j is local expert j."""

    def __init__(self, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        prm = lambda t: torch.nn.Parameter(t.cuda(), requires_grad=False)  # noqa: E731
        self.w13_weight = prm(torch.randint(-128, 128, (EL, 2 * N, H), dtype=torch.int8,
                                            generator=g))
        self.w2_weight = prm(torch.randint(-128, 128, (EL, H, N), dtype=torch.int8,
                                           generator=g))
        self.w13_weight_scale = prm(torch.rand(EL, 2 * N, 1, generator=g) * 1e-3 + 1e-4)
        self.w2_weight_scale = prm(torch.rand(EL, H, 1, generator=g) * 1e-3 + 1e-4)
        self.register_buffer("_expert_map",
                             torch.from_numpy(expert_map(EG, 2, 0, "round_robin")).cuda())
        self.global_num_experts = EG
        self.use_ep = True

    @property
    def expert_map(self):
        return self._expert_map


class EPInt8Method:
    is_monolithic = False

    def __init__(self, layer, fused_experts, make_cfg):
        self._fused, self._make = fused_experts, make_cfg
        self.moe_quant_config = self.get_fused_moe_quant_config(layer)
        self.moe_kernel = SimpleNamespace(
            fused_experts=SimpleNamespace(quant_config=self.moe_quant_config),
            prepare_finalize=SimpleNamespace(
                activation_format=SimpleNamespace(name="Standard")),
            supports_expert_map=lambda: True)

    def get_fused_moe_quant_config(self, layer):
        return self._make(layer.w13_weight_scale, layer.w2_weight_scale, None, None,
                          per_act_token_quant=True)

    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None,
              shared_experts_input=None):
        return self._fused(x, layer.w13_weight, layer.w2_weight, topk_weights, topk_ids,
                           quant_config=self.moe_kernel.fused_experts.quant_config,
                           global_num_experts=layer.global_num_experts,
                           expert_map=layer.expert_map)


def test_ep_layer_equals_stock_bit_exact(vllm_moe, monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_SLOTS", str(S_L))
    monkeypatch.setenv("EXPERT_CACHE_EP", "1")
    from vllm_expert_cache.backends import generic
    layer = EPLayer(seed=3)
    m = EPInt8Method(layer, *vllm_moe)
    stock = m.apply
    log = Log()
    assert generic.arm(layer, m, log), log.msgs
    full_map = layer._expert_map
    rng = np.random.default_rng(5)
    for step in range(8):
        tokens = 1                               # 4 ids <= 6 slots: the cached path
        ids = torch.from_numpy(np.stack([rng.choice(EG, K, replace=False)
                                         for _ in range(tokens)]).astype(np.int32)).cuda()
        w = torch.softmax(torch.from_numpy(rng.standard_normal((tokens, K))).float(),
                          1).cuda()
        x = (torch.from_numpy(rng.standard_normal((tokens, H))).float() * 0.5).to(
            torch.bfloat16).cuda()
        got = m.apply(layer, x, w, ids)
        want = stock(layer, x, w, ids)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"step {step}"
        assert layer._expert_map is full_map          # vLLM's map is back after the step
    assert int(layer._expert_cache.step.item()) == 8
