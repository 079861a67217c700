"""Arming logic (backends/generic.py) on CPU stand-ins for vLLM's classes.

The same checks as the reference's tests/test_generic.py:142-352: which per-expert tensors
are discovered, that the rebuilt quant config is slot-bound, wide steps read through, the
layer is restored exactly, vLLM's keyword call is accepted, and each refusal fires with a
reason.  ``cache.refresh`` is replaced by the identity, so no kernel runs.
"""

from __future__ import annotations

from dataclasses import dataclass

import pytest
import torch

from vllm_expert_cache.backends import generic

E, S = 16, 4
H, N = 8, 12


class Log:
    def __init__(self):
        self.msgs = []

    def _rec(self, fmt, *a):
        self.msgs.append(fmt % a if a else fmt)

    warning = info = debug = _rec

    def said(self, needle):
        return any(needle in m for m in self.msgs)


@dataclass
class Desc:
    scale: torch.Tensor | None = None
    alpha_or_gscale: torch.Tensor | None = None
    zp: torch.Tensor | None = None
    bias: torch.Tensor | None = None


@dataclass
class QuantConfig:
    _a1: Desc
    _a2: Desc
    _w1: Desc
    _w2: Desc


class FusedExperts:
    def __init__(self, cfg):
        self.quant_config = cfg


class MoEKernel:
    def __init__(self, cfg):
        self.fused_experts = FusedExperts(cfg)


class RoutedExperts(torch.nn.Module):
    """Per-expert tensors as registered Parameters, like vLLM's MoE layer."""

    def __init__(self, extra=(), n_experts=E):
        super().__init__()
        p = lambda t: torch.nn.Parameter(t, requires_grad=False)  # noqa: E731
        self.w13_weight = p(torch.randn(n_experts, N, H))
        self.w2_weight = p(torch.randn(n_experts, H, N // 2))
        for name, shape in extra:
            setattr(self, name, p(torch.randn(*shape)))
        self.global_num_experts = n_experts
        if not isinstance(getattr(type(self), "expert_map", None), property):
            self.expert_map = None


class QuantMethod:
    """A FusedMoEMethodBase stand-in whose config factory reads ``reads`` off the layer."""

    is_monolithic = False

    def __init__(self, layer, reads=(), hidden=None):
        self.reads = list(reads)
        self.hidden = hidden      # a per-expert tensor the factory returns from nowhere
        self.moe_quant_config = self._cfg(layer)
        self.moe_kernel = MoEKernel(self.moe_quant_config)
        self.seen = None

    def _cfg(self, layer):
        got = [getattr(layer, n) for n in self.reads]
        w1 = Desc(scale=got[0] if len(got) > 0 else None, zp=got[2] if len(got) > 2 else None)
        w2 = Desc(scale=got[1] if len(got) > 1 else None, zp=got[3] if len(got) > 3 else None)
        if self.hidden is not None:
            w1.bias = self.hidden
        return QuantConfig(Desc(), Desc(), w1, w2)

    def get_fused_moe_quant_config(self, layer):
        return self._cfg(layer)

    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None,
              shared_experts_input=None):
        self.seen = dict(w13=layer.w13_weight, w2=layer.w2_weight,
                         cfg=self.moe_kernel.fused_experts.quant_config,
                         ids=topk_ids.clone(), gne=layer.global_num_experts)
        return torch.zeros(1)


@pytest.fixture(autouse=True)
def _slots(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_SLOTS", str(S))


def arm(layer, method):
    log = Log()
    return generic.arm(layer, method, log), log


SCALES = [("w13_weight_scale", (E, N, 1)), ("w2_weight_scale", (E, H, 1))]


def test_unquantized_mirrors_two_weights():
    layer = RoutedExperts()
    ok, _ = arm(layer, QuantMethod(layer))
    assert ok
    assert set(layer._expert_cache.names) == {"w13_weight", "w2_weight"}


def test_int8_like_mirrors_weights_and_scales():
    layer = RoutedExperts(SCALES)
    ok, _ = arm(layer, QuantMethod(layer, reads=["w13_weight_scale", "w2_weight_scale"]))
    assert ok
    assert set(layer._expert_cache.names) == {"w13_weight", "w2_weight",
                                              "w13_weight_scale", "w2_weight_scale"}


def test_wna16_like_six_tensors():
    extra = SCALES + [("w13_weight_zero_point", (E, N, 1)), ("w2_weight_zero_point", (E, H, 1))]
    layer = RoutedExperts(extra)
    ok, _ = arm(layer, QuantMethod(layer, reads=[n for n, _ in extra]))
    assert ok
    assert len(layer._expert_cache.names) == 6


def test_eight_tensors_split_across_gather_launches():
    extra = SCALES + [(f"aux{i}", (E, 4, 4)) for i in range(4)]
    layer = RoutedExperts(extra)
    ok, _ = arm(layer, QuantMethod(layer, reads=["w13_weight_scale", "w2_weight_scale"]))
    assert ok
    assert len(layer._expert_cache.names) == 8


def test_packed_weights_with_alias():
    layer = RoutedExperts()
    for base in ("w13", "w2"):
        t = getattr(layer, f"{base}_weight")
        del layer._parameters[f"{base}_weight"]
        layer.register_parameter(f"{base}_weight_packed", t)
        setattr(layer, f"{base}_weight", t)        # bare attribute alias, same storage
    m = QuantMethod(layer)
    ok, log = arm(layer, m)
    assert ok, log.msgs
    cache = layer._expert_cache
    assert len(cache.slots) == 2
    assert set(cache.bound) == {"w13_weight", "w13_weight_packed", "w2_weight",
                                "w2_weight_packed"}
    assert cache.bound["w13_weight"].data_ptr() == cache.bound["w13_weight_packed"].data_ptr()
    cache.refresh = lambda ids: ids.clone()
    m.apply(layer, torch.randn(1, H), torch.ones(1, 2), torch.zeros(1, 2, dtype=torch.int32))
    assert m.seen["w13"].data_ptr() == cache.slots["w13_weight_packed"].data_ptr()
    assert layer.w13_weight.data_ptr() == layer.w13_weight_packed.data_ptr()


def test_wide_step_reads_through():
    layer = RoutedExperts(SCALES)
    m = QuantMethod(layer, reads=["w13_weight_scale", "w2_weight_scale"])
    assert arm(layer, m)[0]
    layer._expert_cache.refresh = lambda ids: pytest.fail("wide step must not refresh")
    m.apply(layer, torch.randn(1, H), torch.ones(1, S + 1),
            torch.zeros(1, S + 1, dtype=torch.int32))
    assert m.seen["cfg"]._w1.scale.size(0) == E
    assert m.seen["gne"] == E
    assert m.seen["w13"].data_ptr() == layer.w13_weight.data_ptr()


def test_slot_binding_reaches_the_config():
    layer = RoutedExperts(SCALES)
    m = QuantMethod(layer, reads=["w13_weight_scale", "w2_weight_scale"])
    assert arm(layer, m)[0]
    cache = layer._expert_cache
    cache.refresh = lambda ids: ids.clone() + 100
    m.apply(layer, torch.randn(1, H), torch.ones(1, 2), torch.zeros(1, 2, dtype=torch.int32))
    assert m.seen["w13"].data_ptr() == cache.slots["w13_weight"].data_ptr()
    assert m.seen["cfg"]._w1.scale.size(0) == S
    assert m.seen["gne"] == S
    assert (m.seen["ids"] == 100).all()      # apply saw the slot-space ids


def test_apply_accepts_keyword_call():
    layer = RoutedExperts()
    m = QuantMethod(layer)
    assert arm(layer, m)[0]
    layer._expert_cache.refresh = lambda ids: ids.clone()
    m.apply(layer=layer, x=torch.randn(1, H), topk_weights=torch.ones(1, 2),
            topk_ids=torch.zeros(1, 2, dtype=torch.int32), shared_experts=None,
            shared_experts_input=None)
    assert m.seen is not None


def test_layer_is_restored():
    layer = RoutedExperts(SCALES)
    m = QuantMethod(layer, reads=["w13_weight_scale", "w2_weight_scale"])
    names = ("w13_weight", "w2_weight", "w13_weight_scale", "w2_weight_scale")
    before = {n: getattr(layer, n).data_ptr() for n in names}
    assert arm(layer, m)[0]
    layer._expert_cache.refresh = lambda ids: ids.clone()
    m.apply(layer, torch.randn(1, H), torch.ones(1, 2), torch.zeros(1, 2, dtype=torch.int32))
    assert {n: getattr(layer, n).data_ptr() for n in names} == before
    assert layer.global_num_experts == E
    assert m.moe_kernel.fused_experts.quant_config._w1.scale.size(0) == E
    assert isinstance(layer._parameters["w13_weight"], torch.nn.Parameter)


class FailingMethod(QuantMethod):
    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None,
              shared_experts_input=None):
        super().apply(layer, x, topk_weights, topk_ids)
        raise RuntimeError("stock kernel failed")


def test_restored_even_when_apply_raises():
    layer = RoutedExperts(SCALES)
    m = FailingMethod(layer, reads=["w13_weight_scale", "w2_weight_scale"])
    ptr = layer.w13_weight.data_ptr()
    assert arm(layer, m)[0]
    layer._expert_cache.refresh = lambda ids: ids.clone()
    with pytest.raises(RuntimeError, match="stock kernel failed"):
        m.apply(layer, torch.randn(1, H), torch.ones(1, 2),
                torch.zeros(1, 2, dtype=torch.int32))
    assert m.seen["w13"].data_ptr() == layer._expert_cache.slots["w13_weight"].data_ptr()
    assert layer.w13_weight.data_ptr() == ptr
    assert layer.global_num_experts == E
    assert m.moe_kernel.fused_experts.quant_config._w1.scale.size(0) == E


def test_hidden_per_expert_tensor_is_refused():
    layer = RoutedExperts()
    ok, log = arm(layer, QuantMethod(layer, hidden=torch.randn(E, N)))
    assert not ok
    assert log.said("stayed bound to full") and log.said("_w1.bias")


def test_monolithic_is_refused():
    layer = RoutedExperts()
    m = QuantMethod(layer)
    m.is_monolithic = True
    ok, log = arm(layer, m)
    assert not ok and log.said("monolithic")


def test_missing_moe_kernel_is_refused():
    layer = RoutedExperts()
    m = QuantMethod(layer)
    m.moe_kernel = None
    ok, log = arm(layer, m)
    assert not ok and log.said("no moe_kernel")


def test_expert_parallel_is_refused():
    layer = RoutedExperts()
    layer.expert_map = torch.arange(E)
    ok, log = arm(layer, QuantMethod(layer))
    assert not ok and log.said("expert parallelism")


def test_ragged_auxiliary_is_caught_by_the_leak_check():
    layer = RoutedExperts([("w13_weight_scale", (E, 3))])        # 12 bytes per expert
    ok, log = arm(layer, QuantMethod(layer, reads=["w13_weight_scale"]))
    assert not ok
    assert log.said("stayed bound to full") and log.said("w13_weight_scale")


def test_ragged_weight_is_refused():
    layer = RoutedExperts()
    layer.w13_weight = torch.nn.Parameter(torch.randn(E, 3), requires_grad=False)
    ok, log = arm(layer, QuantMethod(layer))
    assert not ok
    assert log.said("multiple of 16") and log.said("w13_weight")


def test_nothing_to_cache(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_SLOTS", str(E))
    layer = RoutedExperts()
    assert not arm(layer, QuantMethod(layer))[0]


def test_unrecognised_weight_names_are_reported():
    layer = RoutedExperts()
    layer.register_parameter("w13_qweight_x", layer._parameters.pop("w13_weight"))
    ok, log = arm(layer, QuantMethod.__new__(QuantMethod))
    assert not ok and log.said("no recognised expert weight pair")


def test_debug_trace_logs_the_path(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_DEBUG", "2")
    layer = RoutedExperts()
    m = QuantMethod(layer)
    ok, log = arm(layer, m)
    assert ok
    layer._expert_cache.refresh = lambda ids: ids.clone()
    for n in (2, S + 1, 2):
        m.apply(layer, torch.randn(1, H), torch.ones(1, n), torch.zeros(1, n, dtype=torch.int32))
    traced = [x for x in log.msgs if "expert-cache debug" in x]
    assert len(traced) == 2                  # only the first N calls
    assert traced[0].endswith("-> cached") and traced[1].endswith("-> read-through")


# --- opt-in split of wide steps (EXPERT_CACHE_SPLIT_WIDE) ---------------------------------

@dataclass
class ActDesc(Desc):
    dtype: object = None
    shape: object = None


class Shape:
    def __init__(self, row, col):
        self.row, self.col = row, col


class RowMethod(QuantMethod):
    """Per-token stand-in: row i of the output is x[i] + sum(topk_ids[i]) (in slot space
    on the cached path), so chunk order and chunk contents are both visible."""

    def __init__(self, layer, a1=None, a2=None, result=None):
        self.a1, self.a2, self.result = a1 or Desc(), a2 or Desc(), result
        super().__init__(layer)
        self.calls = []

    def _cfg(self, layer):
        cfg = super()._cfg(layer)
        cfg._a1, cfg._a2 = self.a1, self.a2
        return cfg

    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None,
              shared_experts_input=None):
        self.calls.append((tuple(topk_ids.shape), layer.global_num_experts))
        if self.result is not None:
            return self.result
        return x + topk_ids.sum(dim=1, keepdim=True).to(x.dtype)


def armed_rows(monkeypatch, split, **kw):
    monkeypatch.setenv("EXPERT_CACHE_SPLIT_WIDE", str(split))
    layer = RoutedExperts()
    m = RowMethod(layer, **kw)
    ok, log = arm(layer, m)
    assert ok, log.msgs
    refreshed = []

    def refresh(ids):
        refreshed.append(ids.clone())
        return ids + 100
    layer._expert_cache.refresh = refresh
    return layer, m, log, refreshed


def wide_step(tokens, k=2):
    x = torch.arange(tokens * H, dtype=torch.float32).reshape(tokens, H)
    ids = torch.arange(tokens * k, dtype=torch.int32).reshape(tokens, k) % E
    return x, torch.ones(tokens, k), ids


def test_split_is_off_by_default(monkeypatch):
    layer, m, _, refreshed = armed_rows(monkeypatch, 0)
    x, w, ids = wide_step(3)                     # 6 ids > S = 4
    out = m.apply(layer, x, w, ids)
    assert refreshed == [] and m.calls == [((3, 2), E)]
    assert torch.equal(out, x + ids.sum(1, keepdim=True))


def test_wide_step_is_served_in_cached_chunks(monkeypatch):
    layer, m, _, refreshed = armed_rows(monkeypatch, 4)
    x, w, ids = wide_step(5)                     # S // k = 2 tokens a chunk -> 3 chunks
    out = m.apply(layer, x, w, ids)
    assert [tuple(r.shape) for r in refreshed] == [(2, 2), (2, 2), (1, 2)]
    assert torch.equal(torch.cat(refreshed), ids)           # consecutive, in order
    assert m.calls == [((2, 2), S)] * 2 + [((1, 2), S)]     # every chunk slot-bound
    assert torch.equal(out, x + (ids + 100).sum(1, keepdim=True))
    assert layer.global_num_experts == E
    assert layer.w13_weight.size(0) == E


def test_split_limit_reads_through(monkeypatch):
    layer, m, _, refreshed = armed_rows(monkeypatch, 2)
    x, w, ids = wide_step(5)                     # needs 3 chunks, limit 2
    m.apply(layer, x, w, ids)
    assert refreshed == [] and m.calls == [((5, 2), E)]


def test_split_needs_room_for_one_token(monkeypatch):
    layer, m, _, refreshed = armed_rows(monkeypatch, 8)
    x, w, ids = wide_step(1, k=S + 1)            # one token already wider than the slots
    m.apply(layer, x, w, ids)
    assert refreshed == [] and m.calls == [((1, S + 1), E)]


def test_split_skips_steps_with_shared_experts(monkeypatch):
    layer, m, _, refreshed = armed_rows(monkeypatch, 4)
    x, w, ids = wide_step(3)
    m.apply(layer, x, w, ids, shared_experts=object(), shared_experts_input=x)
    assert refreshed == [] and m.calls == [((3, 2), E)]


@pytest.mark.parametrize("a1,a2,splits", [
    (ActDesc(dtype=torch.int8, shape=Shape(1, -1)), None, True),        # per token
    (ActDesc(dtype=torch.int8, shape=Shape(1, 128)), None, True),       # per token group
    (ActDesc(dtype=torch.int8, shape=Shape(128, 128)), None, True),     # K-blocked
    (ActDesc(dtype="mxfp8", shape=None), None, True),                   # micro-scaled
    (ActDesc(dtype=torch.int8, shape=Shape(-1, -1), scale=torch.ones(1)), None, True),
    (ActDesc(dtype=torch.int8, shape=Shape(-1, -1)), None, False),      # dynamic tensor
    (None, ActDesc(dtype=torch.int8, shape=Shape(-1, -1)), False),
    (ActDesc(dtype=torch.int8, shape=None), None, False),
])
def test_split_requires_token_local_activation_quant(monkeypatch, a1, a2, splits):
    layer, m, log, refreshed = armed_rows(monkeypatch, 4, a1=a1, a2=a2)
    x, w, ids = wide_step(3)
    m.apply(layer, x, w, ids)
    assert bool(refreshed) == splits
    assert log.said("not splitting wide steps") == (not splits)


def test_split_falls_back_when_apply_returns_a_pair(monkeypatch):
    layer, m, log, refreshed = armed_rows(monkeypatch, 4,
                                          result=(torch.zeros(1), torch.zeros(1)))
    x, w, ids = wide_step(3)
    out = m.apply(layer, x, w, ids)
    assert isinstance(out, tuple) and log.said("read through from now on")
    assert m.calls[-1] == ((3, 2), E)
    n = len(refreshed)
    m.apply(layer, x, w, ids)                    # splitting stays off for this layer
    assert len(refreshed) == n and m.calls[-1] == ((3, 2), E)


def test_debug_trace_names_the_split(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_DEBUG", "1")
    layer, m, log, _ = armed_rows(monkeypatch, 4)
    x, w, ids = wide_step(5)
    m.apply(layer, x, w, ids)
    assert [x for x in log.msgs if "expert-cache debug" in x][0].endswith("-> split 3")


# --- expert parallelism (EXPERT_CACHE_EP) ------------------------------------------------

class EPExperts(RoutedExperts):
    """vLLM's layout: the map is the ``_expert_map`` buffer behind a read-only property;
    rank 0 of 2, round-robin (global 2j is local j); E local experts of 2E."""

    def __init__(self, extra=()):
        super().__init__(extra)
        emap = torch.full((2 * E,), -1, dtype=torch.int32)
        emap[0::2] = torch.arange(E, dtype=torch.int32)
        self.register_buffer("_expert_map", emap)
        self.global_num_experts = 2 * E
        self.use_ep = True

    @property
    def expert_map(self):
        return self._expert_map


class Fmt:
    def __init__(self, name):
        self.name = name


def ep_method(layer, fmt="Standard", supports=True, **kw):
    m = QuantMethod(layer, **kw)
    m.moe_kernel.prepare_finalize = type("PF", (), {"activation_format": Fmt(fmt)})()
    m.moe_kernel.supports_expert_map = lambda: supports
    m.apply_seen_map = None
    stock = m.apply

    def apply(layer, x, topk_weights, topk_ids, shared_experts=None,
              shared_experts_input=None):
        m.apply_seen_map = layer.expert_map
        return stock(layer, x, topk_weights, topk_ids, shared_experts, shared_experts_input)
    m.apply = apply
    return m


def test_ep_refused_unless_opted_in():
    layer = EPExperts()
    ok, log = arm(layer, ep_method(layer))
    assert not ok and log.said("expert parallelism active")


def test_ep_layer_binds_the_composed_map(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_EP", "1")
    layer = EPExperts(SCALES)
    m = ep_method(layer, reads=["w13_weight_scale", "w2_weight_scale"])
    ok, log = arm(layer, m)
    assert ok, log.msgs
    cache = layer._expert_cache
    assert cache.E == E and cache.S == S
    full = layer._expert_map
    calls = []

    def refresh_ep(ids, emap):
        calls.append((ids.clone(), emap))
        return torch.full((2 * E,), 5, dtype=torch.int32)
    cache.refresh_ep = refresh_ep
    cache.refresh = lambda ids: pytest.fail("an EP step must not remap the routing ids")
    ids = torch.tensor([[0, 7, 2]], dtype=torch.int32)
    m.apply(layer, torch.randn(1, H), torch.ones(1, 3), ids)
    assert calls[0][1] is full                              # manage saw vLLM's own map
    assert torch.equal(m.seen["ids"], ids)                  # ids stay global
    assert (m.apply_seen_map == 5).all()                    # the kernel saw the composed map
    assert m.seen["gne"] == 2 * E                           # global count unchanged
    assert m.seen["w13"].data_ptr() == cache.slots["w13_weight"].data_ptr()
    assert m.seen["cfg"]._w1.scale.size(0) == S
    assert layer._expert_map is full and layer.global_num_experts == 2 * E
    assert layer.w13_weight.size(0) == E


def test_ep_wide_step_reads_through_with_vllms_map(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_EP", "1")
    layer = EPExperts()
    m = ep_method(layer)
    assert arm(layer, m)[0]
    layer._expert_cache.refresh_ep = lambda ids, emap: pytest.fail("wide step")
    m.apply(layer, torch.randn(1, H), torch.ones(1, S + 1),
            torch.zeros(1, S + 1, dtype=torch.int32))
    assert m.apply_seen_map is layer._expert_map


@pytest.mark.parametrize("setup,reason", [
    (dict(fmt="BatchedExperts"), "BatchedExperts activation format"),
    (dict(fmt=None), "unknown activation format"),
    (dict(supports=False), "does not take an expert map"),
    (dict(disable=True), "expert map disabled"),
])
def test_ep_refusals(monkeypatch, setup, reason):
    monkeypatch.setenv("EXPERT_CACHE_EP", "1")
    layer = EPExperts()
    m = ep_method(layer, fmt=setup.get("fmt", "Standard"), supports=setup.get("supports", True))
    if setup.get("fmt", "x") is None:
        m.moe_kernel.prepare_finalize = None
    if setup.get("disable"):
        m.disable_expert_map = True
    ok, log = arm(layer, m)
    assert not ok and log.said(reason), log.msgs


@pytest.mark.parametrize("attr,value", [("eplb_state", object()), ("enable_eplb", True)])
def test_eplb_layer_is_refused(monkeypatch, attr, value):
    # EPLB moves experts between ranks by rewriting the weight rows and expert_map in
    # place; a cache keyed by the old placement would serve the wrong expert's rows.
    monkeypatch.setenv("EXPERT_CACHE_EP", "1")
    layer = EPExperts()
    setattr(layer, attr, value)
    ok, log = arm(layer, ep_method(layer))
    assert not ok and log.said("EPLB"), log.msgs
    assert getattr(layer, "_expert_cache", None) is None


def test_ep_without_a_map_is_refused(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_EP", "1")
    layer = RoutedExperts()
    layer.use_ep = True                    # EP on, but the kernel is given no map
    ok, log = arm(layer, QuantMethod(layer))
    assert not ok and log.said("without an expert_map")


def test_ep_bookkeeping_buffers_are_not_mirrored(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_EP", "1")
    layer = EPExperts()
    layer.register_buffer("expert_local_to_global", torch.arange(E, dtype=torch.int64) * 2)
    ok, log = arm(layer, ep_method(layer))
    assert ok
    assert "expert_local_to_global" not in layer._expert_cache.names
    assert not log.said("not mirroring")


# --- next-layer prefetch linking (EXPERT_CACHE_PREFETCH) ---------------------------------

def gated(gate=None):
    layer = RoutedExperts()
    w = torch.randn(E, 64).to(torch.bfloat16) if gate is None else gate
    layer.runner = type("Runner", (), {})()
    layer.runner.gate = torch.nn.Linear(64, E, bias=False)
    layer.runner.gate.weight = torch.nn.Parameter(w, requires_grad=False)
    return layer


def armed_chain(layers):
    chain = []
    for ly in layers:
        assert arm(ly, QuantMethod(ly))[0]
        chain.append((ly, ly._expert_cache))
    return chain


def test_prefetch_links_consecutive_layers_with_usable_routers(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_PREFETCH", "3")
    bad_dtype = gated(torch.randn(E, 64))                        # fp32 router
    bad_width = gated(torch.randn(E, 60).to(torch.bfloat16))     # hidden % 8 != 0
    layers = [gated(), gated(), bad_dtype, gated(), bad_width]
    chain = armed_chain(layers)
    log = Log()
    assert generic._link_prefetch(chain, log) == 2
    caches = [c for _, c in chain]
    assert caches[0].next is caches[1]
    assert caches[0].next_gate is layers[1].runner.gate.weight
    assert caches[0].pred.shape == (S,) and caches[0].pred.dtype == torch.int32
    assert caches[0].prefetch_top == 3
    assert caches[1].next is None                 # the next router is fp32
    assert caches[2].next is caches[3]
    assert caches[3].next is None and caches[4].next is None
    assert log.said("not bf16") and log.said("layout")


def test_prefetch_skips_layers_without_a_router():
    plain = RoutedExperts()
    chain = armed_chain([gated(), plain])
    log = Log()
    assert generic._link_prefetch(chain, log) == 0
    assert log.said("no router weight")


def test_prefetch_not_linked_across_expert_parallel_layers(monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_EP", "1")
    ep = EPExperts()
    ep.runner = gated().runner
    assert arm(ep, ep_method(ep))[0]
    first = gated()
    assert arm(first, QuantMethod(first))[0]
    chain = [(first, first._expert_cache), (ep, ep._expert_cache)]
    assert generic._link_prefetch(chain, Log()) == 0


def test_prefetch_is_skipped_while_vllm_captures_piecewise(monkeypatch):
    import vllm.forward_context as fc
    monkeypatch.setattr(fc, "is_forward_context_available", lambda: True)
    for name, allowed in (("PIECEWISE", False), ("FULL", True), ("NONE", True)):
        ctx = type("Ctx", (), {"cudagraph_runtime_mode": type("M", (), {"name": name})()})()
        monkeypatch.setattr(fc, "get_forward_context", lambda c=ctx: c)
        assert generic._prefetch_allowed() == allowed, name


def test_prefetch_waits_for_a_full_step_of_the_next_layer(monkeypatch):
    # A prefetch parks the experts flagged in the next layer's `routed`; those must be the
    # next layer's last full cached step, never a prefetch's predictions, a split chunk's
    # subset or a stale state left by a read-through.
    monkeypatch.setenv("EXPERT_CACHE_PREFETCH", "2")
    monkeypatch.setenv("EXPERT_CACHE_SPLIT_WIDE", "4")
    nxt = gated()
    m = RowMethod(nxt)
    assert arm(nxt, m)[0]
    cache = nxt._expert_cache
    cache.refresh = lambda ids: ids + 100
    first = gated()
    assert arm(first, QuantMethod(first))[0]
    assert generic._link_prefetch([(first, first._expert_cache), (nxt, cache)], Log()) == 1
    x = torch.randn(1, 64).to(torch.bfloat16)

    def forks():    # a fork that gets past the check would need CUDA streams here
        try:
            generic._fork_prefetch(first._expert_cache, x, 2)
        except (RuntimeError, AssertionError, AttributeError):
            return True
        return False

    assert not cache.routed_is_step and not forks()        # never stepped yet
    m.apply(nxt, *wide_step(1))                             # a full cached step
    assert cache.routed_is_step and forks()
    m.apply(nxt, *wide_step(5))                             # split into chunks
    assert not cache.routed_is_step and not forks()
    m.apply(nxt, *wide_step(1))
    assert cache.routed_is_step
    m.apply(nxt, *wide_step(12))                            # too wide: reads through
    assert not cache.routed_is_step and not forks()
