"""Split wide steps (EXPERT_CACHE_SPLIT_WIDE) through vLLM's own fused-MoE kernel on a B200.

A stand-in MoE method whose ``apply`` is vLLM's Triton ``fused_experts`` with the W8A8 int8
per-token config (the compressed-tensors int8 MoE path) is armed by the real
``generic.arm``; the slot cache runs the sm_100a manage and gather kernels.  A step wider
than the slots is then served as cached chunks, and its output must equal, bit for bit,
the stock kernel run over the same chunks on the full expert tensors: the cache changes
where each expert's bytes are read from, never the arithmetic.  Against the stock kernel
over the whole step at once the int8 path (integer accumulation, per-token activation
scales) is expected to agree too; that comparison uses a bf16 tolerance because it is a
property of vLLM's kernel, not of the cache.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from test_generic import Log

pytestmark = pytest.mark.gpu

E, S, H, N, K = 16, 8, 256, 128, 4          # 8 slots, top-4: 2 tokens per chunk


@pytest.fixture(scope="module")
def vllm_moe():
    fm = pytest.importorskip("vllm.model_executor.layers.fused_moe.fused_moe")
    cfg = pytest.importorskip("vllm.model_executor.layers.fused_moe.config")
    return fm.fused_experts, cfg.int8_w8a8_moe_quant_config


class Layer(torch.nn.Module):
    def __init__(self, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        p = lambda t: torch.nn.Parameter(t.cuda(), requires_grad=False)  # noqa: E731
        self.w13_weight = p(torch.randint(-128, 128, (E, 2 * N, H), dtype=torch.int8,
                                          generator=g))
        self.w2_weight = p(torch.randint(-128, 128, (E, H, N), dtype=torch.int8, generator=g))
        self.w13_weight_scale = p(torch.rand(E, 2 * N, 1, generator=g) * 1e-3 + 1e-4)
        self.w2_weight_scale = p(torch.rand(E, H, 1, generator=g) * 1e-3 + 1e-4)
        self.global_num_experts = E
        self.expert_map = None


class Int8Method:
    """compressed-tensors W8A8 int8 MoE, reduced to what arming and ``apply`` touch."""

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


def routing(tokens, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(tokens)])
    w = torch.softmax(torch.randn(tokens, K, generator=g), dim=1)
    x = (torch.randn(tokens, H, generator=g) * 0.5).to(torch.bfloat16)
    return x.cuda(), w.cuda(), ids.to(torch.int32).cuda()


@pytest.mark.parametrize("tokens", [3, 5, 8])
def test_split_equals_stock_chunks_bit_exact(vllm_moe, monkeypatch, tokens):
    monkeypatch.setenv("EXPERT_CACHE_SLOTS", str(S))
    monkeypatch.setenv("EXPERT_CACHE_SPLIT_WIDE", "4")
    from vllm_expert_cache.backends import generic
    layer = Layer(seed=tokens)
    m = Int8Method(layer, *vllm_moe)
    stock = m.apply
    log = Log()
    assert generic.arm(layer, m, log), log.msgs
    per = S // K
    for step in range(6):                     # a drive: the chunks evict one another
        x, w, ids = routing(tokens, seed=100 * tokens + step)
        got = m.apply(layer, x, w, ids)
        want_chunks = torch.cat([stock(layer, x[i:i + per], w[i:i + per], ids[i:i + per])
                                 for i in range(0, tokens, per)])
        want_whole = stock(layer, x, w, ids)
        torch.cuda.synchronize()
        assert torch.equal(got, want_chunks), f"step {step}"
        torch.testing.assert_close(got, want_whole, rtol=1.6e-2, atol=1e-2)
    # the layer is left on its full tensors between steps
    assert layer.w13_weight.size(0) == E and layer.global_num_experts == E


def test_fitting_step_is_cached_and_exact(vllm_moe, monkeypatch):
    monkeypatch.setenv("EXPERT_CACHE_SLOTS", str(S))
    from vllm_expert_cache.backends import generic
    layer = Layer(seed=7)
    m = Int8Method(layer, *vllm_moe)
    stock = m.apply
    assert generic.arm(layer, m, Log())
    for step in range(4):
        x, w, ids = routing(2, seed=900 + step)   # 8 ids == S: the ordinary cached path
        got = m.apply(layer, x, w, ids)
        assert torch.equal(got, stock(layer, x, w, ids)), f"step {step}"
    assert int(layer._expert_cache.step.item()) == 4
