"""The loader hook against the installed vLLM (CPU, no kernels).

``backends.generic.install`` must rebind ``process_weights_after_loading`` in vLLM's
``model_loader.utils`` and in every module that imported it by name (``base_loader`` does,
reference vllm_expert_cache/backends/generic.py:342-352), and the rebound hook must run
vLLM's own post-load step and then arm each FusedMoEMethodBase layer.  The layer and its
method are CPU stand-ins (the kernels are covered by the GPU tests).
"""

from __future__ import annotations

import types

import pytest
import torch

vllm_loader = pytest.importorskip("vllm.model_executor.model_loader.utils")

from test_generic import SCALES, Log, MoEKernel, RoutedExperts  # noqa: E402


def _method_class():
    from vllm.model_executor.layers.fused_moe.fused_moe_method_base import FusedMoEMethodBase

    class StandInMethod(FusedMoEMethodBase):
        """A FusedMoEMethodBase whose config factory reads the two scale tensors."""

        def create_weights(self, *a, **k):
            raise NotImplementedError

        def process_weights_after_loading(self, layer):
            self.processed = True

        def get_fused_moe_quant_config(self, layer):
            from test_generic import Desc, QuantConfig
            return QuantConfig(Desc(), Desc(), Desc(scale=layer.w13_weight_scale),
                               Desc(scale=layer.w2_weight_scale))

        def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None,
                  shared_experts_input=None):
            self.seen = (layer.w13_weight.shape[0], topk_ids.clone())
            return torch.zeros(1)

    return StandInMethod


def test_install_rebinds_hook_and_arms_layers(monkeypatch):
    from vllm.model_executor.model_loader import base_loader

    from vllm_expert_cache.backends import generic

    monkeypatch.setenv("EXPERT_CACHE_SLOTS", "4")
    stock = vllm_loader.process_weights_after_loading
    monkeypatch.setattr(generic, "_installed", False)
    log = Log()
    try:
        assert generic.install(log)
        hook = vllm_loader.process_weights_after_loading
        assert hook is not stock
        assert base_loader.process_weights_after_loading is hook
        assert log.said("hooked the MoE loader")

        cls = _method_class()
        model = torch.nn.Module()
        for i in range(2):
            layer = RoutedExperts(SCALES)
            method = object.__new__(cls)          # skip vLLM's constructor: a stand-in
            method.moe_kernel = MoEKernel(None)
            method.moe_kernel.is_monolithic = False
            method.moe_quant_config = method.get_fused_moe_quant_config(layer)
            layer.quant_method = method
            model.add_module(f"moe{i}", layer)
        cfg = types.SimpleNamespace(quantization=None, dtype=torch.bfloat16)
        base_loader.process_weights_after_loading(model, cfg, torch.device("cpu"))

        for layer in (model.moe0, model.moe1):
            assert layer.quant_method.processed          # vLLM's own step ran first
            cache = layer._expert_cache                   # then the layer was armed
            assert cache.S == 4 and cache.E == 16
            assert set(cache.names) == {"w13_weight", "w2_weight", "w13_weight_scale",
                                        "w2_weight_scale"}
        assert log.said("active on 2 MoE layer(s)")

        # the wrapped apply serves a fitting step from slot storage
        layer = model.moe0
        layer._expert_cache.refresh = lambda ids: ids.clone() + 1
        layer.quant_method.apply(layer=layer, x=torch.randn(1, 8),
                                 topk_weights=torch.ones(1, 2),
                                 topk_ids=torch.zeros(1, 2, dtype=torch.int32))
        n_rows, ids = layer.quant_method.seen
        assert n_rows == 4 and (ids == 1).all()
    finally:
        vllm_loader.process_weights_after_loading = stock
        base_loader.process_weights_after_loading = stock


def _cfgs():
    """vLLM's own quant-config factories, with whether a token of the config computes
    independently of the rest of its step."""
    from vllm.model_executor.layers.fused_moe import config as c
    w = torch.ones(4, 8, 1)
    yield "unquantized", c.FUSED_MOE_UNQUANTIZED_CONFIG, True
    yield "int8 per-token dynamic", c.int8_w8a8_moe_quant_config(
        w, w, None, None, per_act_token_quant=True), True
    yield "int8 per-tensor dynamic", c.int8_w8a8_moe_quant_config(w, w, None, None), False
    yield "int8 per-tensor static", c.int8_w8a8_moe_quant_config(
        w, w, torch.ones(1), torch.ones(1)), True
    yield "fp8 block", c.fp8_w8a8_moe_quant_config(w, w, block_shape=[128, 128]), True
    yield "fp8 per-tensor dynamic", c.fp8_w8a8_moe_quant_config(w, w), False
    yield "int4 weight-only", c.int4_w4a16_moe_quant_config(w, w, None, None), True


@pytest.mark.parametrize("name,cfg,local", list(_cfgs()), ids=lambda v: v
                         if isinstance(v, str) else "")
def test_token_locality_of_vllm_quant_configs(name, cfg, local):
    from vllm_expert_cache.backends import generic
    assert (generic._token_local(cfg) is None) == local, name
