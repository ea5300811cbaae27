"""The vLLM plugin (ashqk.integrations.vllm_plugin): registration of the "ashqk_awq" method,
config parsing, which layers it takes over, and its product (GPU test). The weight creation and
loading are vLLM's own AWQ code, which needs vLLM's runtime context and is not re-tested here."""

from __future__ import annotations

import pytest
import torch

vllm = pytest.importorskip("vllm")

AWQ_CFG = {"quant_method": "awq", "w_bit": 4, "q_group_size": 128, "zero_point": True, "version": "gemm"}


def _plugin():
    from ashqk.integrations import vllm_plugin

    return vllm_plugin


def test_registered_and_parsed():
    from vllm.model_executor.layers.quantization import get_quantization_config

    vp = _plugin()
    assert get_quantization_config("ashqk_awq") is vp.AshqkAWQConfig
    cfg = vp.AshqkAWQConfig.from_config(AWQ_CFG)
    assert cfg.get_name() == "ashqk_awq" and cfg.group_size == 128 and cfg.weight_bits == 4
    assert vp.AshqkAWQConfig.get_min_capability() == 100
    assert torch.float16 in cfg.get_supported_act_dtypes()


def test_selected_only_when_asked():
    vp = _plugin()
    assert vp.AshqkAWQConfig.override_quantization_method({"quant_method": "awq"}, "ashqk_awq") == "ashqk_awq"
    assert vp.AshqkAWQConfig.override_quantization_method({"quant_method": "awq"}, None) is None
    assert vp.AshqkAWQConfig.override_quantization_method({"quant_method": "gptq"}, "ashqk_awq") is None


def test_takes_over_awq_linear_layers_only(monkeypatch):
    from vllm.model_executor.layers.quantization.awq import AWQConfig, AWQLinearMethod

    vp = _plugin()
    cfg = vp.AshqkAWQConfig.from_config(AWQ_CFG)
    monkeypatch.setattr(AWQConfig, "get_quant_method", lambda self, layer, prefix: AWQLinearMethod(self))
    assert isinstance(cfg.get_quant_method(torch.nn.Module(), "model.layers.0.mlp.down_proj"), vp.AshqkAWQLinearMethod)
    other = object()
    monkeypatch.setattr(AWQConfig, "get_quant_method", lambda self, layer, prefix: other)
    assert cfg.get_quant_method(torch.nn.Module(), "lm_head") is other
    monkeypatch.setattr(AWQConfig, "get_quant_method", lambda self, layer, prefix: None)
    assert cfg.get_quant_method(torch.nn.Module(), "norm") is None


@pytest.mark.gpu
def test_apply_is_the_b200_product():
    from ashqk import w4a16_linear
    from oracle import awq_oracle as O
    from tests._helpers import to_cuda

    vp = _plugin()
    method = vp.AshqkAWQLinearMethod(vp.AshqkAWQConfig.from_config(AWQ_CFG))
    x, qw, qz, s = O.make_problem(5, 1024, 2048, 128, seed=3)
    xd, qwd, qzd, sd = to_cuda(x, qw, qz, s)
    layer = torch.nn.Module()
    layer.qweight, layer.qzeros, layer.scales = qwd, qzd, sd
    bias = torch.randn(1024, device="cuda").half()
    y = method.apply(layer, xd.view(1, 5, 2048), bias)
    assert y.shape == (1, 5, 1024)
    assert torch.equal(y, (w4a16_linear(xd, qwd, qzd, sd) + bias).view(1, 5, 1024))
