"""vLLM integration: AutoAWQ checkpoints served through the B200 kernels.

Importing this module registers the quantization method ``"ashqk_awq"`` with vLLM
(``vllm.model_executor.layers.quantization.register_quantization_config``). It reuses vLLM's own
AWQ weight handling -- the checkpoint tensors ``qweight`` / ``qzeros`` / ``scales`` and their
tensor-parallel loaders are exactly the AutoAWQ "GEMM" layout the kernels consume, with no repack
-- and replaces only the product: ``apply`` calls ``ashqk.w4a16_linear`` (decode GEMV for
M <= 16, the tcgen05 GEMM above). Select it with ``quantization="ashqk_awq"`` on an AWQ checkpoint
(vLLM's own ``awq`` method is left untouched). This is the integration the reference lists as its
next step (its README.md roadmap, v0.3 "SGLang integration + e2e").
"""

from __future__ import annotations

from typing import Any, Optional

import torch
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.awq import AWQConfig, AWQLinearMethod

from ..ops import w4a16_linear

METHOD = "ashqk_awq"


class AshqkAWQLinearMethod(AWQLinearMethod):
    """vLLM's AWQ weights, multiplied by the sm_100a kernels."""

    def apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        y = w4a16_linear(x, layer.qweight, layer.qzeros, layer.scales)
        return y + bias if bias is not None else y


@register_quantization_config(METHOD)
class AshqkAWQConfig(AWQConfig):
    """AutoAWQ 4-bit, zero point, GEMM packing; needs an sm_100 GPU."""

    def get_name(self) -> str:
        return METHOD

    @classmethod
    def get_min_capability(cls) -> int:
        return 100

    @classmethod
    def override_quantization_method(cls, hf_quant_cfg: dict[str, Any], user_quant: Optional[str]) -> Optional[str]:
        # AWQ checkpoints say quant_method "awq"; take them when the user asks for this method.
        if user_quant == METHOD and str(hf_quant_cfg.get("quant_method", "")).lower() == "awq":
            return METHOD
        return None

    def get_quant_method(self, layer: torch.nn.Module, prefix: str):
        method = super().get_quant_method(layer, prefix)
        if type(method) is AWQLinearMethod:
            return AshqkAWQLinearMethod(self)
        return method  # unquantised layers (modules_to_not_convert) and MoE stay vLLM's
