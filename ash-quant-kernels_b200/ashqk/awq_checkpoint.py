"""AutoAWQ "GEMM" checkpoints: load the packed tensors, run them through ``w4a16_linear``.

The reference's format contract (its README.md "Format" section, ashqk/ref.py:1-21) is the tensor
layout AutoAWQ writes and vLLM / SGLang load: per linear layer ``<name>.qweight`` int32 [K, N/8],
``<name>.qzeros`` int32 [K/G, N/8] and ``<name>.scales`` fp16 [K/G, N] (optionally ``<name>.bias``),
with the quantisation settings in the model's ``config.json`` (``quantization_config``) or in
``quant_config.json``. This module reads such checkpoints from ``.safetensors`` files (one file,
or shards listed in ``model.safetensors.index.json``) without repacking anything, and offers a
``torch.nn.Module`` that computes the layer with the B200 kernels.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Dict, Iterable, Optional

import torch

from .ops import w4a16_linear

_SUFFIXES = ("qweight", "qzeros", "scales")


@dataclass(frozen=True)
class AWQConfig:
    """The AutoAWQ settings this package supports: 4-bit, zero point, GEMM packing."""

    bits: int = 4
    group_size: int = 128
    zero_point: bool = True
    version: str = "gemm"

    @staticmethod
    def from_dict(d: dict) -> "AWQConfig":
        q = d.get("quantization_config", d)
        method = str(q.get("quant_method", "awq")).lower()
        cfg = AWQConfig(bits=int(q.get("w_bit", q.get("bits", 4))),
                        group_size=int(q.get("q_group_size", q.get("group_size", 128))),
                        zero_point=bool(q.get("zero_point", True)),
                        version=str(q.get("version", "gemm")).lower())
        if method != "awq":
            raise ValueError(f"not an AWQ checkpoint (quant_method={method!r})")
        if cfg.bits != 4 or not cfg.zero_point or cfg.version != "gemm":
            raise ValueError(f"unsupported AWQ variant {cfg}: only 4-bit, zero-point, GEMM packing")
        if cfg.group_size <= 0:
            raise ValueError("group_size must be positive (per-channel -1 is not AutoAWQ GEMM)")
        return cfg


def read_config(model_dir: str) -> AWQConfig:
    """The AWQ settings of a checkpoint directory (``config.json`` or ``quant_config.json``)."""
    for name in ("config.json", "quant_config.json", "quantize_config.json"):
        p = os.path.join(model_dir, name)
        if os.path.exists(p):
            with open(p) as f:
                d = json.load(f)
            if name != "config.json" or "quantization_config" in d:
                return AWQConfig.from_dict(d)
    raise FileNotFoundError(f"no AWQ quantisation config in {model_dir}")


def _shards(path: str) -> list[str]:
    if os.path.isfile(path):
        return [path]
    index = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, f) for f in files]
    files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {path}")
    return [os.path.join(path, f) for f in files]


@dataclass
class AWQLayer:
    qweight: torch.Tensor
    qzeros: torch.Tensor
    scales: torch.Tensor
    bias: Optional[torch.Tensor] = None

    @property
    def in_features(self) -> int:
        return self.qweight.shape[0]

    @property
    def out_features(self) -> int:
        return self.qweight.shape[1] * 8


def check_layer(name: str, layer: AWQLayer, group_size: Optional[int] = None) -> None:
    """Shape and dtype checks of one layer (the reference's asserts, kernels/w4a16_gemv.py:134-141)."""
    qw, qz, s = layer.qweight, layer.qzeros, layer.scales
    if qw.dtype != torch.int32 or qz.dtype != torch.int32 or s.dtype != torch.float16:
        raise ValueError(f"{name}: expected int32 qweight/qzeros and fp16 scales, got {qw.dtype}, {qz.dtype}, "
                         f"{s.dtype}")
    if qw.dim() != 2 or qz.dim() != 2 or s.dim() != 2:
        raise ValueError(f"{name}: AWQ tensors must be 2-D")
    k, words = qw.shape
    groups = s.shape[0]
    if qz.shape != (groups, words) or s.shape[1] != words * 8 or groups == 0 or k % groups:
        raise ValueError(f"{name}: inconsistent shapes qweight {tuple(qw.shape)}, qzeros {tuple(qz.shape)}, "
                         f"scales {tuple(s.shape)}")
    if group_size is not None and k // groups != group_size:
        raise ValueError(f"{name}: group size {k // groups} != configured {group_size}")
    if layer.bias is not None and layer.bias.shape != (words * 8,):
        raise ValueError(f"{name}: bias shape {tuple(layer.bias.shape)} != ({words * 8},)")


def load_awq_layers(path: str, device: str | torch.device = "cuda", names: Optional[Iterable[str]] = None,
                    group_size: Optional[int] = None) -> Dict[str, AWQLayer]:
    """Every AWQ linear layer of a checkpoint (a ``.safetensors`` file or a directory of shards).

    Returns ``{layer name: AWQLayer}`` with the tensors as stored (no repack), moved to ``device``.
    ``names`` restricts the result to those layers. The group size is taken from the directory's
    config when present (and checked against every layer), else inferred per layer.
    """
    from safetensors import safe_open

    if group_size is None and os.path.isdir(path):
        try:
            group_size = read_config(path).group_size
        except FileNotFoundError:
            group_size = None
    wanted = set(names) if names is not None else None
    found: Dict[str, Dict[str, torch.Tensor]] = {}
    for shard in _shards(path):
        with safe_open(shard, framework="pt", device="cpu") as f:
            for key in f.keys():
                base, _, suffix = key.rpartition(".")
                if suffix not in _SUFFIXES + ("bias",):
                    continue
                if wanted is not None and base not in wanted:
                    continue
                found.setdefault(base, {})[suffix] = f.get_tensor(key)
    layers = {}
    for base, t in sorted(found.items()):
        if not all(s in t for s in _SUFFIXES):
            continue  # an ordinary (unquantised) layer's bias, or a partial entry
        layer = AWQLayer(*(t[s].to(device) for s in _SUFFIXES),
                         bias=t["bias"].to(device=device, dtype=torch.float16) if "bias" in t else None)
        check_layer(base, layer, group_size)
        layers[base] = layer
    if wanted is not None and set(layers) != wanted:
        raise KeyError(f"layers not found in {path}: {sorted(wanted - set(layers))}")
    return layers


class AWQLinear(torch.nn.Module):
    """A linear layer y = x @ W (+ bias) with W held as AutoAWQ int4 tensors; CUDA only."""

    def __init__(self, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                 bias: Optional[torch.Tensor] = None):
        super().__init__()
        check_layer("AWQLinear", AWQLayer(qweight, qzeros, scales, bias))
        self.register_buffer("qweight", qweight)
        self.register_buffer("qzeros", qzeros)
        self.register_buffer("scales", scales)
        self.register_buffer("bias", bias)
        self.in_features, self.out_features = qweight.shape[0], qweight.shape[1] * 8

    @staticmethod
    def from_layer(layer: AWQLayer) -> "AWQLinear":
        return AWQLinear(layer.qweight, layer.qzeros, layer.scales, layer.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = w4a16_linear(x, self.qweight, self.qzeros, self.scales)
        return y + self.bias if self.bias is not None else y

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"group_size={self.in_features // self.scales.shape[0]}, bias={self.bias is not None}")


def replace_linear_layers(model: torch.nn.Module, layers: Dict[str, AWQLayer]) -> list[str]:
    """Swap each ``nn.Linear`` of ``model`` named in ``layers`` for an ``AWQLinear``.

    Names follow ``model.named_modules()``. The quantised layer must have the Linear's in/out
    features. Returns the replaced names; layers of the checkpoint that match no module are an error.
    """
    modules = dict(model.named_modules())
    missing = [n for n in layers if n not in modules]
    if missing:
        raise KeyError(f"checkpoint layers with no module in the model: {missing[:5]}")
    replaced = []
    for name, layer in layers.items():
        mod = modules[name]
        if not isinstance(mod, torch.nn.Linear):
            raise TypeError(f"{name} is a {type(mod).__name__}, not nn.Linear")
        if (mod.in_features, mod.out_features) != (layer.in_features, layer.out_features):
            raise ValueError(f"{name}: checkpoint is {layer.in_features}->{layer.out_features}, module is "
                             f"{mod.in_features}->{mod.out_features}")
        parent_name, _, child = name.rpartition(".")
        parent = modules[parent_name] if parent_name else model
        setattr(parent, child, AWQLinear.from_layer(layer))
        replaced.append(name)
    return replaced
