"""AutoAWQ checkpoint loading (ashqk.awq_checkpoint): a synthetic checkpoint written with
safetensors, single-file and sharded, read back unchanged; config validation; module
replacement; the CUDA-only forward (GPU test) against the oracle."""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import awq_oracle as O

LAYERS = {"model.layers.0.self_attn.o_proj": (256, 128, True), "model.layers.0.mlp.down_proj": (512, 256, False)}
GROUP = 64


def _make_tensors(seed=0):
    rng = np.random.default_rng(seed)
    tensors = {"model.embed_tokens.weight": torch.randn(32, 256, dtype=torch.float16)}
    for name, (k, n, bias) in LAYERS.items():
        w = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(np.float32)
        qw, qz, s = O.quantize_awq(w, GROUP)
        tensors[f"{name}.qweight"] = torch.from_numpy(qw)
        tensors[f"{name}.qzeros"] = torch.from_numpy(qz)
        tensors[f"{name}.scales"] = torch.from_numpy(s)
        if bias:
            tensors[f"{name}.bias"] = torch.randn(n, dtype=torch.float16)
    return tensors


def _config(**over):
    q = {"quant_method": "awq", "bits": 4, "group_size": GROUP, "zero_point": True, "version": "gemm"}
    q.update(over)
    return {"architectures": ["Toy"], "quantization_config": q}


def _write(tmp_path, sharded=False, **cfg):
    from safetensors.torch import save_file

    t = _make_tensors()
    with open(tmp_path / "config.json", "w") as f:
        json.dump(_config(**cfg), f)
    if not sharded:
        save_file(t, str(tmp_path / "model.safetensors"))
        return t
    keys = sorted(t)
    parts = [keys[: len(keys) // 2], keys[len(keys) // 2:]]
    weight_map = {}
    for i, part in enumerate(parts):
        fn = f"model-{i + 1:05d}-of-00002.safetensors"
        save_file({k: t[k] for k in part}, str(tmp_path / fn))
        weight_map.update({k: fn for k in part})
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
    return t


@pytest.mark.parametrize("sharded", [False, True])
def test_load_round_trip(tmp_path, sharded):
    from ashqk.awq_checkpoint import load_awq_layers, read_config

    t = _write(tmp_path, sharded=sharded)
    assert read_config(str(tmp_path)).group_size == GROUP
    layers = load_awq_layers(str(tmp_path), device="cpu")
    assert set(layers) == set(LAYERS)
    for name, (k, n, bias) in LAYERS.items():
        L = layers[name]
        assert torch.equal(L.qweight, t[f"{name}.qweight"]) and torch.equal(L.qzeros, t[f"{name}.qzeros"])
        assert torch.equal(L.scales, t[f"{name}.scales"])
        assert (L.in_features, L.out_features) == (k, n)
        assert (L.bias is not None) == bias
    one = load_awq_layers(str(tmp_path), device="cpu", names=["model.layers.0.mlp.down_proj"])
    assert list(one) == ["model.layers.0.mlp.down_proj"]
    with pytest.raises(KeyError):
        load_awq_layers(str(tmp_path), device="cpu", names=["model.layers.1.mlp.down_proj"])


@pytest.mark.parametrize("bad", [{"version": "gemv"}, {"bits": 8}, {"zero_point": False}, {"quant_method": "gptq"},
                                 {"group_size": 128}])
def test_config_and_shape_validation(tmp_path, bad):
    from ashqk.awq_checkpoint import load_awq_layers

    _write(tmp_path, **bad)
    with pytest.raises(ValueError):
        load_awq_layers(str(tmp_path), device="cpu")


def test_inconsistent_tensors_rejected():
    from ashqk.awq_checkpoint import AWQLayer, check_layer

    qw = torch.zeros(256, 16, dtype=torch.int32)
    qz = torch.zeros(4, 16, dtype=torch.int32)
    s = torch.ones(4, 128, dtype=torch.float16)
    check_layer("ok", AWQLayer(qw, qz, s))
    with pytest.raises(ValueError):
        check_layer("scales", AWQLayer(qw, qz, torch.ones(4, 120, dtype=torch.float16)))
    with pytest.raises(ValueError):
        check_layer("dtype", AWQLayer(qw, qz, s.float()))
    with pytest.raises(ValueError):
        check_layer("groups", AWQLayer(qw, torch.zeros(3, 16, dtype=torch.int32), torch.ones(3, 128, dtype=torch.half)))


class _Toy(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList([torch.nn.Module()])
        blk = self.model.layers[0]
        blk.self_attn = torch.nn.Module()
        blk.self_attn.o_proj = torch.nn.Linear(256, 128)
        blk.mlp = torch.nn.Module()
        blk.mlp.down_proj = torch.nn.Linear(512, 256, bias=False)


def test_replace_linear_layers(tmp_path):
    from ashqk.awq_checkpoint import AWQLinear, load_awq_layers, replace_linear_layers

    _write(tmp_path)
    model = _Toy()
    replaced = replace_linear_layers(model, load_awq_layers(str(tmp_path), device="cpu"))
    assert sorted(replaced) == sorted(LAYERS)
    assert isinstance(model.model.layers[0].mlp.down_proj, AWQLinear)
    assert model.model.layers[0].self_attn.o_proj.bias is not None
    wrong = _Toy()
    wrong.model.layers[0].mlp.down_proj = torch.nn.Linear(512, 128)
    with pytest.raises(ValueError):
        replace_linear_layers(wrong, load_awq_layers(str(tmp_path), device="cpu"))


def test_forward_has_no_cpu_path(tmp_path):
    """The layer computes only on CUDA: a CPU input fails loudly instead of falling back."""
    from ashqk.awq_checkpoint import AWQLinear, load_awq_layers

    _write(tmp_path)
    lin = AWQLinear.from_layer(load_awq_layers(str(tmp_path), device="cpu")["model.layers.0.mlp.down_proj"])
    with pytest.raises(NotImplementedError):  # the operators are registered for CUDA only
        lin(torch.randn(2, 512, dtype=torch.float16))


@pytest.mark.gpu
def test_awq_linear_forward_matches_oracle(tmp_path):
    from ashqk.awq_checkpoint import AWQLinear, load_awq_layers
    from tests._helpers import rel_err

    t = _write(tmp_path)
    name = "model.layers.0.self_attn.o_proj"
    lin = AWQLinear.from_layer(load_awq_layers(str(tmp_path), device="cuda")[name])
    x = torch.randn(3, 256, dtype=torch.float16)
    y = lin(x.cuda())
    qw, qz, s = (t[f"{name}.{k}"].numpy() for k in ("qweight", "qzeros", "scales"))
    truth = O.c_gemm(x.numpy(), qw, qz, s) + t[f"{name}.bias"].float().numpy()
    w16 = torch.from_numpy(O.dequantize_awq(qw, qz, s, np.float16)).cuda()
    e_cublas = rel_err(x.cuda() @ w16 + t[f"{name}.bias"].cuda(), truth)
    assert rel_err(y, truth) <= 2 * e_cublas + 1e-5
