"""Qwen3.5-9B layer shapes (the reference's default benchmark model, bench/shapes.py there):
the skinny in_proj_ba (N=64) and the other linear layers at decode and prefill sizes, parity with
the oracle under the reference's criterion."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import awq_oracle as O
from tests._helpers import rel_err, to_cuda

pytestmark = pytest.mark.gpu

QWEN35 = [("in_proj_qkvz", 12288, 4096), ("in_proj_ba", 64, 4096), ("out_proj", 4096, 4096),
          ("qkv_proj", 10240, 4096), ("gate_up_proj", 24576, 4096), ("down_proj", 4096, 12288)]


@pytest.mark.parametrize("m", [1, 4, 16, 200])
@pytest.mark.parametrize("layer", QWEN35, ids=[l[0] for l in QWEN35])
def test_qwen35_layers(layer, m):
    from ashqk import w4a16_linear

    _, n, k = layer
    if m == 200 and n * k > 60_000_000:
        pytest.skip("prefill size covered by the smaller layers (oracle time)")
    x, qw, qz, s = O.make_problem(m, n, k, 128, seed=n + k + m)
    y = w4a16_linear(*to_cuda(x, qw, qz, s))
    torch.cuda.synchronize()
    y_true = O.c_gemm(x, qw, qz, s)
    w16 = torch.from_numpy(O.dequantize_awq(qw, qz, s, np.float16)).cuda()
    e_cublas = rel_err(torch.from_numpy(x).cuda() @ w16, y_true)
    assert rel_err(y, y_true) <= 2 * e_cublas + 1e-5
