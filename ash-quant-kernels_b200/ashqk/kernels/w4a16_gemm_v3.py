"""Prefill GEMM shim: same signature as ashqk/kernels/w4a16_gemm_v3.py:131.

The work happens in the sm_100a kernel behind ``torch.ops.ashqk.w4a16_gemm``
(csrc/gemm_sm100.cu). The reference's Triton ``config`` keys are accepted and
ignored: the CUDA kernel has one tile shape.
"""

from __future__ import annotations

import torch

from .. import _ext
from ._common import check_awq

_CONFIG_KEYS = {"block_m", "block_n", "block_k", "split_k", "num_warps", "num_stages"}


def _default_config(M: int) -> dict:
    return dict(block_m=128, block_n=256, block_k=64, split_k=1)


def w4a16_gemm_v3(x, qweight, qzeros, scales, config: dict | None = None) -> torch.Tensor:
    """x: [M, K] fp16; AWQ tensors as in ashqk.ref. Returns y: [M, N] fp16."""
    M, N, K, group_size = check_awq(x, qweight, qzeros, scales)
    cfg = dict(_default_config(M), **(config or {}))
    unknown = set(cfg) - _CONFIG_KEYS
    assert not unknown, f"unknown config keys {sorted(unknown)}"
    return _ext.ops().w4a16_gemm(x, qweight, qzeros, scales)
