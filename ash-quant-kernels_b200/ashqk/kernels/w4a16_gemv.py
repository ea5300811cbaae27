"""Decode GEMV shim: same signature as ashqk/kernels/w4a16_gemv.py:132.

The work happens in the sm_100a kernel behind ``torch.ops.ashqk.w4a16_gemv``
(csrc/gemv.cu). ``config`` keeps the reference's keys: ``split_k`` is passed on
as the K-split hint (the kernel may raise it to fit its shared-memory slice);
the Triton tile keys (``block_m``, ``block_n``, ``block_k``, ``num_warps``,
``num_stages``) have no meaning for the CUDA kernel and are accepted and ignored.
"""

from __future__ import annotations

import torch

from .. import _ext
from ._common import check_awq

_CONFIG_KEYS = {"block_m", "block_n", "block_k", "split_k", "num_warps", "num_stages"}


def _default_config(M: int, N: int) -> dict:
    # split_k 0 = the kernel picks the split from the SM count and problem size.
    return dict(block_m=min(M, 16), block_n=128, block_k=16, split_k=0)


def w4a16_gemv(x, qweight, qzeros, scales, config: dict | None = None) -> torch.Tensor:
    """x: [M, K] fp16 (small M); AWQ tensors as in ashqk.ref. Returns [M, N] fp16."""
    M, N, K, group_size = check_awq(x, qweight, qzeros, scales)
    cfg = dict(_default_config(M, N), **(config or {}))
    unknown = set(cfg) - _CONFIG_KEYS
    assert not unknown, f"unknown config keys {sorted(unknown)}"
    return _ext.ops().w4a16_gemv(x, qweight, qzeros, scales, int(cfg["split_k"]))
