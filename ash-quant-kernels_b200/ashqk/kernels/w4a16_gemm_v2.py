"""Name kept from the reference's second GEMM (ashqk/kernels/w4a16_gemm_v2.py:100).

Superseded by v3 in the reference; here it runs the same sm_100a GEMM as
``w4a16_gemm_v3`` and accepts (and ignores) the same ``config`` keys.
"""

from __future__ import annotations

import torch

from .w4a16_gemm_v3 import w4a16_gemm_v3


def w4a16_gemm_v2(x, qweight, qzeros, scales, config: dict | None = None) -> torch.Tensor:
    """x: [M, K] fp16; AWQ tensors as in ashqk.ref. Returns y: [M, N] fp16."""
    return w4a16_gemm_v3(x, qweight, qzeros, scales, config)
