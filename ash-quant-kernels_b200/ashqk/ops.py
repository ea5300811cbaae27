"""Public entry point ``w4a16_linear`` (mirrors ashqk/ops.py:18-26).

M <= GEMV_MAX_M rows go to the decode GEMV (tensor-core dot products on
register-dequantised int4, split-K in one launch); larger M goes to the
prefill GEMM. The reference's threshold was 2 (ashqk/ops.py:15), set by the
CUDA-core FMA limit of its Triton GEMV; the sm_100a GEMV uses mma.sync, whose
cost per weight does not grow with M up to 16, so the threshold is 16.
"""

from __future__ import annotations

import torch

from .kernels.w4a16_gemm_v3 import w4a16_gemm_v3
from .kernels.w4a16_gemv import w4a16_gemv

GEMV_MAX_M = 16


def w4a16_linear(x: torch.Tensor, qweight, qzeros, scales) -> torch.Tensor:
    """y = x @ dequant(AWQ weights); x: [..., K] fp16 -> [..., N] fp16."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.shape[0] <= GEMV_MAX_M:
        y = w4a16_gemv(x2, qweight, qzeros, scales)
    else:
        y = w4a16_gemm_v3(x2, qweight, qzeros, scales)
    return y.reshape(*lead, y.shape[-1])


def w4a16_linear_into(x: torch.Tensor, qweight, qzeros, scales, out: torch.Tensor) -> torch.Tensor:
    """Like ``w4a16_linear`` for a 2-D x, writing into ``out`` ([M, N] fp16, unit column stride).

    ``out`` may be a row-strided view (a slice of a larger buffer), which is how
    the tensor-parallel path lays out its gather buffer without a copy.
    """
    from . import _ext

    return _ext.ops().w4a16_linear_out(x, qweight, qzeros, scales, out)
