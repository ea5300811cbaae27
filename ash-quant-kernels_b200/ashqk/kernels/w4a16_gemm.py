"""Name kept from the reference's first GEMM (ashqk/kernels/w4a16_gemm.py:79).

The Triton v1 kernel is superseded; this entry point runs the same sm_100a GEMM
as ``w4a16_gemm_v3`` so code that imports it keeps working. The tile keyword
arguments of the reference are accepted and ignored.
"""

from __future__ import annotations

import torch

from .w4a16_gemm_v3 import w4a16_gemm_v3


def w4a16_gemm(x, qweight, qzeros, scales, block_m: int = 16, block_n: int = 64, block_k: int = 64,
               num_warps: int = 4, num_stages: int = 3) -> torch.Tensor:
    """x: [M, K] fp16; AWQ tensors as in ashqk.ref. Returns y: [M, N] fp16."""
    return w4a16_gemm_v3(x, qweight, qzeros, scales)
