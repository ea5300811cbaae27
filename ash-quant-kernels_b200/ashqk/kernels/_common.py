"""Argument checks shared by the kernel shims.

The reference validates with Python ``assert`` (ashqk/kernels/w4a16_gemv.py:134-141,
ashqk/kernels/w4a16_gemm_v3.py:137-144); the shims keep that, so a malformed
call raises ``AssertionError`` before reaching native code.
"""

from __future__ import annotations

import torch


def check_awq(x: torch.Tensor, qweight, qzeros, scales):
    assert x.dtype == torch.float16 and x.dim() == 2
    M, K = x.shape
    N = qweight.shape[1] * 8
    group_size = K // scales.shape[0]
    assert qweight.shape == (K, N // 8)
    assert qzeros.shape == (K // group_size, N // 8)
    assert scales.shape == (K // group_size, N)
    assert K % group_size == 0
    return M, N, K, group_size
