"""Shared helpers for the tests (problem generation, error metrics)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import awq_oracle as O


def rel_err(y, y_true) -> float:
    """Relative Frobenius error (tests/test_gemm.py:42-43 of the reference)."""
    if isinstance(y, torch.Tensor):
        y = y.detach().float().cpu().numpy()
    if isinstance(y_true, torch.Tensor):
        y_true = y_true.detach().float().cpu().numpy()
    return O.rel_err(y, y_true)


def quantized_problem(m, n, k, group_size, seed=0):
    """x ~ N(0,1) fp16, W ~ 0.02 N(0,1) RTN-quantised (tests/test_gemm.py:46-51 of the reference).

    Generated on the CPU with numpy so every device sees the same bytes.
    """
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32).astype(np.float16)
    w = (rng.standard_normal((k, n), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    qw, qz, s = O.quantize_awq(w, group_size)
    return x, qw, qz, s


def to_cuda(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]
