"""The decode GEMV entry point that allocates nothing (ashqk_w4a16_gemv_noalloc).

Callers that cannot allocate device memory -- a plugin handed only device
pointers by its host, or code that must not call cudaMalloc on its hot path --
use this entry point; its split-K scratch is a fixed array inside the library.
These tests call it through the C ABI, twice in a row on each problem (the
second call reuses the scratch the first one left behind), and compare with the
workspace-taking entry point ashqk_w4a16_gemv and with the oracle. The file is
named to be collected last; it also passes when run alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import awq_oracle as O
from tests._helpers import quantized_problem, rel_err, to_cuda

pytestmark = pytest.mark.gpu

VP, I64, CI = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int


def _lib():
    from ashqk import _ext

    lib = ctypes.CDLL(_ext.C_LIBRARY)
    lib.ashqk_w4a16_gemv_noalloc.argtypes = [VP, I64, VP, I64, VP, I64, VP, I64, VP, I64, CI, CI, CI, CI, CI, VP]
    lib.ashqk_w4a16_gemv.argtypes = [VP, I64, VP, I64, VP, I64, VP, I64, VP, I64, CI, CI, CI, CI, CI, VP,
                                     ctypes.c_size_t, VP]
    lib.ashqk_gemv_workspace_size.argtypes = [CI, CI, CI, CI, CI, ctypes.POINTER(ctypes.c_size_t)]
    return lib


def _call_noalloc(lib, xd, qwd, qzd, sd, y, m, n, k, g, split):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.ashqk_w4a16_gemv_noalloc(xd.data_ptr(), xd.stride(0), qwd.data_ptr(), qwd.stride(0), qzd.data_ptr(),
                                        qzd.stride(0), sd.data_ptr(), sd.stride(0), y.data_ptr(), y.stride(0), m, n,
                                        k, g, split, stream)


def _call_workspace(lib, xd, qwd, qzd, sd, y, m, n, k, g, split):
    size = ctypes.c_size_t(0)
    assert lib.ashqk_gemv_workspace_size(min(m, 16), n, k, g, split, ctypes.byref(size)) == 0
    ws = torch.zeros(max(int(size.value), 1), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.ashqk_w4a16_gemv(xd.data_ptr(), xd.stride(0), qwd.data_ptr(), qwd.stride(0), qzd.data_ptr(),
                              qzd.stride(0), sd.data_ptr(), sd.stride(0), y.data_ptr(), y.stride(0), m, n, k, g, split,
                              ws.data_ptr(), ws.numel(), stream)
    torch.cuda.synchronize()
    return rc


@pytest.mark.parametrize("m,n,k,g,split", [
    (1, 6144, 4096, 128, 0),    # qkv, decode
    (4, 24576, 4096, 128, 0),   # gate_up
    (16, 4096, 12288, 128, 0),  # down, two n8 token tiles
    (7, 1000, 512, 64, 3),      # register-streaming kernel (N % 32 != 0), forced split
    (20, 512, 1024, 32, 4),     # M > 16: processed 16 rows at a time
])
def test_noalloc_matches_workspace_entry_point(m, n, k, g, split):
    lib = _lib()
    x, qw, qz, s = quantized_problem(m, n, k, g, seed=m + n + k)
    xd, qwd, qzd, sd = to_cuda(x, qw, qz, s)
    y_ref = torch.empty(m, n, dtype=torch.float16, device="cuda")
    assert _call_workspace(lib, xd, qwd, qzd, sd, y_ref, m, n, k, g, split) == 0

    y_true = O.c_gemm(x, qw, qz, s)
    w16 = torch.from_numpy(O.dequantize_awq(qw, qz, s, np.float16)).cuda()
    e_cublas = rel_err(xd @ w16, y_true)
    for attempt in range(2):  # the second call runs on the scratch the first one left
        y = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
        assert _call_noalloc(lib, xd, qwd, qzd, sd, y, m, n, k, g, split) == 0
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref), attempt  # same kernel, deterministic split-K order
        assert rel_err(y, y_true) <= 2 * e_cublas + 1e-5, attempt


def test_noalloc_rejects_problems_beyond_its_scratch():
    """A split forcing more than 8 MiB of partial sums is refused before any launch. (The default
    kernel takes a split without scratch, so the split-K kernel, which uses it, is forced here.)"""
    lib = _lib()
    m, n, k, g = 16, 24576, 4096, 128
    size = ctypes.c_size_t(0)
    assert lib.ashqk_gemv_workspace_size(m, n, k, g, 32, ctypes.byref(size)) == 0
    assert size.value > (8 << 20)
    xd, qwd, qzd, sd = to_cuda(*O.make_problem(m, n, k, g, seed=1))
    y = torch.zeros(m, n, dtype=torch.float16, device="cuda")
    assert lib.ashqk_set_gemv_kernel(2) == 0
    try:
        assert _call_noalloc(lib, xd, qwd, qzd, sd, y, m, n, k, g, 32) == 3  # ASHQK_ERR_WORKSPACE
    finally:
        assert lib.ashqk_set_gemv_kernel(0) == 0
    torch.cuda.synchronize()
    assert int(y.abs().sum()) == 0  # nothing was written
