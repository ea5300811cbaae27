"""The cluster-split decode GEMV (``csrc/gemv_cluster.cu``) on a B200, against the oracle.

Forces the kernel (``ashqk_set_gemv_kernel(4)``) and sweeps its work split
(``ashqk_gemv_set_tuning``: shared-memory budget, CTAs per cluster, tile width)
so that both tile widths (256 columns x 256-row stages, 512 x 128), clusters
of 1 to 16 CTAs, uneven stage ranges and one-stage rings all run. Every result
meets the reference's criterion against the fp64 oracle; repeated calls are
bitwise identical (the cluster sums partial strips in fixed rank order).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import awq_oracle as O
from tests._helpers import quantized_problem, rel_err, to_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from ashqk import _ext

    lib = ctypes.CDLL(_ext.C_LIBRARY)
    assert lib.ashqk_set_gemv_kernel(4) == 0
    yield lib
    assert lib.ashqk_set_gemv_kernel(0) == 0
    assert lib.ashqk_gemv_set_tuning(0, 0, 0, 0) == 0


def _check(x, qw, qz, s, y):
    y_true = O.c_gemm(x, qw, qz, s)
    w16 = torch.from_numpy(O.dequantize_awq(qw, qz, s, np.float16)).cuda()
    e_cublas = rel_err(torch.from_numpy(x).cuda() @ w16, y_true)
    e = rel_err(y, y_true)
    assert e <= 2 * e_cublas + 1e-5, (e, e_cublas)


# (smem_kb, cluster CTAs, tile columns, max CTAs); 0 = automatic
TUNINGS = [(0, 0, 0, 0), (0, 1, 256, 0), (0, 3, 512, 0), (0, 5, 256, 0), (0, 16, 256, 0), (0, 7, 512, 0),
           (48, 2, 512, 0), (0, 0, 0, 7), (0, 1, 512, 0)]


@pytest.mark.parametrize("tuning", TUNINGS, ids=[f"smem{a}-c{b}-w{c}-max{d}" for a, b, c, d in TUNINGS])
@pytest.mark.parametrize("m,n,k,g", [(1, 6144, 4096, 128), (1, 4096, 12288, 128), (4, 4096, 4096, 128),
                                     (3, 1024, 1152, 64), (8, 768, 640, 32), (13, 2048, 1024, 128),
                                     (16, 512, 2048, 256), (2, 96, 4096, 128), (1, 64, 4096, 16),
                                     (13, 256, 8192, 64), (5, 512, 3072, 256)])
def test_cluster_gemv_matches_oracle(lib, tuning, m, n, k, g):
    from ashqk import w4a16_linear

    assert lib.ashqk_gemv_set_tuning(*tuning) == 0
    try:
        plan = (ctypes.c_int * 11)()
        if lib.ashqk_gemv_cluster_plan(m, n, k, g, 0, plan) == 2:
            pytest.skip("this forced split does not fit the shared-memory budget")
        x, qw, qz, s = quantized_problem(m, n, k, g, seed=m * 31 + n + k + g)
        xd, qwd, qzd, sd = to_cuda(x, qw, qz, s)
        y = w4a16_linear(xd, qwd, qzd, sd)
        _check(x, qw, qz, s, y)
        assert torch.equal(w4a16_linear(xd, qwd, qzd, sd), y)  # fixed summation order
    finally:
        assert lib.ashqk_gemv_set_tuning(0, 0, 0, 0) == 0


@pytest.mark.parametrize("m", [1, 2, 4, 8, 16])
def test_cluster_gemv_baseline_layers(lib, m):
    """BASELINE config 2 shapes at full size with uniform q, z (the bench's distribution)."""
    from ashqk import w4a16_linear

    for n, k in ((6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288)):
        x, qw, qz, s = O.make_problem(m, n, k, 128, seed=n + k + m)
        _check(x, qw, qz, s, w4a16_linear(*to_cuda(x, qw, qz, s)))


def test_cluster_gemv_strided_views(lib):
    """Row-strided x and y, column-sliced (tensor-parallel) weight views."""
    from ashqk.kernels.w4a16_gemv import w4a16_gemv

    x, qw, qz, s = quantized_problem(4, 4096, 2048, 128, seed=3)
    xd, qwd, qzd, sd = to_cuda(x, qw, qz, s)
    wide = torch.zeros(4, 4096 + 64, dtype=torch.float16, device="cuda")
    wide[:, :2048] = xd
    y_view = w4a16_gemv(wide[:, :2048], qwd[:, 128:384], qzd[:, 128:384], sd[:, 1024:3072])
    _check(x, qw[:, 128:384], qz[:, 128:384], s[:, 1024:3072], y_view)


def test_cluster_plan_fills_the_gpu(lib):
    class Plan(ctypes.Structure):
        _fields_ = [(f, ctypes.c_int) for f in ("tile_cols", "stage_rows", "tiles", "stages_per_tile", "cluster_ctas",
                                                 "ctas", "max_stages_per_cta", "threads", "ring_stages", "stage_bytes",
                                                 "smem_bytes")]

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for n, k in ((6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288)):
        p = Plan()
        assert lib.ashqk_gemv_cluster_plan(1, n, k, 128, 0, ctypes.byref(p)) == 0
        assert 0.85 * sms <= p.ctas <= 1.65 * sms and p.smem_bytes <= 113 * 1024, (n, k, p.ctas, p.smem_bytes)


def test_no_device_errors(lib):
    bits = ctypes.c_uint(0)
    assert lib.ashqk_get_device_errors(ctypes.byref(bits), 0) == 0
    assert bits.value == 0
