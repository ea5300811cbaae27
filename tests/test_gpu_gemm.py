"""Prefill GEMM on B200 (tcgen05 + TMEM kernel, and the chunked-GEMV fallback).

* Dequantised weight tile, bit for bit: with x = the identity, y = x @ W is W
  itself (one non-zero product per output), so the fp16 output must equal
  ``dequantize_awq(..., fp16)`` of the oracle exactly.
* Parity (the reference's criterion, tests/test_gemm.py:106-111 of
  MMMchou/ash-quant-kernels): rel_err <= 2 * rel_err(cuBLAS fp16) + 1e-5 against
  the oracle's fp32 truth, over group sizes, both tile widths, ragged M, strided
  operands, and the prefill configurations of the benchmark (M up to 2048 on the
  Qwen3-8B gate_up and down shapes, truth from fp32 GEMM on the GPU there).
* Both GEMM kernels agree, graph capture works, no kernel reports a timeout.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import awq_oracle as O
from tests._helpers import quantized_problem, rel_err, to_cuda

pytestmark = pytest.mark.gpu


def _lib():
    from ashqk import _ext

    lib = ctypes.CDLL(_ext.C_LIBRARY)
    lib.ashqk_get_device_errors.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]
    return lib


@pytest.fixture(params=[3, 4, 1], ids=["tcgen05-1cta", "tcgen05-pair", "chunked-gemv"])
def gemm_kernel(request):
    """Run a test once per prefill GEMM kernel (ashqk_set_gemm_kernel), then restore auto."""
    lib = _lib()
    assert lib.ashqk_set_gemm_kernel(request.param) == 0
    yield request.param
    assert lib.ashqk_set_gemm_kernel(0) == 0


def _skip_unless_eligible(impl, m, n):
    if impl == 4 and not (m > 128 and n % 256 == 0):
        pytest.skip("the CTA-pair kernel takes M > 128 and N % 256 == 0")


def _gemm(x, qw, qz, s):
    from ashqk.kernels.w4a16_gemm_v3 import w4a16_gemm_v3

    return w4a16_gemm_v3(x, qw, qz, s)


def _check(x, qw, qz, s, y, y_true=None):
    if y_true is None:
        y_true = O.c_gemm(x, qw, qz, s)
    w16 = torch.from_numpy(O.dequantize_awq(qw, qz, s, np.float16)).cuda()
    e_cublas = rel_err(torch.from_numpy(x).cuda() @ w16, y_true)
    e = rel_err(y, y_true)
    assert e <= 2 * e_cublas + 1e-5, (e, e_cublas)


@pytest.mark.parametrize("g", [16, 32, 64, 128])
@pytest.mark.parametrize("n", [256, 384])
def test_dequant_tile_bit_exact(n, g, gemm_kernel):
    k = 256
    _skip_unless_eligible(gemm_kernel, k, n)
    _, qw, qz, s = quantized_problem(1, n, k, g, seed=n + g)
    x = np.eye(k, dtype=np.float16)
    y = _gemm(*to_cuda(x, qw, qz, s))
    torch.cuda.synchronize()
    w = O.dequantize_awq(qw, qz, s, np.float16)
    assert np.array_equal(y.cpu().numpy().view(np.uint16), w.view(np.uint16))


@pytest.mark.parametrize("m,n,k,g", [
    (17, 256, 512, 128),      # smallest M the dispatcher sends here
    (128, 512, 1024, 64),
    (129, 768, 512, 32),      # ragged M, 128-column tiles (768 % 256 != 0 -> 256 tiles would not divide)
    (200, 1024, 2048, 16),
    (256, 4096, 4096, 128),
    (300, 384, 1024, 256),
    (512, 2048, 1024, 128),
])
def test_gemm_parity(m, n, k, g, gemm_kernel):
    _skip_unless_eligible(gemm_kernel, m, n)
    x, qw, qz, s = quantized_problem(m, n, k, g, seed=m + n + k + g)
    y = _gemm(*to_cuda(x, qw, qz, s))
    torch.cuda.synchronize()
    _check(x, qw, qz, s, y)


def test_strided_operands():
    """Row-strided x and y, column-sliced weights (a tensor-parallel shard) through the tcgen05 kernel."""
    from ashqk.ops import w4a16_linear_into

    m, n, k, g = 160, 1024, 1024, 128
    x, qw, qz, s = quantized_problem(m, 2 * n, k, g, seed=3)
    xd, qwd, qzd, sd = to_cuda(x, qw, qz, s)
    xpad = torch.zeros(m, k + 64, dtype=torch.float16, device="cuda")
    xpad[:, :k] = xd
    xs = xpad[:, :k]
    half = n // 8
    qw_s, qz_s, s_s = qwd[:, half:], qzd[:, half:], sd[:, n:]
    out = torch.full((m, n + 128), float("nan"), dtype=torch.float16, device="cuda")
    y = w4a16_linear_into(xs, qw_s, qz_s, s_s, out[:, :n])
    torch.cuda.synchronize()
    assert torch.isnan(out[:, n:]).all()  # nothing written outside the view
    _check(x, qw[:, half:], qz[:, half:], s[:, n:], y)


@pytest.mark.parametrize("m", [128, 512, 2048])
@pytest.mark.parametrize("layer", [("gate_up", 24576, 4096), ("down", 4096, 12288)])
def test_prefill_configs(layer, m):
    """The benchmark's prefill shapes: uniform q, z, scales ~ U(0.002, 0.02), G=128; fp32 truth on the GPU."""
    _, n, k = layer
    x, qw, qz, s = O.make_problem(m, n, k, 128, seed=m + n)
    xd, qwd, qzd, sd = to_cuda(x, qw, qz, s)
    y = _gemm(xd, qwd, qzd, sd)
    from ashqk import _ext

    w32 = _ext.ops().dequantize_awq(qwd, qzd, sd, torch.float32)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        y_true = xd.float() @ w32
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    y16 = xd @ w32.half()
    e_cublas = float((y16.float() - y_true).norm() / y_true.norm())
    e = float((y.float() - y_true).norm() / y_true.norm())
    assert e <= 2 * e_cublas + 1e-5, (e, e_cublas)


def test_kernels_agree():
    lib = _lib()
    m, n, k, g = 320, 2048, 2048, 128
    x, qw, qz, s = quantized_problem(m, n, k, g, seed=5)
    args = to_cuda(x, qw, qz, s)
    out = {}
    for impl in (1, 3, 4):
        assert lib.ashqk_set_gemm_kernel(impl) == 0
        out[impl] = _gemm(*args).float()
    assert lib.ashqk_set_gemm_kernel(0) == 0
    for impl in (3, 4):
        diff = float((out[1] - out[impl]).norm() / out[1].norm())
        assert diff < 2e-3, (impl, diff)  # different fp32 summation orders, same fp16 rounding
    # the one-CTA and pair kernels run the same MMA sequence per output element
    assert float((out[3] - out[4]).norm() / out[3].norm()) < 2e-3


def test_unsupported_shape_when_forced():
    """Forcing tcgen05 on a shape it does not take is an error, not a silent fallback."""
    lib = _lib()
    x, qw, qz, s = quantized_problem(40, 1000, 512, 64, seed=6)
    for impl in (2, 3, 4):
        assert lib.ashqk_set_gemm_kernel(impl) == 0
        try:
            with pytest.raises(RuntimeError):
                _gemm(*to_cuda(x, qw, qz, s))
        finally:
            assert lib.ashqk_set_gemm_kernel(0) == 0
    # the pair kernel also refuses M <= 128 when forced
    x2, qw2, qz2, s2 = quantized_problem(64, 512, 512, 64, seed=7)
    assert lib.ashqk_set_gemm_kernel(4) == 0
    try:
        with pytest.raises(RuntimeError):
            _gemm(*to_cuda(x2, qw2, qz2, s2))
    finally:
        assert lib.ashqk_set_gemm_kernel(0) == 0
    y = _gemm(*to_cuda(x, qw, qz, s))  # auto: the chunked GEMV takes it
    torch.cuda.synchronize()
    _check(x, qw, qz, s, y)


def test_graph_capture_and_replay():
    from ashqk import w4a16_linear

    m, n, k, g = 256, 1024, 1024, 128
    x, qw, qz, s = quantized_problem(m, n, k, g, seed=8)
    xd, qwd, qzd, sd = to_cuda(x, qw, qz, s)
    y0 = w4a16_linear(xd, qwd, qzd, sd)
    torch.cuda.synchronize()
    g_ = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_):
        y = w4a16_linear(xd, qwd, qzd, sd)
    for _ in range(3):
        g_.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, y0)  # deterministic: no split-K, fixed tile order


def test_no_device_errors():
    lib = _lib()
    bits = ctypes.c_uint(0)
    assert lib.ashqk_get_device_errors(ctypes.byref(bits), 1) == 0
    assert bits.value == 0
