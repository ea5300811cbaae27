"""ashqk.ref (the format layer of the package) against the golden vectors and the oracle.

Mirrors the format tests of the reference (tests/test_ref.py:17-52): nibble
order, sign bit, round trip, RTN error bound -- plus bit-exact agreement with
the reference's own outputs recorded in tests/golden/awq_golden.npz.
"""

import os

import numpy as np
import pytest
import torch

import ashqk
from ashqk.ref import AWQ_ORDER, dequantize_awq, pack_awq, quantize_awq, unpack_awq
from oracle import awq_oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "awq_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_public_names():
    for name in ("w4a16_linear", "AWQ_ORDER", "AWQ_REVERSE_ORDER", "dequantize_awq", "pack_awq", "quantize_awq",
                 "unpack_awq", "w4a16_gemm_fp32", "w4a16_gemm_ref"):
        assert hasattr(ashqk, name), name
    assert ashqk.GEMV_MAX_M == 16


def test_pack_layout_matches_awq_order():
    x = torch.arange(1, 9, dtype=torch.int32).view(1, 8)
    word = int(pack_awq(x)[0, 0]) & 0xFFFFFFFF
    assert [(word >> (4 * i)) & 0xF for i in range(8)] == [AWQ_ORDER[i] + 1 for i in range(8)]


def test_pack_sign_bit():
    x = torch.full((2, 8), 15, dtype=torch.int32)
    p = pack_awq(x)
    assert p.dtype == torch.int32 and int(p[0, 0]) == -1
    assert torch.equal(unpack_awq(p), x)


@pytest.mark.parametrize("shape", [(1, 8), (64, 128), (4096, 512)])
def test_pack_unpack_roundtrip(shape):
    g = torch.Generator().manual_seed(0)
    x = torch.randint(0, 16, shape, dtype=torch.int32, generator=g)
    assert torch.equal(unpack_awq(pack_awq(x)), x)
    assert np.array_equal(pack_awq(x).numpy(), O.pack_awq(x.numpy()))


@pytest.mark.parametrize("group_size", [32, 64, 128])
def test_quantize_error_bound(group_size):
    g = torch.Generator().manual_seed(0)
    k, n = 512, 256
    w = torch.randn(k, n, generator=g)
    qw, qz, s = quantize_awq(w, group_size)
    assert qw.shape == (k, n // 8) and qz.shape == (k // group_size, n // 8)
    assert s.shape == (k // group_size, n) and s.dtype == torch.float16
    step = s.float().repeat_interleave(group_size, dim=0)
    assert ((w - dequantize_awq(qw, qz, s)).abs() <= step * 1.01).all()


@pytest.mark.parametrize("gs", [32, 64, 128])
def test_matches_reference_bit_exact(golden, gs):
    w = torch.from_numpy(golden["quant_w"])
    qw, qz, s = quantize_awq(w, gs)
    assert np.array_equal(qw.numpy(), golden[f"quant_g{gs}_qweight"])
    assert np.array_equal(qz.numpy(), golden[f"quant_g{gs}_qzeros"])
    assert np.array_equal(s.numpy().view(np.uint16), golden[f"quant_g{gs}_scales"].view(np.uint16))
    assert np.array_equal(dequantize_awq(qw, qz, s).numpy().view(np.uint32),
                          golden[f"quant_g{gs}_deq_f32"].view(np.uint32))
    assert np.array_equal(dequantize_awq(qw, qz, s, torch.float16).numpy().view(np.uint16),
                          golden[f"quant_g{gs}_deq_f16"].view(np.uint16))


def test_gemm_helpers_match_golden(golden):
    for name in [str(c) for c in golden["gemm_cases"]][:6]:
        x, qw, qz, s = (torch.from_numpy(golden[f"{name}_{k}"]) for k in ("x", "qweight", "qzeros", "scales"))
        y = ashqk.w4a16_gemm_fp32(x, qw, qz, s)
        assert O.rel_err(y.numpy(), golden[f"{name}_y_fp32"]) < 2e-6
        yr = ashqk.w4a16_gemm_ref(x, qw, qz, s)
        assert yr.dtype == torch.float16 and O.rel_err(yr.numpy(), golden[f"{name}_y_ref"]) < 1e-4


def test_kernel_shims_validate_like_reference():
    """Shape errors raise AssertionError in the shim, before any native call."""
    from ashqk.kernels.w4a16_gemv import w4a16_gemv
    from ashqk.kernels.w4a16_gemm_v3 import w4a16_gemm_v3

    x = torch.zeros(2, 256, dtype=torch.float16)
    qw = torch.zeros(256, 8, dtype=torch.int32)
    qz = torch.zeros(2, 8, dtype=torch.int32)
    s = torch.zeros(2, 64, dtype=torch.float16)
    with pytest.raises(AssertionError):
        w4a16_gemv(x.float(), qw, qz, s)
    with pytest.raises(AssertionError):
        w4a16_gemm_v3(x, qw[:128], qz, s)
    with pytest.raises(AssertionError):
        w4a16_gemv(x, qw, qz, s, {"not_a_key": 1})


def test_no_cpu_fallback():
    """The kernels refuse CPU tensors loudly instead of computing on the host."""
    from ashqk import _ext

    x = torch.zeros(1, 256, dtype=torch.float16)
    qw = torch.zeros(256, 8, dtype=torch.int32)
    qz = torch.zeros(2, 8, dtype=torch.int32)
    s = torch.zeros(2, 64, dtype=torch.float16)
    if not os.path.exists(_ext.TORCH_BINDING):
        with pytest.raises(ImportError):
            ashqk.w4a16_linear(x, qw, qz, s)
    else:
        with pytest.raises((RuntimeError, NotImplementedError)):
            ashqk.w4a16_linear(x, qw, qz, s)
