"""The CPU oracle against the golden vectors produced by the reference itself.

tests/golden/make_golden.py ran MMMchou/ash-quant-kernels' ``ashqk/ref.py`` and its
Triton kernels (in the Triton CPU interpreter) on seeded inputs; these tests pin
oracle/awq_oracle.py (numpy) and oracle/awq_oracle.c (C) to those outputs.
"""

import os

import numpy as np
import pytest

from oracle import awq_oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "awq_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_pack_order_kat(golden):
    # tests/test_ref.py:17-23 of the reference: column j holds j + 1.
    packed = O.pack_awq(golden["kat_order_in"])
    assert np.array_equal(packed, golden["kat_order_out"])
    word = int(packed[0, 0]) & 0xFFFFFFFF
    assert [(word >> (4 * i)) & 0xF for i in range(8)] == [O.AWQ_ORDER[i] + 1 for i in range(8)]


def test_pack_sign_kat(golden):
    # tests/test_ref.py:26-31: all-15 packs to -1 and round-trips.
    packed = O.pack_awq(golden["kat_sign_in"])
    assert np.array_equal(packed, golden["kat_sign_out"]) and int(packed[0, 0]) == -1
    assert np.array_equal(O.unpack_awq(packed), golden["kat_sign_in"])


def test_roundtrip(golden):
    packed = O.pack_awq(golden["roundtrip_in"])
    assert np.array_equal(packed, golden["roundtrip_packed"])
    assert np.array_equal(O.unpack_awq(packed), golden["roundtrip_unpacked"])


@pytest.mark.parametrize("gs", [32, 64, 128])
def test_quantize_bit_exact(golden, gs):
    qw, qz, s = O.quantize_awq(golden["quant_w"], gs)
    assert np.array_equal(qw, golden[f"quant_g{gs}_qweight"])
    assert np.array_equal(qz, golden[f"quant_g{gs}_qzeros"])
    assert np.array_equal(s.view(np.uint16), golden[f"quant_g{gs}_scales"].view(np.uint16))


@pytest.mark.parametrize("gs", [32, 64, 128])
def test_dequantize_bit_exact(golden, gs):
    args = [golden[f"quant_g{gs}_{k}"] for k in ("qweight", "qzeros", "scales")]
    assert np.array_equal(O.dequantize_awq(*args).view(np.uint32), golden[f"quant_g{gs}_deq_f32"].view(np.uint32))
    assert np.array_equal(O.dequantize_awq(*args, dtype=np.float16).view(np.uint16),
                          golden[f"quant_g{gs}_deq_f16"].view(np.uint16))
    assert np.array_equal(O.c_dequantize_f32(*args).view(np.uint32), golden[f"quant_g{gs}_deq_f32"].view(np.uint32))


def _cases(golden):
    return [str(c) for c in golden["gemm_cases"]]


def test_gemm_truth_matches_reference(golden):
    for name in _cases(golden):
        x, qw, qz, s = (golden[f"{name}_{k}"] for k in ("x", "qweight", "qzeros", "scales"))
        y_true = golden[f"{name}_y_fp32"]
        # fp32 truths agree to fp32 summation-order noise.
        assert O.rel_err(O.w4a16_gemm_fp32(x, qw, qz, s), y_true) < 2e-6, name
        assert O.rel_err(O.c_gemm(x, qw, qz, s), y_true) < 2e-6, name
        # The unfused fp16 path: the reference's CPU fp16 matmul and this
        # restatement round the same fp32 sums; allow rare 1-ulp order effects.
        y_ref = O.w4a16_gemm_ref(x, qw, qz, s)
        diff = y_ref.view(np.uint16) != golden[f"{name}_y_ref"].view(np.uint16)
        assert diff.mean() < 0.01, name
        assert O.rel_err(y_ref, golden[f"{name}_y_ref"]) < 1e-4, name


def test_reference_kernels_meet_criterion(golden):
    """The reference's own Triton GEMV / v3 outputs satisfy the parity criterion
    (rel err <= 2x that of the fp16 unfused path + 1e-5) against the oracle truth:
    the criterion and the truth used for the CUDA kernels are the reference's."""
    for name in _cases(golden):
        x, qw, qz, s = (golden[f"{name}_{k}"] for k in ("x", "qweight", "qzeros", "scales"))
        y_true = O.c_gemm(x, qw, qz, s)
        e_fp16 = O.rel_err(golden[f"{name}_y_ref"], y_true)
        for impl in ("y_gemv", "y_v3"):
            assert O.rel_err(golden[f"{name}_{impl}"], y_true) <= 2 * e_fp16 + 1e-5, (name, impl)


def test_make_problem_distributions():
    x, qw, qz, s = O.make_problem(4, 64, 256, 128, seed=3)
    q = O.unpack_awq(qw)
    z = O.unpack_awq(qz)
    assert x.dtype == np.float16 and s.dtype == np.float16
    assert q.min() >= 0 and q.max() <= 15 and z.min() >= 0 and z.max() <= 15
    assert s.min() >= np.float16(0.002) and s.max() <= np.float16(0.02)


def test_bytes_model():
    # bench/bench_gemm.py:45-46 of the reference; qkv M=1 is 13.10 MB.
    assert O.w4a16_bytes(1, 6144, 4096, 128) == 1 * 4096 * 2 + 4096 * 6144 // 2 + 32 * 6144 * 2 + 32 * 6144 // 2 + 6144 * 2
    assert abs(O.w4a16_bytes(1, 6144, 4096, 128) / 1e6 - 13.10) < 0.01


@pytest.mark.parametrize("mutation", ["sequential_nibbles", "zero_point_off_by_one", "scale_of_next_group",
                                      "fp16_accumulation"])
def test_criterion_catches_planted_mistakes(golden, mutation):
    """The parity criterion has teeth: products computed with a planted mistake (in the oracle,
    on the CPU) fail it. The reference records the first of these by hand: sequential nibble
    order gives rel err 1.24 (results/v0.1-naive-findings.md:8)."""
    name = _cases(golden)[0]
    x, qw, qz, s = (golden[f"{name}_{k}"] for k in ("x", "qweight", "qzeros", "scales"))
    y_true = O.c_gemm(x, qw, qz, s)
    e_fp16 = O.rel_err(golden[f"{name}_y_ref"], y_true)
    k, g = qw.shape[0], qw.shape[0] // s.shape[0]
    q = O.unpack_awq(qw).astype(np.float32)
    z = O.unpack_awq(qz).astype(np.float32)
    if mutation == "sequential_nibbles":  # nibble i read as column i instead of AWQ_ORDER[i]
        w8 = qw.view(np.uint32)
        q = np.stack([(w8 >> np.uint32(4 * i)) & np.uint32(15) for i in range(8)], -1).reshape(k, -1)
        q = q.astype(np.float32)
    elif mutation == "zero_point_off_by_one":
        z = z + 1
    zs = np.repeat(z, g, axis=0)
    ss = np.repeat(s.astype(np.float32), g, axis=0)
    if mutation == "scale_of_next_group":
        ss = np.repeat(np.roll(s.astype(np.float32), -1, axis=0), g, axis=0)
    w = ((q - zs) * ss).astype(np.float16).astype(np.float32)
    if mutation == "fp16_accumulation":  # every partial sum rounded to fp16
        acc = np.zeros((x.shape[0], w.shape[1]), np.float16)
        for kk in range(k):
            acc = (acc + (x[:, kk:kk + 1].astype(np.float32) * w[kk]).astype(np.float16)).astype(np.float16)
        y = acc.astype(np.float32)
    else:
        y = x.astype(np.float32) @ w
    assert O.rel_err(y, y_true) > 2 * e_fp16 + 1e-5, (mutation, O.rel_err(y, y_true), e_fp16)
