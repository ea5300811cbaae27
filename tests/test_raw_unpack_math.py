"""Arithmetic of the decode GEMV's per-group zero-point correction, emulated in numpy (no GPU).

The cluster-split kernel (csrc/gemv_cluster.cu) feeds the magic-number halves 1024 + q (low-nibble
columns 0, 1, 4, 5 of a packed word) and 1024 + 16 q (high-nibble columns 2, 3, 6, 7) to the mma
without subtracting the zero point, accumulates each group's sum of x with an mma against ones,
and corrects once per group:

    sum x (q - z) = f * dot - (c + z) * sum x,   f = 1, c = 1024 (low);  f = 1/16, c = 64 (high)

The emulation keeps the kernel's order of operations in fp32 (16-row mma chunks added to a running
fp32 group partial, the correction, the scale fma, the sum over groups) and checks that (1) the
identity holds exactly in exact arithmetic, and (2) with fp32 rounding the result stays within the
reference's parity criterion (rel err <= 2 x cuBLAS fp16 + 1e-5 vs fp32 truth,
tests/test_gemm.py:1-7 of the reference), on N(0,1) activations and on activations with outlier
channels.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import awq_oracle as O
from tests._helpers import quantized_problem

LOW_COLS = np.array([c % 4 < 2 for c in range(8)])  # columns 0, 1, 4, 5 of every packed word


def _unpacked(qw, qz):
    return O.unpack_awq(qw).astype(np.int64), O.unpack_awq(qz).astype(np.int64)


def _raw_gemv(x, qw, qz, s, g):
    """The kernel's arithmetic (uncorrected mma, ones-mma, per-group correction): fp16 y [M, N]."""
    q, z = _unpacked(qw, qz)
    k, n = q.shape
    low = np.tile(LOW_COLS, n // 8)
    magic = np.where(low, 1024 + q, 1024 + 16 * q).astype(np.float32)     # exact in fp16 and fp32
    f = np.where(low, np.float32(1), np.float32(1 / 16)).astype(np.float32)
    c = np.where(low, np.float32(1024), np.float32(64)).astype(np.float32)
    x32 = x.astype(np.float32)
    m = x.shape[0]
    acc = np.zeros((m, n), np.float32)
    for gi in range(k // g):
        part = np.zeros((m, n), np.float32)
        psx = np.zeros((m, 1), np.float32)
        for k0 in range(gi * g, (gi + 1) * g, 16):  # one mma per 16 rows: exact products, fp32 sum
            ch = slice(k0, k0 + 16)
            part = (part + (x32[:, ch].astype(np.float64) @ magic[ch].astype(np.float64)).astype(np.float32))
            psx = (psx + x32[:, ch].astype(np.float64).sum(1, keepdims=True).astype(np.float32))
        zk = (c + z[gi].astype(np.float32)).astype(np.float32)
        corrected = (part * f - (zk * psx).astype(np.float32)).astype(np.float32)
        acc = (acc + s[gi].astype(np.float32) * corrected).astype(np.float32)
    return acc.astype(np.float16)


def test_identity_is_exact():
    """In exact (integer) arithmetic the per-group correction gives sum x (q - z) for every column."""
    rng = np.random.default_rng(0)
    k, n, g = 256, 64, 128
    q = rng.integers(0, 16, (k, n))
    z = rng.integers(0, 16, (k // g, n))
    x = rng.integers(-50, 50, (3, k))
    low = np.tile(LOW_COLS, n // 8)
    magic = np.where(low, 1024 + q, 1024 + 16 * q)
    for gi in range(k // g):
        r = slice(gi * g, (gi + 1) * g)
        dot = x[:, r] @ magic[r]
        sx = x[:, r].sum(1, keepdims=True)
        corrected16 = np.where(low, 16 * dot - 16 * (1024 + z[gi]) * sx, dot - 16 * (64 + z[gi]) * sx)
        assert np.array_equal(corrected16, 16 * (x[:, r] @ (q[r] - z[gi])))


def test_nibble_columns_match_awq_order():
    """Low nibbles of the byte-permuted words are the columns the kernel treats as low (0, 1, 4, 5):
    nibble i of a word holds column AWQ_ORDER[i] (ashqk/ref.py:20-21); the prmt 0x6420 / 0x7531
    selections put nibbles {0, 4} / {2, 6} (columns 0, 1 / 4, 5) at the low positions of each byte
    pair, so LOP3 with 0x000F000F yields them unscaled."""
    order = list(O.AWQ_ORDER)
    lo_bytes = {0x6420: (0, 2), 0x7531: (1, 3)}
    seen_low, seen_high = set(), set()
    for sel, (b_lo, b_hi) in lo_bytes.items():
        # Byte b of a word holds nibbles 2b (low) and 2b + 1 (high). The permute puts bytes b_lo
        # and b_hi of each row's word at T's bytes 0 and 1; T and T >> 8 then expose each byte's
        # low nibble to the 0x000F000F mask and its high nibble to 0x00F000F0.
        low = {order[2 * b_lo], order[2 * b_hi]}
        high = {order[2 * b_lo + 1], order[2 * b_hi + 1]}
        assert all(LOW_COLS[c] for c in low) and not any(LOW_COLS[c] for c in high), (hex(sel), low, high)
        seen_low |= low
        seen_high |= high
    assert seen_low | seen_high == set(range(8))


@pytest.mark.parametrize("m,outliers", [(1, False), (4, False), (16, False), (1, True), (8, True)])
def test_fp32_rounding_stays_within_parity(m, outliers):
    n, k, g = 1024, 4096, 128
    x, qw, qz, s = quantized_problem(m, n, k, g, seed=100 + m)
    if outliers:  # a few activation channels two orders of magnitude larger (LLM-like)
        rng = np.random.default_rng(7)
        ch = rng.choice(k, 8, replace=False)
        x = x.astype(np.float32)
        x[:, ch] *= 60.0
        x = x.astype(np.float16)
    y_true = O.w4a16_gemm_fp64(x, qw, qz, s)
    w16 = O.dequantize_awq(qw, qz, s, np.float16)
    y_cublas = (x.astype(np.float32) @ w16.astype(np.float32)).astype(np.float16)
    e_cublas = O.rel_err(y_cublas.astype(np.float32), y_true)
    y_raw = _raw_gemv(x, qw, qz, s, g)
    e_raw = O.rel_err(y_raw.astype(np.float32), y_true)
    assert e_raw <= 2 * e_cublas + 1e-5, (e_raw, e_cublas)
    # The correction's cancellation costs little next to the fp16 output rounding.
    assert e_raw <= 1.5 * e_cublas, (e_raw, e_cublas)
