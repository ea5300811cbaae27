"""CPU oracle for the AWQ W4A16 linear path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it. The CUDA path in ``ashqk`` never calls it and has
no CPU fallback.

It restates, in numpy, the reference's PyTorch format code ``ashqk/ref.py``
(MMMchou/ash-quant-kernels). Each function cites the reference lines it follows.
Parity is pinned: ``tests/test_oracle.py`` checks every function here against the
golden vectors in ``tests/golden/awq_golden.npz``, which
``tests/golden/make_golden.py`` produced by running the reference itself.

Storage format (ashqk/ref.py:1-14, AutoAWQ "GEMM" tensors):
    qweight  int32 [K, N/8]    eight uint4 per word, packed along N
    qzeros   int32 [K/G, N/8]  same packing
    scales   fp16  [K/G, N]
    W[k, n] = (q[k, n] - z[k // G, n]) * s[k // G, n];  y = x @ W
Inside a word, nibble i (bits 4i..4i+3) holds column AWQ_ORDER[i] of its
8-column block (ashqk/ref.py:20-21).
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

# ashqk/ref.py:20-22
AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)          # nibble -> column within the 8-column block
AWQ_REVERSE_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)  # column -> nibble
PACK_FACTOR = 8

_NIBBLE_SHIFT = np.array(AWQ_REVERSE_ORDER, dtype=np.uint32) * 4  # shift that extracts column j


def pack_awq(q: np.ndarray) -> np.ndarray:
    """uint4 values [R, C] -> int32 [R, C/8] in AWQ nibble order (ashqk/ref.py:25-36)."""
    q = np.asarray(q)
    if q.ndim != 2 or q.shape[1] % PACK_FACTOR:
        raise ValueError("pack_awq wants a 2-D array whose column count is a multiple of 8")
    if q.size and (q.min() < 0 or q.max() > 15):
        raise ValueError("values must be uint4 (0..15)")
    r, c = q.shape
    blocks = q.astype(np.uint32).reshape(r, c // PACK_FACTOR, PACK_FACTOR)
    word = np.zeros((r, c // PACK_FACTOR), dtype=np.uint32)
    for nibble, col in enumerate(AWQ_ORDER):
        word |= blocks[..., col] << np.uint32(4 * nibble)
    # Same bit pattern, read as signed: nibble 7 may set bit 31 (ashqk/ref.py:34-35).
    return word.view(np.int32)


def unpack_awq(packed: np.ndarray) -> np.ndarray:
    """int32 [R, C] -> int32 [R, 8C] with values 0..15 (ashqk/ref.py:49-55)."""
    packed = np.asarray(packed)
    if packed.dtype != np.int32 or packed.ndim != 2:
        raise ValueError("unpack_awq wants a 2-D int32 array")
    u = packed.view(np.uint32)
    vals = (u[..., None] >> _NIBBLE_SHIFT) & np.uint32(0xF)
    return vals.reshape(packed.shape[0], -1).astype(np.int32)


def quantize_awq(w: np.ndarray, group_size: int = 128):
    """Asymmetric round-to-nearest int4 quantisation in AWQ layout (ashqk/ref.py:58-75).

    All arithmetic is fp32, in the reference's order, and rounding is half-to-even
    like ``torch.round``, so the outputs are bit-identical to the reference's.
    """
    w = np.asarray(w, dtype=np.float32)
    k, n = w.shape
    if k % group_size or n % PACK_FACTOR:
        raise ValueError("K must be a multiple of group_size and N a multiple of 8")
    wg = w.reshape(k // group_size, group_size, n)
    w_max = wg.max(axis=1)
    w_min = wg.min(axis=1)
    scales = np.maximum(w_max - w_min, np.float32(1e-5)) / np.float32(15.0)
    zeros = np.clip(np.round(-w_min / scales), 0, 15)
    q = np.round(wg / scales[:, None, :]) + zeros[:, None, :]
    q = np.clip(q, 0, 15).astype(np.int32).reshape(k, n)
    return pack_awq(q), pack_awq(zeros.astype(np.int32)), scales.astype(np.float16)


def dequantize_awq(qweight, qzeros, scales, dtype=np.float32) -> np.ndarray:
    """W = (q - z) * s computed in fp32, then cast to ``dtype`` (ashqk/ref.py:78-86)."""
    q = unpack_awq(qweight)
    z = unpack_awq(qzeros)
    k, _ = q.shape
    group_size = k // scales.shape[0]
    z = np.repeat(z, group_size, axis=0)
    s = np.repeat(np.asarray(scales).astype(np.float32), group_size, axis=0)
    return ((q - z).astype(np.float32) * s).astype(dtype)


def w4a16_gemm_fp32(x, qweight, qzeros, scales) -> np.ndarray:
    """Ground truth: x (as fp32) @ W (fp32) (ashqk/ref.py:95-103)."""
    w = dequantize_awq(qweight, qzeros, scales, np.float32)
    return np.asarray(x).astype(np.float32) @ w


def w4a16_gemm_fp64(x, qweight, qzeros, scales) -> np.ndarray:
    """Higher-precision truth (fp64 accumulation) used to bound the fp32 truth's own error."""
    w = dequantize_awq(qweight, qzeros, scales, np.float32).astype(np.float64)
    return np.asarray(x).astype(np.float64) @ w


def w4a16_gemm_ref(x, qweight, qzeros, scales) -> np.ndarray:
    """Unfused baseline (ashqk/ref.py:89-92): dequantise to fp16, fp16 GEMM.

    An fp16 GEMM accumulates in fp32 and rounds the output once to fp16; that is
    what this restatement does.
    """
    w = dequantize_awq(qweight, qzeros, scales, np.float16).astype(np.float32)
    return (np.asarray(x).astype(np.float32) @ w).astype(np.float16)


def rel_err(y, y_true) -> float:
    """Relative Frobenius error, the reference's parity metric (tests/test_gemm.py:42-43)."""
    y = np.asarray(y, dtype=np.float64)
    y_true = np.asarray(y_true, dtype=np.float64)
    return float(np.linalg.norm(y - y_true) / np.linalg.norm(y_true))


def w4a16_bytes(m: int, n: int, k: int, g: int) -> int:
    """Algorithmic HBM bytes of one W4A16 linear call (bench/bench_gemm.py:45-46)."""
    return m * k * 2 + k * n // 2 + (k // g) * n * 2 + (k // g) * n // 2 + m * n * 2


def make_problem(m: int, n: int, k: int, group_size: int, seed: int = 0):
    """Seeded synthetic AWQ problem with the distributions the benchmark configs name.

    x fp16 ~ N(0, 1); q and z uniform over 0..15; scales fp16 ~ U(0.002, 0.02).
    Generated with numpy's PCG64 so CPU and GPU sides see the same bytes.
    """
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32).astype(np.float16)
    q = rng.integers(0, 16, size=(k, n), dtype=np.int32)
    z = rng.integers(0, 16, size=(k // group_size, n), dtype=np.int32)
    s = rng.uniform(0.002, 0.02, size=(k // group_size, n)).astype(np.float16)
    return x, pack_awq(q), pack_awq(z), s


# ---------------------------------------------------------------------------
# C restatement (oracle/awq_oracle.c), loaded through ctypes. It is the fast
# multi-threaded CPU path used for full-size checks and the timed CPU baseline.
# ---------------------------------------------------------------------------

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libawq_oracle.so")
_lib = None


def c_oracle():
    """Load oracle/_build/libawq_oracle.so (built by ``make -C oracle``)."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise FileNotFoundError(f"{_LIB_PATH} missing: run `make -C oracle`")
        lib = ctypes.CDLL(_LIB_PATH)
        i64 = ctypes.c_int64
        vp = ctypes.c_void_p
        lib.awq_oracle_dequant_f32.argtypes = [vp, vp, vp, vp, i64, i64, i64]
        lib.awq_oracle_dequant_f32.restype = ctypes.c_int
        lib.awq_oracle_gemm.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, i64, ctypes.c_int]
        lib.awq_oracle_gemm.restype = ctypes.c_int
        lib.awq_oracle_threads.argtypes = []
        lib.awq_oracle_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def c_dequantize_f32(qweight, qzeros, scales) -> np.ndarray:
    qweight = np.ascontiguousarray(qweight, dtype=np.int32)
    qzeros = np.ascontiguousarray(qzeros, dtype=np.int32)
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    k = qweight.shape[0]
    n = qweight.shape[1] * 8
    g = k // scales.shape[0]
    out = np.empty((k, n), dtype=np.float32)
    rc = c_oracle().awq_oracle_dequant_f32(_ptr(qweight), _ptr(qzeros), _ptr(scales), _ptr(out), k, n, g)
    if rc:
        raise ValueError(f"awq_oracle_dequant_f32 failed ({rc})")
    return out


def c_gemm(x, qweight, qzeros, scales, out_fp16: bool = False) -> np.ndarray:
    """y = x @ W with W dequantised in fp32 and fp64 accumulation (C restatement).

    ``out_fp16`` rounds the fp64 result once to fp16; otherwise returns fp32.
    """
    x = np.ascontiguousarray(x, dtype=np.float16)
    qweight = np.ascontiguousarray(qweight, dtype=np.int32)
    qzeros = np.ascontiguousarray(qzeros, dtype=np.int32)
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    m, k = x.shape
    n = qweight.shape[1] * 8
    g = k // scales.shape[0]
    y = np.empty((m, n), dtype=np.float64)
    rc = c_oracle().awq_oracle_gemm(_ptr(x), _ptr(qweight), _ptr(qzeros), _ptr(scales), _ptr(y),
                                    m, n, k, g, 0)
    if rc:
        raise ValueError(f"awq_oracle_gemm failed ({rc})")
    return y.astype(np.float16) if out_fp16 else y.astype(np.float32)
