"""AWQ W4A16 storage format and its PyTorch reference arithmetic.

Public helpers with the names, signatures and results of the reference's
``ashqk/ref.py`` (MMMchou/ash-quant-kernels). They run on any device through
plain PyTorch ops and are the format layer, not the hot path: ``w4a16_linear``
never calls them.

Layout (AutoAWQ "GEMM" checkpoints, ashqk/ref.py:1-14):

    qweight : [K, N // 8]       int32   eight uint4 per word, packed along N
    qzeros  : [K // G, N // 8]  int32   same packing
    scales  : [K // G, N]       fp16
    W[k, n] = (q[k, n] - z[k // G, n]) * s[k // G, n];  y = x @ W

Within a word, nibble i (bits 4i..4i+3) holds column AWQ_ORDER[i] of the
8-column block; column j therefore sits at nibble AWQ_REVERSE_ORDER[j].
"""

from __future__ import annotations

import torch

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)
AWQ_REVERSE_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)
PACK_FACTOR = 8

# Per-device int32 shift table, cached so that unpack_awq never performs a
# host-to-device copy (which would be illegal inside CUDA-graph capture).
_shift_cache: dict = {}


def _column_shifts(device) -> torch.Tensor:
    key = torch.device(device)
    shifts = _shift_cache.get(key)
    if shifts is None:
        shifts = torch.tensor([4 * n for n in AWQ_REVERSE_ORDER], dtype=torch.int32, device=key)
        _shift_cache[key] = shifts
    return shifts


def pack_awq(x: torch.Tensor) -> torch.Tensor:
    """uint4 values [R, C] (C % 8 == 0) -> int32 [R, C // 8] in AWQ nibble order."""
    assert x.dim() == 2 and x.shape[1] % PACK_FACTOR == 0
    assert int(x.min()) >= 0 and int(x.max()) <= 15, "values must be uint4"
    rows, cols = x.shape
    blocks = x.to(torch.int64).reshape(rows, cols // PACK_FACTOR, PACK_FACTOR)
    word = torch.zeros(rows, cols // PACK_FACTOR, dtype=torch.int64, device=x.device)
    for nibble, col in enumerate(AWQ_ORDER):
        word |= blocks[..., col] << (4 * nibble)
    # Keep the 32-bit pattern; values >= 2**31 become negative int32.
    word = word - ((word >> 31) & 1) * (1 << 32)
    return word.to(torch.int32)


def unpack_awq(packed: torch.Tensor) -> torch.Tensor:
    """int32 [R, C] -> int32 [R, 8 C] of values in 0..15 (inverse of pack_awq)."""
    assert packed.dtype == torch.int32 and packed.dim() == 2
    # Arithmetic shift of a negative word is harmless: the mask keeps 4 bits.
    nibbles = (packed.unsqueeze(-1) >> _column_shifts(packed.device)) & 0xF
    return nibbles.reshape(packed.shape[0], packed.shape[1] * PACK_FACTOR)


def quantize_awq(w: torch.Tensor, group_size: int = 128):
    """Asymmetric round-to-nearest int4 quantisation of W [K, N] into AWQ tensors.

    Only the storage format of AWQ, not its activation-aware scale search.
    fp32 arithmetic in the reference's order (ashqk/ref.py:58-75), so results
    match it bit for bit. Returns (qweight, qzeros, scales).
    """
    k, n = w.shape
    assert k % group_size == 0 and n % PACK_FACTOR == 0
    groups = w.float().reshape(k // group_size, group_size, n)
    hi = groups.amax(dim=1)
    lo = groups.amin(dim=1)
    step = (hi - lo).clamp(min=1e-5) / 15.0
    zero = torch.round(-lo / step).clamp(0, 15)
    q = (torch.round(groups / step.unsqueeze(1)) + zero.unsqueeze(1)).clamp(0, 15)
    q = q.to(torch.int32).reshape(k, n)
    return pack_awq(q), pack_awq(zero.to(torch.int32)), step.to(torch.float16)


def dequantize_awq(qweight, qzeros, scales, dtype=torch.float32) -> torch.Tensor:
    """W = (q - z) * s in fp32, cast to ``dtype``; returns [K, N]."""
    q = unpack_awq(qweight)
    k = q.shape[0]
    group_size = k // scales.shape[0]
    z = unpack_awq(qzeros).repeat_interleave(group_size, dim=0)
    s = scales.float().repeat_interleave(group_size, dim=0)
    return ((q - z).float() * s).to(dtype)


def w4a16_gemm_ref(x, qweight, qzeros, scales) -> torch.Tensor:
    """Unfused baseline: dequantise to x.dtype, then a dense GEMM (cuBLAS on GPU)."""
    return x @ dequantize_awq(qweight, qzeros, scales, dtype=x.dtype)


def w4a16_gemm_fp32(x, qweight, qzeros, scales) -> torch.Tensor:
    """Correctness ground truth: x and W in fp32, matmul with TF32 disabled."""
    w = dequantize_awq(qweight, qzeros, scales, dtype=torch.float32)
    saved = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return x.float() @ w
    finally:
        torch.backends.cuda.matmul.allow_tf32 = saved
