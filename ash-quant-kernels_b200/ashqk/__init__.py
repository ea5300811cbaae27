"""ashqk on B200: AWQ-format W4A16 linear layers with hand-written sm_100a kernels.

Same public names as MMMchou/ash-quant-kernels (ashqk/__init__.py:1-24): the
dispatcher ``w4a16_linear`` and the format helpers of ``ashqk.ref``.
"""

from .ops import GEMV_MAX_M, w4a16_linear
from .ref import (
    AWQ_ORDER,
    AWQ_REVERSE_ORDER,
    dequantize_awq,
    pack_awq,
    quantize_awq,
    unpack_awq,
    w4a16_gemm_fp32,
    w4a16_gemm_ref,
)

__all__ = [
    "w4a16_linear",
    "GEMV_MAX_M",
    "AWQ_ORDER",
    "AWQ_REVERSE_ORDER",
    "dequantize_awq",
    "pack_awq",
    "quantize_awq",
    "unpack_awq",
    "w4a16_gemm_fp32",
    "w4a16_gemm_ref",
]
__version__ = "0.1.0"
