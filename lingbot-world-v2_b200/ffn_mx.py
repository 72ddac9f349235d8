"""MX FFN matmuls with the reference's interface (kernels/ffn_mx.py:44-50, :159-182).

  prequantize_weight(w [N, K] bf16) -> (data [N, K] uint8 codes, scales uint8)   once per weight
  mm(x [M, K] bf16, data, scales) -> [M, N] bf16                                per call

Scales are E8M0, one per 32 values along K, in the tiled layout of lbw_mx_quantize (include/lbw.h).
mm quantises the activation to the same MX format (lbw_mx_quantize_fmt) and runs the block-scaled tcgen05 GEMM
(lbw_mx_linear_fmt: kind::mxf8f6f4 for E4M3 / E5M2, kind::mxf4 for E2M1) with fp32 accumulation and a bf16
result.

The element format follows the reference's LINGBOT_MX_FP8 (kernels/ffn_mx.py:8,18: float8_e4m3fn, the default, or
float8_e5m2), read once at import as there; fmt= overrides it per call ("e4m3", "e5m2", or "e2m1" for MXFP4 with
two codes per byte).
"""
import os

import torch

from . import kernels

K_ALIGN = 128
_FMT_OF_DTYPE = {"float8_e4m3fn": "e4m3", "float8_e5m2": "e5m2"}
FP8 = os.environ.get("LINGBOT_MX_FP8", "float8_e4m3fn")
if FP8 not in _FMT_OF_DTYPE:
    raise ValueError(f"LINGBOT_MX_FP8={FP8!r}: expected one of {sorted(_FMT_OF_DTYPE)}")
FMT = _FMT_OF_DTYPE[FP8]


def prequantize_weight(w, fmt=None):
    data, scales, _ = kernels.mx_quantize(w.to(torch.bfloat16).contiguous(), fmt=fmt or FMT)
    return data, scales


def mm(x, w_data, w_scales, fmt=None):
    """[M, K] bf16 x MX weight -> [M, N] bf16 (activation quantised to the same format per 32 along K)."""
    f = fmt or FMT
    xd, xs, _ = kernels.mx_quantize(x.to(torch.bfloat16).contiguous(), fmt=f)
    return kernels.mx_linear(xd, xs, w_data, w_scales, fmt=f)
