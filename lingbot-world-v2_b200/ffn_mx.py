"""MXFP8 FFN matmuls with the reference's interface (kernels/ffn_mx.py:44-50, :159-182).

  prequantize_weight(w [N, K] bf16) -> (data [N, K] uint8 E4M3 codes, scales uint8)   once per weight
  mm(x [M, K] bf16, data, scales) -> [M, N] bf16                                      per call

Scales are E8M0, one per 32 values along K, in the tiled layout of lbw_mx_quantize (include/lbw.h).
mm quantises the activation to MXFP8 (lbw_mx_quantize) and runs the block-scaled tcgen05 GEMM
(lbw_mx_linear, kind::mxf8f6f4) with fp32 accumulation and a bf16 result.
"""
import torch

from . import kernels

K_ALIGN = 128


def prequantize_weight(w):
    data, scales, _ = kernels.mx_quantize(w.to(torch.bfloat16).contiguous())
    return data, scales


def mm(x, w_data, w_scales):
    """[M, K] bf16 x MXFP8 weight -> [M, N] bf16 (activation quantised to MXFP8 per 32 along K)."""
    xd, xs, _ = kernels.mx_quantize(x.to(torch.bfloat16).contiguous())
    return kernels.mx_linear(xd, xs, w_data, w_scales)
