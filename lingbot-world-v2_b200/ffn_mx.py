"""MXFP8 FFN matmuls with the reference's interface (kernels/ffn_mx.py:44-50, :159-182).

  prequantize_weight(w [N, K] bf16) -> (data [N, K] uint8 E4M3 codes, scales uint8)   once per weight
  mm(x [M, K] bf16, data, scales) -> [M, N] bf16                                      per call

Scales are E8M0, one per 32 values along K, in the tiled layout of lbw_mx_quantize (include/lbw.h).
This build computes the block-scaled product on the bf16 tensor pipe: the activation is quantised
and dequantised in-kernel and the weight's dequantised copy (exact in bf16) is kept next to its
codes, so the result equals an MXFP8 x MXFP8 product with fp32 accumulation.
"""
import torch

from . import kernels

K_ALIGN = 128
_DEQ = {}


def prequantize_weight(w):
    data, scales, deq = kernels.mx_quantize(w.to(torch.bfloat16).contiguous(), dequant=True)
    _DEQ[(data.data_ptr(), scales.data_ptr())] = deq
    return data, scales


def dequantized(data, scales):
    try:
        return _DEQ[(data.data_ptr(), scales.data_ptr())]
    except KeyError:
        raise ValueError("weight was not prequantised by lbw_b200.ffn_mx.prequantize_weight") from None


def mm(x, w_data, w_scales):
    """[M, K] bf16 x MXFP8 weight -> [M, N] bf16 (activation quantised to MXFP8 per 32 along K)."""
    w = dequantized(w_data, w_scales)
    _, _, xq = kernels.mx_quantize(x.to(torch.bfloat16).contiguous(), dequant=True)
    return kernels.gemm_bf16(xq, w)
