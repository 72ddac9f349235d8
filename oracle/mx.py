"""MXFP8 (E4M3 elements, E8M0 shared scale per 32 values) quantise-dequantise emulation.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Written from the OCP Microscaling Formats (MX) v1.0 specification, section 6.3 (conversion):
    X = 2 ** (floor(log2(max_i |V_i|)) - emax_elem),   emax_elem = 8 for E4M3 (largest normal 448)
    P_i = quantize_E4M3(V_i / X)   round-to-nearest-even, saturating to +-448
and X is clamped to the E8M0 range [2^-127, 2^127]; an all-zero block takes X = 2^-127.

The reference quantises with nkilib's quantize_block_mxfp8_kernel / matmul_mxfp8
(kernels/ffn_mx.py:14-15, :44-50, :159-182), a Neuron SDK library that is not vendored and not
pinned; its weight padding of K to 512 (ffn_mx.K_ALIGN, :20) adds zero blocks only and does not
change any product.
"""
import torch

BLOCK = 32
E4M3_MAX = 448.0
EMAX_E4M3 = 8


def shared_exponent(amax: torch.Tensor) -> torch.Tensor:
    """floor(log2(amax)) - 8, clamped to [-127, 127]; -127 where amax == 0."""
    _, e = torch.frexp(amax.float())          # amax = m * 2**e, m in [0.5, 1)
    s = (e - 1 - EMAX_E4M3).clamp(-127, 127)
    return torch.where(amax > 0, s, torch.full_like(s, -127))


def quantize(x: torch.Tensor):
    """x [..., K] (K % 32 == 0) -> (E4M3 codes as float8_e4m3fn [..., K], exponents int32 [..., K/32])."""
    k = x.shape[-1]
    assert k % BLOCK == 0, k
    xb = x.float().reshape(*x.shape[:-1], k // BLOCK, BLOCK)
    s = shared_exponent(xb.abs().amax(dim=-1, keepdim=True))
    q = torch.ldexp(xb, (-s).float()).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.reshape(x.shape), s.squeeze(-1).to(torch.int32)


def dequantize(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    k = q.shape[-1]
    qb = q.float().reshape(*q.shape[:-1], k // BLOCK, BLOCK)
    return torch.ldexp(qb, s.float().unsqueeze(-1)).reshape(q.shape)


def qdq(x: torch.Tensor) -> torch.Tensor:
    """Quantise-dequantise along the last dim; returns fp32 values (exact in bf16)."""
    q, s = quantize(x)
    return dequantize(q, s)


def sf_offset(r, j, k_cols):
    """Byte offset of scale (row r, block column j) in the tiled scale layout of the GPU library:
    512-byte atoms of 128 rows x 4 scales, row-block major; row r = r0 + 32*r1 at 16*r0 + 4*r1 + j%4."""
    atoms_per_rowblock = k_cols // 128
    atom = (r // 128) * atoms_per_rowblock + j // 4
    rr = r % 128
    return atom * 512 + 16 * (rr % 32) + 4 * (rr // 32) + (j % 4)


def scales_tiled(s: torch.Tensor, k_cols: int) -> torch.Tensor:
    """Exponents [rows, K/32] -> E8M0 bytes in the tiled layout (rows padded to 128, pad = 0)."""
    rows = s.shape[0]
    rows_pad = (rows + 127) // 128 * 128
    out = torch.zeros(rows_pad * (k_cols // 32), dtype=torch.uint8)
    r = torch.arange(rows).view(-1, 1).expand(rows, k_cols // 32)
    j = torch.arange(k_cols // 32).view(1, -1).expand(rows, k_cols // 32)
    out[sf_offset(r, j, k_cols).reshape(-1)] = (s + 127).to(torch.uint8).reshape(-1)
    return out


def mx_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """MXFP8 x MXFP8 matmul with fp32 accumulation and a bf16 result, the contract of
    ffn_mx.mm (kernels/ffn_mx.py:159-182): x [M, K] bf16, w [N, K] bf16 -> [M, N] bf16."""
    return (qdq(x) @ qdq(w).t()).to(torch.bfloat16)
