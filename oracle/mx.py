"""MX (E8M0 shared scale per 32 values) quantise-dequantise emulation: E4M3 and E5M2 (MXFP8), E2M1 (MXFP4).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Written from the OCP Microscaling Formats (MX) v1.0 specification, section 6.3 (conversion):
    X = 2 ** (floor(log2(max_i |V_i|)) - emax_elem),   emax_elem = exponent of the element type's largest normal
    P_i = quantize_elem(V_i / X)   round-to-nearest-even, saturating to the largest finite element
and X is clamped to the E8M0 range [2^-127, 2^127]; an all-zero block takes X = 2^-127.
    E4M3: emax 8, largest 448 (the reference's default, kernels/ffn_mx.py:18)
    E5M2: emax 15, largest 57344 (LINGBOT_MX_FP8=float8_e5m2, kernels/ffn_mx.py:8, :18)
    E2M1: emax 2, largest 6, values {0, 0.5, 1, 1.5, 2, 3, 4, 6} (MXFP4; not in the reference, the FFN GEMM
          sweep of the benchmark configuration asks for it)

The reference quantises with nkilib's quantize_block_mxfp8_kernel / matmul_mxfp8
(kernels/ffn_mx.py:14-15, :44-50, :159-182), a Neuron SDK library that is not vendored and not
pinned; its weight padding of K to 512 (ffn_mx.K_ALIGN, :20) adds zero blocks only and does not
change any product.
"""
import torch

BLOCK = 32
E4M3_MAX = 448.0
EMAX_E4M3 = 8
# element type -> (emax_elem, largest finite magnitude)
FORMATS = {"e4m3": (8, 448.0), "e5m2": (15, 57344.0), "e2m1": (2, 6.0)}
E2M1_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)   # magnitude of code 0..7 (bit 3 = sign)


def shared_exponent(amax: torch.Tensor, emax: int = EMAX_E4M3) -> torch.Tensor:
    """floor(log2(amax)) - emax, clamped to [-127, 127]; -127 where amax == 0."""
    _, e = torch.frexp(amax.float())          # amax = m * 2**e, m in [0.5, 1)
    s = (e - 1 - emax).clamp(-127, 127)
    return torch.where(amax > 0, s, torch.full_like(s, -127))


def _rne(x: torch.Tensor) -> torch.Tensor:
    return torch.round(x)                     # torch.round rounds half to even


def e2m1_round(v: torch.Tensor) -> torch.Tensor:
    """Round fp32 values to the E2M1 grid, to nearest with ties to the even code, saturating at +-6."""
    a = v.abs()
    q = torch.where(a < 2, _rne(a * 2) / 2, torch.where(a < 4, _rne(a), 2 * _rne(a / 2)))
    return torch.copysign(q.clamp(max=6.0), v)


def e2m1_codes(q: torch.Tensor) -> torch.Tensor:
    """E2M1 values (on the grid) -> 4-bit codes (uint8 0..15): bit 3 sign, bits 2..1 exponent, bit 0 mantissa."""
    grid = torch.tensor(E2M1_GRID)
    idx = (q.abs().unsqueeze(-1) == grid).float().argmax(-1).to(torch.uint8)
    return idx | (torch.signbit(q).to(torch.uint8) << 3)


def e2m1_pack(codes: torch.Tensor) -> torch.Tensor:
    """Codes [..., K] -> bytes [..., K/2]: element 2i in the low nibble, 2i + 1 in the high nibble."""
    return codes[..., 0::2] | (codes[..., 1::2] << 4)


def e2m1_unpack(packed: torch.Tensor) -> torch.Tensor:
    """Bytes [..., K/2] -> fp32 values [..., K]."""
    lo, hi = packed & 15, packed >> 4
    codes = torch.stack([lo, hi], dim=-1).flatten(-2)
    mag = torch.tensor(E2M1_GRID)[(codes & 7).long()]
    return torch.where((codes & 8) != 0, -mag, mag)


def quantize(x: torch.Tensor, fmt: str = "e4m3"):
    """x [..., K] (K % 32 == 0) -> (element values [..., K], exponents int32 [..., K/32]). Element values are
    float8_e4m3fn / float8_e5m2 tensors for the FP8 formats and fp32 values on the E2M1 grid for "e2m1"."""
    emax, vmax = FORMATS[fmt]
    k = x.shape[-1]
    assert k % BLOCK == 0, k
    xb = x.float().reshape(*x.shape[:-1], k // BLOCK, BLOCK)
    s = shared_exponent(xb.abs().amax(dim=-1, keepdim=True), emax)
    v = torch.ldexp(xb, (-s).float()).clamp(-vmax, vmax)
    if fmt == "e2m1":
        q = e2m1_round(v)
    else:
        q = v.to(torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2)
    return q.reshape(x.shape), s.squeeze(-1).to(torch.int32)


def dequantize(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    k = q.shape[-1]
    qb = q.float().reshape(*q.shape[:-1], k // BLOCK, BLOCK)
    return torch.ldexp(qb, s.float().unsqueeze(-1)).reshape(q.shape)


def qdq(x: torch.Tensor, fmt: str = "e4m3") -> torch.Tensor:
    """Quantise-dequantise along the last dim; returns fp32 values (exact in bf16)."""
    q, s = quantize(x, fmt)
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


def mx_linear(x: torch.Tensor, w: torch.Tensor, fmt: str = "e4m3") -> torch.Tensor:
    """MX x MX matmul (both operands in `fmt`) with fp32 accumulation and a bf16 result, the contract of
    ffn_mx.mm (kernels/ffn_mx.py:159-182): x [M, K] bf16, w [N, K] bf16 -> [M, N] bf16."""
    return (qdq(x, fmt) @ qdq(w, fmt).t()).to(torch.bfloat16)
