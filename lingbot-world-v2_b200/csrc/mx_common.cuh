// MXFP8 (OCP Microscaling Formats v1.0) block arithmetic shared by the quantiser, the
// bf16-pipe FFN epilogue and the block-scaled GEMM epilogue.
//
// One block = 32 consecutive values along K. Shared scale X = 2^s with
//   s = clamp(floor(log2(amax)) - 8, -127, 127)      (8 = exponent of E4M3's largest normal, 448)
// stored as the E8M0 byte s + 127; elements = RNE(v / X) to E4M3 with saturation to +-448.
// An all-zero block gets s = -127.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace lbw {

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  float inner = k0 * (x + k1 * x * x * x);
  return 0.5f * x * (1.f + tanhf(inner));
}
// The same function through the identity 0.5 x (1 + tanh(z)) = x / (1 + e^(-2z)), with the SFU's ex2.approx
// (relative error ~2^-22) and a fast division: a few instructions, and accurate to a few fp32 ulps, so that the
// bf16 rounding of the result (and the MXFP8 code chosen from it) rarely differs from the fp32 GELU's
// (tanh.approx.f32 has a relative error of ~2^-11, a quarter of a bf16 ulp). For x -> -inf the exponential
// overflows and the quotient is -0.
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float inner = k0 * fmaf(k1 * x, x * x, x);
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-2.8853900817779268f * inner));  // e^(-2 inner)
  return __fdividef(x, 1.f + e);
}
// 2^e as a float for e in [-126, 127] (exact).
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }

// Shared exponent of a block from its absolute maximum (exact, from the fp32 bit pattern).
__device__ __forceinline__ int mx_shared_exp(float amax) {
  if (!(amax > 0.f)) return -127;
  int e = (int)((__float_as_uint(amax) >> 23) & 0xFF);
  int fl = (e == 0) ? -127 : e - 127;  // subnormal amax: floor(log2) <= -127
  int s = fl - 8;
  return s < -127 ? -127 : (s > 127 ? 127 : s);
}

__device__ __forceinline__ uint8_t mx_to_e4m3(float q) {
  return (uint8_t)__nv_cvt_float_to_fp8(q, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float mx_from_e4m3(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

// Quantise 32 values: elements into q[32], returns the E8M0 scale byte.
__device__ __forceinline__ uint8_t mx_quant32(const float (&v)[32], uint8_t (&q)[32]) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const int s = mx_shared_exp(amax);
  // v * 2^-s is exact: s lies in [-127, 119] for finite bf16-range inputs, so 2^-s is a normal float.
  const float inv = exp2i(-s);
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const __nv_fp8x2_storage_t p =
        __nv_cvt_float2_to_fp8x2(make_float2(v[i] * inv, v[i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
    q[i] = (uint8_t)(p & 0xFF);
    q[i + 1] = (uint8_t)(p >> 8);
  }
  return (uint8_t)(s + 127);
}

// ---- element formats of the block-scaled path (OCP MX v1.0): E4M3 (emax 8), E5M2 (emax 15), E2M1 (emax 2) ----
enum MxFmt : int { MX_E4M3 = 0, MX_E5M2 = 1, MX_E2M1 = 2 };
__host__ __device__ constexpr int mx_emax(int fmt) { return fmt == MX_E5M2 ? 15 : (fmt == MX_E2M1 ? 2 : 8); }
// bytes of one 32-value block's elements (E2M1: two per byte, element 2i in the low nibble)
__host__ __device__ constexpr int mx_block_bytes(int fmt) { return fmt == MX_E2M1 ? 16 : 32; }

// Shared exponent floor(log2(amax)) - emax, clamped to the E8M0 range [-127, 127]; -127 for an all-zero block.
__device__ __forceinline__ int mx_shared_exp_fmt(float amax, int emax) {
  if (!(amax > 0.f)) return -127;
  int e = (int)((__float_as_uint(amax) >> 23) & 0xFF);
  int fl = (e == 0) ? -127 : e - 127;
  int s = fl - emax;
  return s < -127 ? -127 : (s > 127 ? 127 : s);
}

// Quantise 32 values to format FMT: element bytes into q (mx_block_bytes(FMT) of them), returns the E8M0 byte.
// Elements are round-to-nearest-even of v / 2^s, saturated to the format's largest finite value.
template <int FMT>
__device__ __forceinline__ uint8_t mx_quant32_fmt(const float (&v)[32], uint8_t* q) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const int s = mx_shared_exp_fmt(amax, mx_emax(FMT));
  // v * 2^-s is exact: -s lies in [-125, 127], so 2^-s is a normal float
  const float inv = exp2i(-s);
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const float2 f = make_float2(v[i] * inv, v[i + 1] * inv);
    if (FMT == MX_E2M1) {
      q[i >> 1] = (uint8_t)__nv_cvt_float2_to_fp4x2(f, __NV_E2M1, cudaRoundNearest);
    } else {
      const __nv_fp8x2_storage_t p = __nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, FMT == MX_E5M2 ? __NV_E5M2 : __NV_E4M3);
      q[i] = (uint8_t)(p & 0xFF);
      q[i + 1] = (uint8_t)(p >> 8);
    }
  }
  return (uint8_t)(s + 127);
}

// Element i of a block (bytes q) as a float, before the shared scale.
template <int FMT>
__device__ __forceinline__ float mx_elem(const uint8_t* q, int i) {
  if (FMT == MX_E2M1) {
    const __nv_fp4_storage_t c = (__nv_fp4_storage_t)((q[i >> 1] >> ((i & 1) * 4)) & 0xF);
    return __half2float(__half(__nv_cvt_fp4_to_halfraw(c, __NV_E2M1)));
  }
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)q[i], FMT == MX_E5M2 ? __NV_E5M2 : __NV_E4M3);
  return __half2float(__half(h));
}

// Quantise-dequantise 32 values and pack the (exactly representable) results as bf16 pairs.
__device__ __forceinline__ void mx_qdq32(const float (&v)[32], uint32_t (&pk)[16]) {
  uint8_t q[32];
  int s = (int)mx_quant32(v, q) - 127;
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float a = ldexpf(mx_from_e4m3(q[i]), s), b = ldexpf(mx_from_e4m3(q[i + 1]), s);
    __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    pk[i / 2] = *reinterpret_cast<uint32_t*>(&p);
  }
}

// Byte offset of scale (row r, scale column j) in the tiled scale-factor layout used by the
// block-scaled GEMM: 512-byte atoms of 128 rows x 4 scale columns, atoms ordered row-block
// major; inside an atom row r = r0 + 32 r1 sits at 16 r0 + 4 r1 + (j % 4).
__host__ __device__ __forceinline__ long long mx_sf_offset(long long r, long long j, long long k_cols) {
  long long atoms_per_rowblock = k_cols / 128;  // K/32 scales / 4 per atom
  long long atom = (r >> 7) * atoms_per_rowblock + (j >> 2);
  int rr = (int)(r & 127);
  return atom * 512 + 16 * (rr & 31) + 4 * (rr >> 5) + (j & 3);
}

}  // namespace lbw
