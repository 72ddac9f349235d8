// Row kernels of the block forward (HBM-bound; one CTA per row, 16-byte vector accesses):
//   layernorm_mod   LN(x) * (1 + scale) + shift, or LN(x) * w + b  -> bf16 (optionally MXFP8 QDQ)
//                   WanLayerNorm + adaLN modulation, wan/modules/model_fast.py:3045, :3101, :2865-2867;
//                   wan/modules/model.py:145-156; kernels/glue.py:69-166
//   rmsnorm_rope    bf16(bf16(x * rsqrt(mean(x^2) + eps)) * gamma), then the 3-D RoPE rotation
//                   wan/modules/model.py:126-143; model_fast.py:878-979; kernels/qk_post.py:37-413
//                   (qk_rmsnorm_rope: q and k of the same tokens in one launch)
//   mx_quantize     bf16 -> E4M3 + E8M0 scales (tiled layout), kernels/ffn_mx.py:44-47
#include "host_common.cuh"
#include "lbw_common.cuh"
#include "mx_common.cuh"

namespace lbw {

constexpr int ROW_THREADS = 128;

// The two halves of a packed bf16x2 word (pack_bf16: low half = first value) as floats.
__device__ __forceinline__ float bf16_lo(uint32_t p) { return __uint_as_float(p << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t p) { return __uint_as_float(p & 0xFFFF0000u); }
constexpr int LN_MAXV = 12;  // 12 x 128 threads x 4 values = rows up to 6144 wide
constexpr int RR_MAXIT = 6;  // 6 x 128 threads x 8 bf16 values = rows up to 6144 wide

__device__ __forceinline__ float block_sum128(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  return red[0] + red[1] + red[2] + red[3];
}

// One CTA per row; thread t owns the float4 groups t, t + 128, ... so every warp access (x, the
// modulation vectors, the output) is one contiguous 512-byte (or 256/128-byte) span. The mean, the variance and
// the output pass each read the row (the second and third from L1 / L2): 40 registers per thread, so 12 rows are in
// flight per SM (7 when the row was held in registers), and a 1,350-row shard runs in one wave (B200, bit-identical
// results: 13.0 -> 10.6 us at 1,350 x 5,120, 70.5 -> 65.0 us at 10,800).
__global__ void __launch_bounds__(ROW_THREADS) layernorm_mod_kernel(const float* __restrict__ x, int C, float eps,
                                                                    const float* __restrict__ scale,
                                                                    const float* __restrict__ shift,
                                                                    const float* __restrict__ weight,
                                                                    const float* __restrict__ bias, int mx,
                                                                    __nv_bfloat16* __restrict__ out,
                                                                    uint8_t* __restrict__ mx_data,
                                                                    uint8_t* __restrict__ mx_scales, int mx_fmt) {
  __shared__ float red[4];
  const long long row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * C);
  const int G = C >> 2;
  // The row is read three times (sum, squared deviations, output) instead of held in registers: the re-reads hit
  // L1 / L2, and the small register footprint keeps 16 rows in flight per SM instead of 7.
  float s = 0.f;
#pragma unroll
  for (int it = 0; it < LN_MAXV; ++it) {
    const int g = it * ROW_THREADS + threadIdx.x;
    if (g < G) {
      const float4 a = __ldg(xr + g);
      s += (a.x + a.y) + (a.z + a.w);
    }
  }
  const float mean = block_sum128(s, red) / (float)C;
  float q = 0.f;
#pragma unroll
  for (int it = 0; it < LN_MAXV; ++it) {
    const int g = it * ROW_THREADS + threadIdx.x;
    if (g < G) {
      const float4 v = __ldg(xr + g);
      const float a = v.x - mean, b = v.y - mean, c = v.z - mean, d = v.w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
  }
  const float var = block_sum128(q, red) / (float)C;
  const float rstd = 1.f / sqrtf(var + eps);
  const float4* mul4 = reinterpret_cast<const float4*>(scale ? scale : weight);
  const float4* add4 = reinterpret_cast<const float4*>(scale ? shift : bias);
  const float one = scale ? 1.f : 0.f;  // (1 + scale) for the adaLN modulation, w for the affine
#pragma unroll
  for (int it = 0; it < LN_MAXV; ++it) {
    const int g = it * ROW_THREADS + threadIdx.x;
    if (it * ROW_THREADS >= G) break;  // block-uniform
    float y[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t p01 = 0u, p23 = 0u;
    if (g < G) {
      const float4 v = __ldcs(xr + g);
      float n[4] = {(v.x - mean) * rstd, (v.y - mean) * rstd, (v.z - mean) * rstd, (v.w - mean) * rstd};
      if (mul4) {
        const float4 m4 = __ldg(mul4 + g), a4 = __ldg(add4 + g);
        n[0] = n[0] * (one + m4.x) + a4.x;
        n[1] = n[1] * (one + m4.y) + a4.y;
        n[2] = n[2] * (one + m4.z) + a4.z;
        n[3] = n[3] * (one + m4.w) + a4.w;
      }
      p01 = pack_bf16(n[0], n[1]);  // the output's bf16 pairs (one cvt.rn.bf16x2 each)
      p23 = pack_bf16(n[2], n[3]);
      y[0] = bf16_lo(p01);
      y[1] = bf16_hi(p01);
      y[2] = bf16_lo(p23);
      y[3] = bf16_hi(p23);
    }
    if (mx || mx_data) {
      // 32-value MX block = 8 consecutive threads x 4 values (C % 32 == 0 keeps blocks inside the row)
      float amax = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      const bool e5 = mx_data && mx_fmt == MX_E5M2;
      const int se = e5 ? mx_shared_exp_fmt(amax, mx_emax(MX_E5M2)) : mx_shared_exp(amax);
      if (mx_data) {  // E4M3 (or E5M2) codes + E8M0 scale (tiled layout): the next MX GEMM's A operand
        // y * 2^-se is exact: se lies in [-127, 119] for bf16-range values, so 2^-se is a normal float
        const float inv = exp2i(-se);
        const __nv_fp8_interpretation_t kind = e5 ? __NV_E5M2 : __NV_E4M3;
        const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(y[0] * inv, y[1] * inv), __NV_SATFINITE, kind);
        const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(y[2] * inv, y[3] * inv), __NV_SATFINITE, kind);
        if (g < G) {
          *reinterpret_cast<uint32_t*>(mx_data + row * C + g * 4) = lo | (hi << 16);
          if ((g & 7) == 0) mx_scales[mx_sf_offset(row, g >> 3, C)] = (uint8_t)(se + 127);
        }
        continue;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = ldexpf(mx_from_e4m3(mx_to_e4m3(ldexpf(y[e], -se))), se);
      p01 = pack_bf16(y[0], y[1]);
      p23 = pack_bf16(y[2], y[3]);
    }
    if (g < G) *reinterpret_cast<uint2*>(out + row * C + g * 4) = make_uint2(p01, p23);
  }
}

// One row of RMSNorm (+ RoPE): thread t owns the 8-value groups t, t + 128, ... of the row. Values are rounded to
// bf16 two at a time (pack_bf16 = one cvt.rn.bf16x2) and unpacked with shifts: the conversions, not the memory
// traffic, bounded the bf16 RoPE mode (B200, 10,800 x 5,120: 78.2 -> 47.5 us; without RoPE 46.0 -> 37.6 us; the same
// bits).
__device__ __forceinline__ void rmsnorm_rope_row(const __nv_bfloat16* __restrict__ x, const float* __restrict__ ss,
                                                 const __nv_bfloat16* __restrict__ gamma, int C, float eps,
                                                 const float* __restrict__ rcos, const float* __restrict__ rsin,
                                                 int n_frames, int gh, int gw, int tok0, __nv_bfloat16* __restrict__ out,
                                                 long long ldo, int out_row_off, long long row, int rope_bf16) {
  const float r = 1.f / sqrtf(ss[row] / (float)C + eps);
  const int tok = tok0 + (int)row;
  const int f = tok / (gh * gw), hh = (tok / gw) % gh, ww = tok % gw;
  const int base_h = n_frames * 22, base_w = base_h + gh * 21;
  const __nv_bfloat16* xr = x + row * C;
  __nv_bfloat16* orow = out + (row + out_row_off) * ldo;
  for (int g = threadIdx.x; g < (C >> 3); g += ROW_THREADS) {
    uint4 xv = *reinterpret_cast<const uint4*>(xr + g * 8);
    uint4 gv = *reinterpret_cast<const uint4*>(gamma + g * 8);
    const __nv_bfloat16* xp = reinterpret_cast<const __nv_bfloat16*>(&xv);
    const __nv_bfloat16* gp = reinterpret_cast<const __nv_bfloat16*>(&gv);
    // bf16(bf16(x * r) * gamma), rounded two values at a time (one cvt.rn.bf16x2 per pair)
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const uint32_t n = pack_bf16(__bfloat162float(xp[e]) * r, __bfloat162float(xp[e + 1]) * r);
      const uint32_t t = pack_bf16(bf16_lo(n) * __bfloat162float(gp[e]), bf16_hi(n) * __bfloat162float(gp[e + 1]));
      y[e] = bf16_lo(t);
      y[e + 1] = bf16_hi(t);
    }
    if (rcos) {
      const int p0 = ((g * 8) & 127) >> 1;  // first pair index inside the head
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int p = p0 + k;
        const int idx = p < 22 ? f * 22 + p : (p < 43 ? base_h + hh * 21 + (p - 22) : base_w + ww * 21 + (p - 43));
        const float re = y[2 * k], im = y[2 * k + 1];
        if (rope_bf16) {
          // the reference's bf16 RoPE (model_fast.py:985-1003, :933-979 with ROPE_DTYPE bf16): bf16 cos / sin, and
          // every product and the sum rounded to bf16 as torch's bf16 elementwise ops do
          // (each cvt.rn.bf16x2 rounds two of those values at once)
          const uint32_t cs = pack_bf16(rcos[idx], rsin[idx]);
          const float c = bf16_lo(cs), s = bf16_hi(cs);
          const uint32_t p1 = pack_bf16(__fmul_rn(re, c), __fmul_rn(im, s));
          const uint32_t p2 = pack_bf16(__fmul_rn(re, s), __fmul_rn(im, c));
          const uint32_t o = pack_bf16(__fsub_rn(bf16_lo(p1), bf16_hi(p1)), __fadd_rn(bf16_lo(p2), bf16_hi(p2)));
          y[2 * k] = bf16_lo(o);
          y[2 * k + 1] = bf16_hi(o);
        } else {
          const float c = rcos[idx], s = rsin[idx];
          y[2 * k] = __fsub_rn(__fmul_rn(re, c), __fmul_rn(im, s));
          y[2 * k + 1] = __fadd_rn(__fmul_rn(re, s), __fmul_rn(im, c));
        }
      }
    }
    uint4 o = make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
    *reinterpret_cast<uint4*>(orow + g * 8) = o;
  }
}

__global__ void __launch_bounds__(ROW_THREADS) rmsnorm_rope_kernel(
    const __nv_bfloat16* __restrict__ x, const float* __restrict__ ss, const __nv_bfloat16* __restrict__ gamma, int C,
    float eps, const float* __restrict__ rcos, const float* __restrict__ rsin, int n_frames, int gh, int gw, int tok0,
    __nv_bfloat16* __restrict__ out, long long ldo, int out_row_off, int rope_bf16) {
  rmsnorm_rope_row(x, ss, gamma, C, eps, rcos, rsin, n_frames, gh, gw, tok0, out, ldo, out_row_off, blockIdx.x,
                   rope_bf16);
}

// q and k of the same tokens in one launch (blocks 0..m-1: q rows, m..2m-1: k rows), as the reference's
// qk_post.qk_norm_rope treats them together; each has its own gamma, row sums of squares and destination.
struct QKRows {
  const __nv_bfloat16* x[2];
  const float* ss[2];
  const __nv_bfloat16* gamma[2];
  __nv_bfloat16* out[2];
  long long ldo[2];
  int out_row_off[2];
};

__global__ void __launch_bounds__(ROW_THREADS) qk_rmsnorm_rope_kernel(const __grid_constant__ QKRows t, int m, int C,
                                                                      float eps, const float* __restrict__ rcos,
                                                                      const float* __restrict__ rsin, int n_frames,
                                                                      int gh, int gw, int tok0, int rope_bf16) {
  const int w = blockIdx.x >= (unsigned)m;
  rmsnorm_rope_row(t.x[w], t.ss[w], t.gamma[w], C, eps, rcos, rsin, n_frames, gh, gw, tok0, t.out[w], t.ldo[w],
                   t.out_row_off[w], (long long)blockIdx.x - (w ? m : 0), rope_bf16);
}

// One thread per 32-value block; rows up to the next multiple of 128 get zero scales. FMT: MX_E4M3 / MX_E5M2
// (one byte per element, row pitch K) or MX_E2M1 (packed nibbles, row pitch K / 2).
template <int FMT>
__global__ void mx_quantize_kernel(const __nv_bfloat16* __restrict__ x, int rows, int K, int rows_pad,
                                   uint8_t* __restrict__ data, uint8_t* __restrict__ scales,
                                   __nv_bfloat16* __restrict__ deq) {
  constexpr int BB = mx_block_bytes(FMT);
  const int nb = K >> 5;
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (long long)rows_pad * nb) return;
  const int r = (int)(id / nb), j = (int)(id % nb);
  if (r >= rows) {
    scales[mx_sf_offset(r, j, K)] = 0;
    return;
  }
  const __nv_bfloat16* xp = x + (long long)r * K + j * 32;
  float v[32];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u = *reinterpret_cast<const uint4*>(xp + q * 8);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[q * 8 + e] = __bfloat162float(b[e]);
  }
  __align__(16) uint8_t qb[32];
  const uint8_t sb = mx_quant32_fmt<FMT>(v, qb);
  scales[mx_sf_offset(r, j, K)] = sb;
  uint4* dp = reinterpret_cast<uint4*>(data + (long long)r * (K / 32 * BB) + j * BB);
  const uint4* w = reinterpret_cast<const uint4*>(qb);
#pragma unroll
  for (int q = 0; q < BB / 16; ++q) dp[q] = w[q];
  if (deq) {
    const int se = (int)sb - 127;
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 32; e += 2)
      pk[e >> 1] = pack_bf16(ldexpf(mx_elem<FMT>(qb, e), se), ldexpf(mx_elem<FMT>(qb, e + 1), se));
    uint4* d4 = reinterpret_cast<uint4*>(deq + (long long)r * K + j * 32);
#pragma unroll
    for (int q = 0; q < 4; ++q) d4[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  }
}

}  // namespace lbw

using namespace lbw;

extern "C" {

int lbw_layernorm_affine_mx(const float* x, int m, int c, float eps, const float* weight, const float* bias,
                            void* data, void* scales, void* stream) {
  return lbw_layernorm_affine_mx_fmt(x, m, c, eps, weight, bias, MX_E4M3, data, scales, stream);
}

int lbw_layernorm_affine_mx_fmt(const float* x, int m, int c, float eps, const float* weight, const float* bias,
                                int fmt, void* data, void* scales, void* stream) {
  if (!x || !data || !scales || !weight || !bias) return set_error(LBW_ERR_INVALID, "layernorm_affine_mx: null pointer");
  if (fmt != MX_E4M3 && fmt != MX_E5M2)
    return set_error(LBW_ERR_INVALID, "layernorm_affine_mx: element format %d (E4M3 or E5M2)", fmt);
  if (m <= 0 || c <= 0 || c % 128 || c > LN_MAXV * ROW_THREADS * 4)
    return set_error(LBW_ERR_SHAPE, "layernorm_affine_mx: width %d must be a multiple of 128 and <= %d", c,
                     LN_MAXV * ROW_THREADS * 4);
  if (!aligned(x, 16) || !aligned(data, 16) || !aligned(weight, 16) || !aligned(bias, 16))
    return set_error(LBW_ERR_ALIGN, "layernorm_affine_mx: x, data, weight and bias need 16-byte alignment");
  layernorm_mod_kernel<<<m, ROW_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, c, eps, nullptr, nullptr, weight, bias, 1, nullptr, reinterpret_cast<uint8_t*>(data),
      reinterpret_cast<uint8_t*>(scales), fmt);
  return cuda_check(cudaGetLastError(), "layernorm_affine_mx launch");
}

int lbw_layernorm_mod(const float* x, int m, int c, float eps, const float* scale, const float* shift,
                      const float* weight, const float* bias, int mx_qdq, void* out, void* stream) {
  if (!x || !out) return set_error(LBW_ERR_INVALID, "layernorm_mod: null pointer");
  if ((scale == nullptr) != (shift == nullptr) || (weight == nullptr) != (bias == nullptr) || (scale && weight))
    return set_error(LBW_ERR_INVALID, "layernorm_mod: give either scale+shift or weight+bias");
  if (m <= 0 || c <= 0 || c % 32 || c > LN_MAXV * ROW_THREADS * 4)
    return set_error(LBW_ERR_SHAPE, "layernorm_mod: width %d must be a multiple of 32 and <= %d", c,
                     LN_MAXV * ROW_THREADS * 4);
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(scale, 16) || !aligned(shift, 16) || !aligned(weight, 16) ||
      !aligned(bias, 16))
    return set_error(LBW_ERR_ALIGN, "layernorm_mod: x, out and the modulation vectors need 16-byte alignment");
  layernorm_mod_kernel<<<m, ROW_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, c, eps, scale, shift, weight, bias, mx_qdq, reinterpret_cast<__nv_bfloat16*>(out), nullptr, nullptr,
      MX_E4M3);
  return cuda_check(cudaGetLastError(), "layernorm_mod launch");
}

int lbw_layernorm_mod_mx(const float* x, int m, int c, float eps, const float* scale, const float* shift, void* data,
                         void* scales, void* stream) {
  return lbw_layernorm_mod_mx_fmt(x, m, c, eps, scale, shift, MX_E4M3, data, scales, stream);
}

int lbw_layernorm_mod_mx_fmt(const float* x, int m, int c, float eps, const float* scale, const float* shift, int fmt,
                             void* data, void* scales, void* stream) {
  if (!x || !data || !scales || !scale || !shift) return set_error(LBW_ERR_INVALID, "layernorm_mod_mx: null pointer");
  if (fmt != MX_E4M3 && fmt != MX_E5M2)
    return set_error(LBW_ERR_INVALID, "layernorm_mod_mx: element format %d (E4M3 or E5M2)", fmt);
  if (m <= 0 || c <= 0 || c % 128 || c > LN_MAXV * ROW_THREADS * 4)
    return set_error(LBW_ERR_SHAPE, "layernorm_mod_mx: width %d must be a multiple of 128 and <= %d", c,
                     LN_MAXV * ROW_THREADS * 4);
  if (!aligned(x, 16) || !aligned(data, 16) || !aligned(scale, 16) || !aligned(shift, 16))
    return set_error(LBW_ERR_ALIGN, "layernorm_mod_mx: x, data and the modulation vectors need 16-byte alignment");
  layernorm_mod_kernel<<<m, ROW_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, c, eps, scale, shift, nullptr, nullptr, 1, nullptr, reinterpret_cast<uint8_t*>(data),
      reinterpret_cast<uint8_t*>(scales), fmt);
  return cuda_check(cudaGetLastError(), "layernorm_mod_mx launch");
}

int lbw_rmsnorm_rope(const void* x, const float* ss, const void* gamma, int m, int c, float eps,
                     const float* rope_cos, const float* rope_sin, int rope_frames, int grid_h, int grid_w, int tok0,
                     void* out, long long ldo, int out_row_off, void* stream) {
  return lbw_rmsnorm_rope_dt(x, ss, gamma, m, c, eps, rope_cos, rope_sin, rope_frames, grid_h, grid_w, tok0, out, ldo,
                             out_row_off, LBW_ROPE_FP32, stream);
}

int lbw_rmsnorm_rope_dt(const void* x, const float* ss, const void* gamma, int m, int c, float eps,
                        const float* rope_cos, const float* rope_sin, int rope_frames, int grid_h, int grid_w, int tok0,
                        void* out, long long ldo, int out_row_off, int rope_dtype, void* stream) {
  if (!x || !ss || !gamma || !out) return set_error(LBW_ERR_INVALID, "rmsnorm_rope: null pointer");
  if (rope_dtype != LBW_ROPE_FP32 && rope_dtype != LBW_ROPE_BF16)
    return set_error(LBW_ERR_INVALID, "rmsnorm_rope: rope dtype %d", rope_dtype);
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return set_error(LBW_ERR_INVALID, "rmsnorm_rope: cos/sin pair");
  if (m <= 0 || c <= 0 || c % 128 || c > RR_MAXIT * ROW_THREADS * 8)
    return set_error(LBW_ERR_SHAPE, "rmsnorm_rope: width %d must be a multiple of 128 and <= %d", c,
                     RR_MAXIT * ROW_THREADS * 8);
  if (rope_cos && (grid_h <= 0 || grid_w <= 0 || rope_frames <= 0 || tok0 < 0 ||
                   (tok0 + m - 1) / (grid_h * grid_w) >= rope_frames))
    return set_error(LBW_ERR_SHAPE, "rmsnorm_rope: tokens %d..%d outside a %d-frame %dx%d grid", tok0, tok0 + m - 1,
                     rope_frames, grid_h, grid_w);
  if (!aligned(x, 16) || !aligned(gamma, 16) || !aligned(out, 16) || ldo % 8)
    return set_error(LBW_ERR_ALIGN, "rmsnorm_rope: alignment");
  const int n_frames = rope_cos ? rope_frames : 0;
  rmsnorm_rope_kernel<<<m, ROW_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ss, reinterpret_cast<const __nv_bfloat16*>(gamma), c, eps, rope_cos,
      rope_sin, n_frames, grid_h > 0 ? grid_h : 1, grid_w > 0 ? grid_w : 1, tok0,
      reinterpret_cast<__nv_bfloat16*>(out), ldo, out_row_off, rope_dtype == LBW_ROPE_BF16);
  return cuda_check(cudaGetLastError(), "rmsnorm_rope launch");
}

int lbw_qk_rmsnorm_rope(const void* q_raw, const float* ss_q, const void* gamma_q, void* q_out, long long ldq,
                        int q_row_off, const void* k_raw, const float* ss_k, const void* gamma_k, void* k_out,
                        long long ldk, int k_row_off, int m, int c, float eps, const float* rope_cos,
                        const float* rope_sin, int rope_frames, int grid_h, int grid_w, int tok0, void* stream) {
  return lbw_qk_rmsnorm_rope_dt(q_raw, ss_q, gamma_q, q_out, ldq, q_row_off, k_raw, ss_k, gamma_k, k_out, ldk,
                                k_row_off, m, c, eps, rope_cos, rope_sin, rope_frames, grid_h, grid_w, tok0,
                                LBW_ROPE_FP32, stream);
}

int lbw_qk_rmsnorm_rope_dt(const void* q_raw, const float* ss_q, const void* gamma_q, void* q_out, long long ldq,
                           int q_row_off, const void* k_raw, const float* ss_k, const void* gamma_k, void* k_out,
                           long long ldk, int k_row_off, int m, int c, float eps, const float* rope_cos,
                           const float* rope_sin, int rope_frames, int grid_h, int grid_w, int tok0, int rope_dtype,
                           void* stream) {
  if (!q_raw || !ss_q || !gamma_q || !q_out || !k_raw || !ss_k || !gamma_k || !k_out)
    return set_error(LBW_ERR_INVALID, "qk_rmsnorm_rope: null pointer");
  if (rope_dtype != LBW_ROPE_FP32 && rope_dtype != LBW_ROPE_BF16)
    return set_error(LBW_ERR_INVALID, "qk_rmsnorm_rope: rope dtype %d", rope_dtype);
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return set_error(LBW_ERR_INVALID, "qk_rmsnorm_rope: cos/sin pair");
  if (m <= 0 || c <= 0 || c % 128 || c > RR_MAXIT * ROW_THREADS * 8 || m > (1 << 30))
    return set_error(LBW_ERR_SHAPE, "qk_rmsnorm_rope: %d rows of width %d (a multiple of 128, <= %d)", m, c,
                     RR_MAXIT * ROW_THREADS * 8);
  if (rope_cos && (grid_h <= 0 || grid_w <= 0 || rope_frames <= 0 || tok0 < 0 ||
                   (tok0 + m - 1) / (grid_h * grid_w) >= rope_frames))
    return set_error(LBW_ERR_SHAPE, "qk_rmsnorm_rope: tokens %d..%d outside a %d-frame %dx%d grid", tok0, tok0 + m - 1,
                     rope_frames, grid_h, grid_w);
  if (q_row_off < 0 || k_row_off < 0) return set_error(LBW_ERR_INVALID, "qk_rmsnorm_rope: negative row offset");
  if (!aligned(q_raw, 16) || !aligned(k_raw, 16) || !aligned(gamma_q, 16) || !aligned(gamma_k, 16) ||
      !aligned(q_out, 16) || !aligned(k_out, 16) || ldq % 8 || ldk % 8 || ldq < c || ldk < c)
    return set_error(LBW_ERR_ALIGN, "qk_rmsnorm_rope: alignment or row stride");
  QKRows t{};
  t.x[0] = reinterpret_cast<const __nv_bfloat16*>(q_raw);
  t.x[1] = reinterpret_cast<const __nv_bfloat16*>(k_raw);
  t.ss[0] = ss_q;
  t.ss[1] = ss_k;
  t.gamma[0] = reinterpret_cast<const __nv_bfloat16*>(gamma_q);
  t.gamma[1] = reinterpret_cast<const __nv_bfloat16*>(gamma_k);
  t.out[0] = reinterpret_cast<__nv_bfloat16*>(q_out);
  t.out[1] = reinterpret_cast<__nv_bfloat16*>(k_out);
  t.ldo[0] = ldq;
  t.ldo[1] = ldk;
  t.out_row_off[0] = q_row_off;
  t.out_row_off[1] = k_row_off;
  const int n_frames = rope_cos ? rope_frames : 0;
  qk_rmsnorm_rope_kernel<<<2 * m, ROW_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      t, m, c, eps, rope_cos, rope_sin, n_frames, grid_h > 0 ? grid_h : 1, grid_w > 0 ? grid_w : 1, tok0,
      rope_dtype == LBW_ROPE_BF16);
  return cuda_check(cudaGetLastError(), "qk_rmsnorm_rope launch");
}

int lbw_mx_quantize_fmt(const void* x, int rows, int k, int fmt, void* data, void* scales, void* dequant,
                        void* stream) {
  if (!x || !data || !scales) return set_error(LBW_ERR_INVALID, "mx_quantize: null pointer");
  if (fmt < MX_E4M3 || fmt > MX_E2M1) return set_error(LBW_ERR_INVALID, "mx_quantize: element format %d", fmt);
  if (rows <= 0 || k <= 0 || k % 128) return set_error(LBW_ERR_SHAPE, "mx_quantize: K=%d must be a multiple of 128", k);
  if (!aligned(x, 16) || !aligned(data, 16) || (dequant && !aligned(dequant, 16)))
    return set_error(LBW_ERR_ALIGN, "mx_quantize: alignment");
  const int rows_pad = (rows + 127) / 128 * 128;
  const long long n = (long long)rows_pad * (k / 32);
  const int threads = 256;
  const unsigned blocks = (unsigned)((n + threads - 1) / threads);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x);
  uint8_t *d = reinterpret_cast<uint8_t*>(data), *sc = reinterpret_cast<uint8_t*>(scales);
  __nv_bfloat16* dq = reinterpret_cast<__nv_bfloat16*>(dequant);
  if (fmt == MX_E4M3) mx_quantize_kernel<MX_E4M3><<<blocks, threads, 0, s>>>(xb, rows, k, rows_pad, d, sc, dq);
  else if (fmt == MX_E5M2) mx_quantize_kernel<MX_E5M2><<<blocks, threads, 0, s>>>(xb, rows, k, rows_pad, d, sc, dq);
  else mx_quantize_kernel<MX_E2M1><<<blocks, threads, 0, s>>>(xb, rows, k, rows_pad, d, sc, dq);
  return cuda_check(cudaGetLastError(), "mx_quantize launch");
}

int lbw_mx_quantize(const void* x, int rows, int k, void* data, void* scales, void* dequant, void* stream) {
  return lbw_mx_quantize_fmt(x, rows, k, MX_E4M3, data, scales, dequant, stream);
}

}  // extern "C"
