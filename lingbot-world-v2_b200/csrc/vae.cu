// Memory-bound kernels of the Wan 2.1 VAE decoder (wan/modules/vae2_1.py), on frames stored channels-last with a
// one-pixel zero border: [frames][H + 2][W + 2][C] bf16 ("padded rows"; C a multiple of 8). The convolutions
// themselves are implicit GEMMs on the tcgen05 GEMM (lbw_vae_conv, gemm_bf16.cu).
//   rms_silu         RMS_norm (x / max(||x||, 1e-12) * sqrt(C) * gamma, :38-53), optionally followed by SiLU
//   upsample2x       nearest 2x in h and w (Upsample 'nearest-exact', :56-62; Resample :65-95) into padded rows
//   time_interleave  the time_conv's [C | C] channel halves -> frames 2t, 2t + 1 (:131-135)
//   gather / scatter the interior rows of padded frames <-> compact token rows (AttentionBlock, :239-267)
//   softmax_rows     row softmax of fp32 scores -> bf16 probabilities (the mid-block attention)
//   transpose        bf16 [rows, cols] -> [cols, rows]
#include "host_common.cuh"
#include "lbw_common.cuh"

namespace lbw {

namespace vae {

// A CTA takes RMS_ROWS consecutive rows, which are one contiguous span of memory: its 256 threads load the span
// as 16-byte vectors (coalesced), leave each vector's sum of squares in shared memory, sum each row's partials
// in a fixed order (deterministic), and write the scaled vectors back. Border rows (all zeros) stay zero.
constexpr int RMS_ROWS = 32, RMS_THREADS = 256, RMS_MAXC = 512;
constexpr int RMS_VPT = RMS_ROWS * (RMS_MAXC / 8) / RMS_THREADS;  // vectors per thread at the widest rows

__global__ void __launch_bounds__(RMS_THREADS) rms_silu_kernel(const __nv_bfloat16* __restrict__ x, long long rows,
                                                               int C, float scale_c, const float* __restrict__ gamma,
                                                               int silu, __nv_bfloat16* __restrict__ out) {
  __shared__ float part[RMS_ROWS * (RMS_MAXC / 8)];
  __shared__ float inv_s[RMS_ROWS];
  const int nv = C >> 3;
  const long long row0 = (long long)blockIdx.x * RMS_ROWS;
  const int nrows = (int)(rows - row0 < RMS_ROWS ? rows - row0 : RMS_ROWS);
  const int nvec = nrows * nv;
  const uint4* src = reinterpret_cast<const uint4*>(x + row0 * C);
  uint4 v[RMS_VPT];
#pragma unroll
  for (int i = 0; i < RMS_VPT; ++i) {
    const int k = threadIdx.x + i * RMS_THREADS;
    if (k < nvec) {
      v[i] = src[k];
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v[i]);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = __bfloat162float(b[e]);
        ss += f * f;
      }
      part[k] = ss;
    }
  }
  __syncthreads();
  if (threadIdx.x < nrows) {
    float ss = 0.f;
    for (int j = 0; j < nv; ++j) ss += part[threadIdx.x * nv + j];
    inv_s[threadIdx.x] = scale_c / fmaxf(sqrtf(ss), 1e-12f);
  }
  __syncthreads();
  uint4* dst = reinterpret_cast<uint4*>(out + row0 * C);
#pragma unroll
  for (int i = 0; i < RMS_VPT; ++i) {
    const int k = threadIdx.x + i * RMS_THREADS;
    if (k < nvec) {
      const int r = k / nv, g = k - r * nv;
      const float inv = inv_s[r];
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v[i]);
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + g * 8));
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + g * 8 + 4));
      const float gm[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float t = __bfloat162float(b[e]) * inv * gm[e];
        if (silu) t = t / (1.f + __expf(-t));
        y[e] = t;
      }
      dst[k] = make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
    }
  }
}

// out [F][2H + 2][2W + 2][C] from x [F][H + 2][W + 2][C]: out(h, w) = x(h / 2, w / 2) inside, zero border.
// One thread per (output row, 8-channel vector).
__global__ void upsample2x_kernel(const __nv_bfloat16* __restrict__ x, int frames, int H, int W, int C,
                                  __nv_bfloat16* __restrict__ out) {
  const int nv = C >> 3;
  const int W2o = 2 * W + 2, H2o = 2 * H + 2;
  const long long Po = (long long)H2o * W2o, Pi = (long long)(H + 2) * (W + 2);
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (long long)frames * Po * nv) return;
  const int g = (int)(id % nv);
  const long long r = id / nv;
  const int f = (int)(r / Po);
  const int q = (int)(r - f * Po);
  const int hp = q / W2o, wp = q - hp * W2o;
  uint4 val = make_uint4(0u, 0u, 0u, 0u);
  if (hp > 0 && hp < H2o - 1 && wp > 0 && wp < W2o - 1) {
    const int hi = (hp - 1) / 2 + 1, wi = (wp - 1) / 2 + 1;
    val = *reinterpret_cast<const uint4*>(x + (f * Pi + (long long)hi * (W + 2) + wi) * C + g * 8);
  }
  *reinterpret_cast<uint4*>(out + r * C + g * 8) = val;
}

// x [F * P][2C] -> out [2F * P][C]: frame 2f <- channels [0, C), frame 2f + 1 <- [C, 2C).
__global__ void time_interleave_kernel(const __nv_bfloat16* __restrict__ x, int frames, long long P, int C,
                                       __nv_bfloat16* __restrict__ out) {
  const int nv = C >> 3;
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= 2LL * frames * P * nv) return;
  const int g = (int)(id % nv);
  const long long r = id / nv;  // output row
  const long long fo = r / P, q = r - fo * P;
  const long long fi = fo >> 1;
  const int half = (int)(fo & 1);
  *reinterpret_cast<uint4*>(out + r * C + g * 8) =
      *reinterpret_cast<const uint4*>(x + (fi * P + q) * (2LL * C) + half * C + g * 8);
}

// interior rows of padded frames -> compact rows t = (f * H + h) * W + w
__global__ void gather_kernel(const __nv_bfloat16* __restrict__ x, int frames, int H, int W, int C,
                              __nv_bfloat16* __restrict__ out) {
  const int nv = C >> 3;
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (long long)frames * H * W * nv) return;
  const int g = (int)(id % nv);
  const long long t = id / nv;
  const int w = (int)(t % W);
  const long long fh = t / W;
  const int h = (int)(fh % H), f = (int)(fh / H);
  const long long src = ((long long)f * (H + 2) + h + 1) * (W + 2) + w + 1;
  *reinterpret_cast<uint4*>(out + t * C + g * 8) = *reinterpret_cast<const uint4*>(x + src * C + g * 8);
}

// out (padded) = bf16(resid + y) inside (y: compact rows), zeros on the border
__global__ void scatter_add_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ resid,
                                   int frames, int H, int W, int C, __nv_bfloat16* __restrict__ out) {
  const int nv = C >> 3;
  const long long P = (long long)(H + 2) * (W + 2);
  const long long id = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= (long long)frames * P * nv) return;
  const int g = (int)(id % nv);
  const long long r = id / nv;
  const int f = (int)(r / P);
  const int q = (int)(r - f * P);
  const int hp = q / (W + 2), wp = q - hp * (W + 2);
  uint4 o = make_uint4(0u, 0u, 0u, 0u);
  if (hp > 0 && hp <= H && wp > 0 && wp <= W) {
    const long long t = ((long long)f * H + hp - 1) * W + wp - 1;
    const uint4 a = *reinterpret_cast<const uint4*>(resid + r * C + g * 8);
    const uint4 b = *reinterpret_cast<const uint4*>(y + t * C + g * 8);
    const __nv_bfloat16* ap = reinterpret_cast<const __nv_bfloat16*>(&a);
    const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&b);
    uint32_t pk[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2)
      pk[e / 2] = pack_bf16(__bfloat162float(ap[e]) + __bfloat162float(bp[e]),
                            __bfloat162float(ap[e + 1]) + __bfloat162float(bp[e + 1]));
    o = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
  *reinterpret_cast<uint4*>(out + r * C + g * 8) = o;
}

// P[r, c] = exp(scale (S[r, c] - max_r)) / sum_r for c < n, 0 for n <= c < n_pad. One CTA (256 threads) per row.
__global__ void __launch_bounds__(256) softmax_rows_kernel(const float* __restrict__ S, long long lds, int n,
                                                           int n_pad, float scale, __nv_bfloat16* __restrict__ P,
                                                           long long ldp) {
  __shared__ float red[2][8];
  const float* sr = S + (long long)blockIdx.x * lds;
  float m = -INFINITY, l = 0.f;
  for (int c = threadIdx.x; c < n; c += 256) {
    const float v = sr[c] * scale;
    if (v > m) {
      l = l * __expf(m - v) + 1.f;
      m = v;
    } else {
      l += __expf(v - m);
    }
  }
  // combine (m, l) over the warp, then over the 8 warps
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, l, o);
    const float mm = fmaxf(m, m2);
    l = (m == -INFINITY ? 0.f : l * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : l2 * __expf(m2 - mm));
    m = mm;
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[0][w] = m;
    red[1][w] = l;
  }
  __syncthreads();
  float M = red[0][0];
#pragma unroll
  for (int i = 1; i < 8; ++i) M = fmaxf(M, red[0][i]);
  float L = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) L += red[0][i] == -INFINITY ? 0.f : red[1][i] * __expf(red[0][i] - M);
  const float inv = 1.f / L;
  __nv_bfloat16* pr = P + (long long)blockIdx.x * ldp;
  for (int c = threadIdx.x; c < n_pad; c += 256)
    pr[c] = __float2bfloat16_rn(c < n ? __expf(sr[c] * scale - M) * inv : 0.f);
}

// out[c][r] = x[r][c] through a 32 x 33 shared tile; x rows have stride ldx, out rows stride ldo.
__global__ void transpose_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, int rows, int cols,
                                 __nv_bfloat16* __restrict__ out, long long ldo) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < rows && c < cols) ? x[(long long)r * ldx + c] : __float2bfloat16_rn(0.f);
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (c < cols && r < rows) out[(long long)c * ldo + r] = tile[threadIdx.x][i];
  }
}

inline unsigned blocks_for(long long n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace vae
}  // namespace lbw

using namespace lbw;

extern "C" {

int lbw_vae_rms_silu(const void* x, long long rows, int c, int c_real, const float* gamma, int silu, void* out,
                     void* stream) {
  if (!x || !gamma || !out) return set_error(LBW_ERR_INVALID, "lbw_vae_rms_silu: null pointer");
  if (rows <= 0 || c <= 0 || c % 8 || c > 512 || c_real <= 0 || c_real > c)
    return set_error(LBW_ERR_SHAPE, "lbw_vae_rms_silu: %d channels (%d real; a multiple of 8, <= 512)", c, c_real);
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(gamma, 16)) return set_error(LBW_ERR_ALIGN, "lbw_vae_rms_silu");
  vae::rms_silu_kernel<<<vae::blocks_for(rows, vae::RMS_ROWS), vae::RMS_THREADS, 0,
                          reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), rows, c, sqrtf((float)c_real), gamma, silu,
      reinterpret_cast<__nv_bfloat16*>(out));
  return cuda_check(cudaGetLastError(), "vae rms_silu launch");
}

int lbw_vae_upsample2x(const void* x, int frames, int h, int w, int c, void* out, void* stream) {
  if (!x || !out) return set_error(LBW_ERR_INVALID, "lbw_vae_upsample2x: null pointer");
  if (frames <= 0 || h <= 0 || w <= 0 || c <= 0 || c % 8) return set_error(LBW_ERR_SHAPE, "lbw_vae_upsample2x: shape");
  if (!aligned(x, 16) || !aligned(out, 16)) return set_error(LBW_ERR_ALIGN, "lbw_vae_upsample2x");
  const long long n = (long long)frames * (2 * h + 2) * (2 * w + 2) * (c / 8);
  vae::upsample2x_kernel<<<vae::blocks_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), frames, h, w, c, reinterpret_cast<__nv_bfloat16*>(out));
  return cuda_check(cudaGetLastError(), "vae upsample2x launch");
}

int lbw_vae_time_interleave(const void* x, int frames, long long frame_rows, int c, void* out, void* stream) {
  if (!x || !out) return set_error(LBW_ERR_INVALID, "lbw_vae_time_interleave: null pointer");
  if (frames <= 0 || frame_rows <= 0 || c <= 0 || c % 8) return set_error(LBW_ERR_SHAPE, "lbw_vae_time_interleave");
  if (!aligned(x, 16) || !aligned(out, 16)) return set_error(LBW_ERR_ALIGN, "lbw_vae_time_interleave");
  const long long n = 2LL * frames * frame_rows * (c / 8);
  vae::time_interleave_kernel<<<vae::blocks_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), frames, frame_rows, c, reinterpret_cast<__nv_bfloat16*>(out));
  return cuda_check(cudaGetLastError(), "vae time_interleave launch");
}

int lbw_vae_gather(const void* x, int frames, int h, int w, int c, void* out, void* stream) {
  if (!x || !out) return set_error(LBW_ERR_INVALID, "lbw_vae_gather: null pointer");
  if (frames <= 0 || h <= 0 || w <= 0 || c <= 0 || c % 8) return set_error(LBW_ERR_SHAPE, "lbw_vae_gather");
  if (!aligned(x, 16) || !aligned(out, 16)) return set_error(LBW_ERR_ALIGN, "lbw_vae_gather");
  const long long n = (long long)frames * h * w * (c / 8);
  vae::gather_kernel<<<vae::blocks_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), frames, h, w, c, reinterpret_cast<__nv_bfloat16*>(out));
  return cuda_check(cudaGetLastError(), "vae gather launch");
}

int lbw_vae_scatter_add(const void* y, const void* resid, int frames, int h, int w, int c, void* out, void* stream) {
  if (!y || !resid || !out) return set_error(LBW_ERR_INVALID, "lbw_vae_scatter_add: null pointer");
  if (frames <= 0 || h <= 0 || w <= 0 || c <= 0 || c % 8) return set_error(LBW_ERR_SHAPE, "lbw_vae_scatter_add");
  if (!aligned(y, 16) || !aligned(resid, 16) || !aligned(out, 16)) return set_error(LBW_ERR_ALIGN, "lbw_vae_scatter_add");
  const long long n = (long long)frames * (h + 2) * (w + 2) * (c / 8);
  vae::scatter_add_kernel<<<vae::blocks_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(y), reinterpret_cast<const __nv_bfloat16*>(resid), frames, h, w, c,
      reinterpret_cast<__nv_bfloat16*>(out));
  return cuda_check(cudaGetLastError(), "vae scatter_add launch");
}

int lbw_softmax_rows(const float* s, long long lds, int rows, int n, int n_pad, float scale, void* p, long long ldp,
                     void* stream) {
  if (!s || !p) return set_error(LBW_ERR_INVALID, "lbw_softmax_rows: null pointer");
  if (rows <= 0 || n <= 0 || n_pad < n || lds < n || ldp < n_pad)
    return set_error(LBW_ERR_SHAPE, "lbw_softmax_rows: %d rows of %d (%d padded)", rows, n, n_pad);
  vae::softmax_rows_kernel<<<rows, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      s, lds, n, n_pad, scale, reinterpret_cast<__nv_bfloat16*>(p), ldp);
  return cuda_check(cudaGetLastError(), "softmax_rows launch");
}

int lbw_transpose_bf16(const void* x, long long ldx, int rows, int cols, void* out, long long ldo, void* stream) {
  if (!x || !out) return set_error(LBW_ERR_INVALID, "lbw_transpose_bf16: null pointer");
  if (rows <= 0 || cols <= 0 || ldx < cols || ldo < rows) return set_error(LBW_ERR_SHAPE, "lbw_transpose_bf16");
  dim3 grid((cols + 31) / 32, (rows + 31) / 32);
  vae::transpose_kernel<<<grid, dim3(32, 8), 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, rows, cols, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return cuda_check(cudaGetLastError(), "transpose launch");
}

}  // extern "C"
