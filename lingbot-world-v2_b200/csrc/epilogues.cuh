// Fused GEMM epilogues shared by the bf16 and the MXFP8 tcgen05 GEMMs. Each epilogue thread owns one
// output row of the tile; chunk() receives 32 consecutive fp32 accumulators of that row (read from TMEM)
// and returns a partial row statistic; tile_done() receives the sum over the tile's chunks.
//   EpiStore     bias + bf16 store into up to three column regions, optional row sums of squares
//   EpiResidual  x += bf16(acc + b) * gate, then optional FiLM x = (1 + s) * x + t on the fp32 residual
//   EpiAct       bf16(act(bf16(acc + b))) [+ addend]: the camera-FiLM MLP layers
//   EpiGelu      GELU_tanh(bf16(acc + b)) as bf16, or GELU_tanh(bf16(bf16(acc) + b)) MXFP8 quantise-dequantised
//   EpiGeluMX    GELU_tanh(bf16(bf16(acc) + b)) quantised to MXFP8 codes + E8M0 scales (the next GEMM's A operand)
// round_acc (EpiStore, EpiResidual, EpiAct): the accumulator is rounded to bf16 before the bias is added, the
// rounding points of an MXFP8 Linear in the reference (kernels/ffn_mx.py mm() returns bf16, then `y + bias` in
// bf16, wan/modules/model_fast.py:1403-1410, :1602-1610); without it bias and accumulator meet in fp32 once
// (nn.Linear).
#pragma once
#include <type_traits>

#include "lbw_common.cuh"
#include "mx_common.cuh"

namespace lbw {

// Epilogues that normalise each output row over all of its columns declare ROW_NORM = true and provide sumsq()
// and chunk_norm(); the GEMM then reads the whole row from TMEM before writing it.
template <class E, class = void>
struct row_norm : std::false_type {};
template <class E>
struct row_norm<E, std::void_t<decltype(E::ROW_NORM)>> : std::integral_constant<bool, E::ROW_NORM> {};

struct EpiStore {
  static constexpr int WARP_SMEM = 0;  // no warp-cooperative chunk()
  __nv_bfloat16* out[3];
  long long ld[3];
  int row_off[3];
  float* ss[3];          // per-region row sum-of-squares accumulators (nullable)
  int region_cols;       // columns per region
  int ss_per_chunk;      // regions not aligned to the 256-column tile: accumulate per 32-column chunk
  const __nv_bfloat16* bias;  // [N] (nullable)
  int round_acc;

  LBW_DEV float chunk(int row, int col, const float (&v)[32]) const {
    int r = col / region_cols;
    int cl = col - r * region_cols;
    __nv_bfloat16* dst = out[r] + (long long)(row + row_off[r]) * ld[r] + cl;
    float ssum = 0.f;
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 32; e += 8) {
      float b[8];
      if (bias) {
        uint4 bb = *reinterpret_cast<const uint4*>(bias + col + e);
        const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&bb);
#pragma unroll
        for (int q = 0; q < 8; ++q) b[q] = __bfloat162float(bp[q]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) b[q] = 0.f;
      }
#pragma unroll
      for (int q = 0; q < 8; q += 2) {
        const float a0 = round_acc ? bf16_round(v[e + q]) : v[e + q];
        const float a1 = round_acc ? bf16_round(v[e + q + 1]) : v[e + q + 1];
        float y0 = bf16_round(a0 + b[q]);
        float y1 = bf16_round(a1 + b[q + 1]);
        ssum += y0 * y0 + y1 * y1;
        pk[(e + q) / 2] = pack_bf16(y0, y1);
      }
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) d4[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    if (ss_per_chunk) {
      if (ss[r]) atomicAdd(ss[r] + row, ssum);
      return 0.f;
    }
    return ssum;
  }
  LBW_DEV void tile_done(int row, int col0, float ssum) const {
    int r = col0 / region_cols;
    if (!ss_per_chunk && ss[r]) atomicAdd(ss[r] + row, ssum);
  }
};

// FILM = false: no FiLM operands (the MXFP8 FFN-down GEMM, cross-o).
// WCOLS > 0: the GEMM hands each warp's 32 rows x 32 columns to chunk_warp(), which transposes them through
// shared memory, WCOLS columns at a time (WARP_SMEM bytes per warp), so that the residual and FiLM rows are
// read and written with 16-byte accesses by WCOLS / 4 lanes per row, and all loads of a WCOLS-column slice are
// issued before its stores. The bf16 GEMM stages 32 columns; the MXFP8 GEMM, whose ring leaves ~28 KB of shared
// memory, stages 16 (measured at 10,800 x 5,120 x 5,120: cross-o 0.70 -> 0.26 ms against one row per thread;
// 8-column slices made the FiLM variant slower, 0.52 vs 0.48 ms). WCOLS = 0: chunk() on one row per thread in
// four 8-column rounds.
template <bool FILM, int WCOLS = (FILM ? 32 : 0)>
struct EpiResidualT {
  static_assert(WCOLS == 0 || WCOLS == 16 || WCOLS == 32, "WCOLS is 0, 16 or 32");
  static constexpr int WARP_SMEM = WCOLS ? 32 * (WCOLS + 1) * 4 : 0;
  float* x;                          // [M, ldx] fp32 residual, updated in place
  long long ldx;
  const __nv_bfloat16* bias;         // [N] nullable
  const float* gate;                 // [N] nullable (gate = 1)
  const __nv_bfloat16* film_scale;   // [M, N] nullable
  const __nv_bfloat16* film_shift;   // [M, N] (with film_scale)
  long long ldf;
  int round_acc;

  LBW_DEV float acc(float v) const { return round_acc ? bf16_round(v) : v; }

  // Columns [off, off + W) of the chunk. Every global read is issued before the first store (the stores may
  // alias those rows as far as the compiler knows), so a part costs one memory round trip.
  template <int W>
  LBW_DEV void part(int row, int col, int off, const float (&v)[32]) const {
    float* xr = x + (long long)row * ldx + col + off;
    float4 xv[W / 4];
#pragma unroll
    for (int q = 0; q < W / 4; ++q) xv[q] = reinterpret_cast<const float4*>(xr)[q];
    uint4 sv[W / 8], tv[W / 8];
    if (FILM && film_scale) {
      const long long fo = (long long)row * ldf + col + off;
#pragma unroll
      for (int q = 0; q < W / 8; ++q) {
        sv[q] = reinterpret_cast<const uint4*>(film_scale + fo)[q];
        tv[q] = reinterpret_cast<const uint4*>(film_shift + fo)[q];
      }
    }
    float* xs = reinterpret_cast<float*>(xv);   // updated in place, 8 values at a time
#pragma unroll
    for (int e = 0; e < W; e += 8) {
      float y[8];
      if (bias) {
        const uint4 bb = __ldg(reinterpret_cast<const uint4*>(bias + col + off + e));
        const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&bb);
#pragma unroll
        for (int q = 0; q < 8; ++q) y[q] = bf16_round(acc(v[off + e + q]) + __bfloat162float(bp[q]));
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) y[q] = bf16_round(v[off + e + q]);
      }
      if (gate) {
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(gate + col + off + e));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(gate + col + off + e + 4));
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) y[q] = __fmul_rn(y[q], g[q]);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) xs[e + q] = __fadd_rn(xs[e + q], y[q]);
      if (FILM && film_scale) {
        const __nv_bfloat16* sp = reinterpret_cast<const __nv_bfloat16*>(&sv[e / 8]);
        const __nv_bfloat16* tp = reinterpret_cast<const __nv_bfloat16*>(&tv[e / 8]);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float s1 = bf16_round(1.f + __bfloat162float(sp[q]));  // (1.0 + bf16 tensor) stays bf16
          xs[e + q] = __fadd_rn(__fmul_rn(s1, xs[e + q]), __bfloat162float(tp[q]));
        }
      }
    }
#pragma unroll
    for (int q = 0; q < W / 4; ++q) reinterpret_cast<float4*>(xr)[q] = xv[q];
  }

  // Warp-cooperative form (all 32 lanes, lane i = row row0 + i, the same 32 columns), one WCOLS-column slice at
  // a time: y = bf16(acc + b) * gate per row into shared memory, then LPR = WCOLS / 4 lanes per row read x / FiLM
  // and write x with 16-byte accesses, 32 / LPR rows per pass, all loads of the slice before its stores.
  // Rows >= M are skipped.
  LBW_DEV void chunk_warp(int row0, int lane, int col, const float (&v)[32], int M, float* sm) const {
    constexpr int WC = WCOLS > 0 ? WCOLS : 32, SP = WC + 1, LPR = WC / 4, RPP = 32 / LPR, PASSES = 32 / RPP;
#pragma unroll
    for (int h = 0; h < 32; h += WC) {
#pragma unroll
      for (int e = 0; e < WC; e += 8) {
        float y[8];
        if (bias) {
          const uint4 bb = __ldg(reinterpret_cast<const uint4*>(bias + col + h + e));
          const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&bb);
#pragma unroll
          for (int q = 0; q < 8; ++q) y[q] = bf16_round(acc(v[h + e + q]) + __bfloat162float(bp[q]));
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) y[q] = bf16_round(v[h + e + q]);
        }
        if (gate) {
          const float4 g0 = __ldg(reinterpret_cast<const float4*>(gate + col + h + e));
          const float4 g1 = __ldg(reinterpret_cast<const float4*>(gate + col + h + e + 4));
          const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
          for (int q = 0; q < 8; ++q) y[q] = __fmul_rn(y[q], g[q]);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) sm[lane * SP + e + q] = y[q];
      }
      __syncwarp();
      const int rr = lane / LPR, c4 = (lane % LPR) * 4, cc = col + h + c4;
      float4 xv[PASSES];
      uint2 sv[PASSES], tv[PASSES];
#pragma unroll
      for (int it = 0; it < PASSES; ++it) {
        const int row = row0 + it * RPP + rr;
        if (row < M) {
          xv[it] = *reinterpret_cast<const float4*>(x + (long long)row * ldx + cc);
          if (FILM && film_scale) {
            const long long fo = (long long)row * ldf + cc;
            sv[it] = *reinterpret_cast<const uint2*>(film_scale + fo);
            tv[it] = *reinterpret_cast<const uint2*>(film_shift + fo);
          }
        }
      }
#pragma unroll
      for (int it = 0; it < PASSES; ++it) {
        const int r = it * RPP + rr, row = row0 + r;
        if (row < M) {
          float o[4] = {xv[it].x, xv[it].y, xv[it].z, xv[it].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) o[q] = __fadd_rn(o[q], sm[r * SP + c4 + q]);
          if (FILM && film_scale) {
            const __nv_bfloat16* sp = reinterpret_cast<const __nv_bfloat16*>(&sv[it]);
            const __nv_bfloat16* tp = reinterpret_cast<const __nv_bfloat16*>(&tv[it]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float s1 = bf16_round(1.f + __bfloat162float(sp[q]));  // (1.0 + bf16 tensor) stays bf16
              o[q] = __fadd_rn(__fmul_rn(s1, o[q]), __bfloat162float(tp[q]));
            }
          }
          *reinterpret_cast<float4*>(x + (long long)row * ldx + cc) = make_float4(o[0], o[1], o[2], o[3]);
        }
      }
      __syncwarp();
    }
  }

  LBW_DEV float chunk(int row, int col, const float (&v)[32]) const {
    if constexpr (WCOLS == 32) {
      part<32>(row, col, 0, v);
    } else {
#pragma unroll
      for (int off = 0; off < 32; off += 8) part<8>(row, col, off, v);
    }
    return 0.f;
  }
  LBW_DEV void tile_done(int, int, float) const {}
};
using EpiResidual = EpiResidualT<true>;

struct EpiGelu {
  static constexpr int WARP_SMEM = 0;  // no warp-cooperative chunk()
  __nv_bfloat16* out;   // [M, ldo] GELU(u + b), or its MXFP8 quantise-dequantise
  long long ldo;
  const __nv_bfloat16* bias;
  int qdq;

  LBW_DEV float chunk(int row, int col, const float (&v)[32]) const {
    float g[32];
#pragma unroll
    for (int e = 0; e < 32; e += 8) {
      uint4 bb = *reinterpret_cast<const uint4*>(bias + col + e);
      const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&bb);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        // MX (qdq): the matmul's bf16 result, then + bias in bf16; plain Linear: one rounding
        float u = bf16_round((qdq ? bf16_round(v[e + q]) : v[e + q]) + __bfloat162float(bp[q]));
        g[e + q] = bf16_round(gelu_tanh_fast(u));
      }
    }
    uint32_t pk[16];
    if (qdq) {
      mx_qdq32(g, pk);
    } else {
#pragma unroll
      for (int e = 0; e < 32; e += 2) pk[e >> 1] = pack_bf16(g[e], g[e + 1]);
    }
    uint4* d4 = reinterpret_cast<uint4*>(out + (long long)row * ldo + col);
#pragma unroll
    for (int q = 0; q < 4; ++q) d4[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    return 0.f;
  }
  LBW_DEV void tile_done(int, int, float) const {}
};

// out = bf16(act(bf16(acc + b))) [+ addend, rounded to bf16], act = identity or SiLU: the camera-FiLM
// MLP of the block (cam_injector_layer1 + SiLU, cam_injector_layer2 + the camera embedding).
struct EpiAct {
  static constexpr int WARP_SMEM = 0;  // no warp-cooperative chunk()
  __nv_bfloat16* out;           // [M, ldo]
  long long ldo;
  const __nv_bfloat16* bias;    // [N] nullable
  const __nv_bfloat16* addend;  // [M, ldo] nullable
  int silu;
  int round_acc;

  LBW_DEV float chunk(int row, int col, const float (&v)[32]) const {
    const long long off = (long long)row * ldo + col;
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 32; e += 8) {
      float b[8], a[8];
      if (bias) {
        uint4 bb = *reinterpret_cast<const uint4*>(bias + col + e);
        const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&bb);
#pragma unroll
        for (int q = 0; q < 8; ++q) b[q] = __bfloat162float(bp[q]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) b[q] = 0.f;
      }
      if (addend) {
        uint4 aa = *reinterpret_cast<const uint4*>(addend + off + e);
        const __nv_bfloat16* ap = reinterpret_cast<const __nv_bfloat16*>(&aa);
#pragma unroll
        for (int q = 0; q < 8; ++q) a[q] = __bfloat162float(ap[q]);
      }
#pragma unroll
      for (int q = 0; q < 8; q += 2) {
        float y[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float t = bf16_round((round_acc ? bf16_round(v[e + q + u]) : v[e + q + u]) + b[q + u]);
          if (silu) t = bf16_round(t / (1.f + __expf(-t)));
          if (addend) t = bf16_round(t + a[q + u]);
          y[u] = t;
        }
        pk[(e + q) / 2] = pack_bf16(y[0], y[1]);
      }
    }
    uint4* d4 = reinterpret_cast<uint4*>(out + off);
#pragma unroll
    for (int q = 0; q < 4; ++q) d4[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    return 0.f;
  }
  LBW_DEV void tile_done(int, int, float) const {}
};

struct EpiGeluMX {
  static constexpr int WARP_SMEM = 0;  // no warp-cooperative chunk()
  uint8_t* data;     // [M, ld] E4M3 (or E5M2, fmt) codes of GELU(u + b)
  uint8_t* scales;   // E8M0 scales in the tiled layout of a [M, sf_cols] matrix (mx_sf_offset)
  long long ld;
  int sf_cols;
  const __nv_bfloat16* bias;
  int fmt;           // MX_E4M3 (0) or MX_E5M2

  LBW_DEV float chunk(int row, int col, const float (&v)[32]) const {
    float g[32];
#pragma unroll
    for (int e = 0; e < 32; e += 8) {
      uint4 bb = *reinterpret_cast<const uint4*>(bias + col + e);
      const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&bb);
      // v is the MX GEMM's accumulator already rounded to bf16 (its epilogue pulls it as bf16 pairs); u = bf16(v + b)
      // and GELU(u) rounded two values per conversion
#pragma unroll
      for (int q = 0; q < 8; q += 2) {
        const uint32_t up = pack_bf16(v[e + q] + __bfloat162float(bp[q]), v[e + q + 1] + __bfloat162float(bp[q + 1]));
        const uint32_t gp = pack_bf16(gelu_tanh_fast(__uint_as_float(up << 16)),
                                      gelu_tanh_fast(__uint_as_float(up & 0xFFFF0000u)));
        g[e + q] = __uint_as_float(gp << 16);
        g[e + q + 1] = __uint_as_float(gp & 0xFFFF0000u);
      }
    }
    __align__(16) uint8_t qb[32];
    const uint8_t sb = fmt == MX_E5M2 ? mx_quant32_fmt<MX_E5M2>(g, qb) : mx_quant32(g, qb);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(qb);
    uint4* dp = reinterpret_cast<uint4*>(data + (long long)row * ld + col);
    dp[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dp[1] = make_uint4(w[4], w[5], w[6], w[7]);
    scales[mx_sf_offset(row, col >> 5, sf_cols)] = sb;
    return 0.f;
  }
  LBW_DEV void tile_done(int, int, float) const {}
};

// VAE decoder convolution over frames with a one-pixel zero border ([frames][H + 2][W + 2][C] rows): bf16(acc + b),
// then + residual rounded to bf16 (the ResidualBlock's shortcut add, wan/modules/vae2_1.py:219); border rows are
// written as zeros so that the output is the next layer's padded input.
struct EpiConv {
  static constexpr int WARP_SMEM = 0;  // no warp-cooperative chunk()
  __nv_bfloat16* out;                // [M, ldo]
  long long ldo;
  const __nv_bfloat16* bias;         // [N] nullable
  const __nv_bfloat16* residual;     // [M, ldr] nullable
  long long ldr;
  int P, W2, H2;                     // rows per frame (H + 2)(W + 2), padded width and height

  LBW_DEV float chunk(int row, int col, const float (&v)[32]) const {
    const int q = row % P, hp = q / W2, wp = q - hp * W2;
    const bool border = hp == 0 || hp == H2 - 1 || wp == 0 || wp == W2 - 1;
    uint32_t pk[16];
    if (border) {
#pragma unroll
      for (int e = 0; e < 16; ++e) pk[e] = 0u;
    } else {
#pragma unroll
      for (int e = 0; e < 32; e += 8) {
        float b[8], r[8];
        if (bias) {
          const uint4 bb = __ldg(reinterpret_cast<const uint4*>(bias + col + e));
          const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&bb);
#pragma unroll
          for (int q2 = 0; q2 < 8; ++q2) b[q2] = __bfloat162float(bp[q2]);
        } else {
#pragma unroll
          for (int q2 = 0; q2 < 8; ++q2) b[q2] = 0.f;
        }
        if (residual) {
          const uint4 rr = *reinterpret_cast<const uint4*>(residual + (long long)row * ldr + col + e);
          const __nv_bfloat16* rp = reinterpret_cast<const __nv_bfloat16*>(&rr);
#pragma unroll
          for (int q2 = 0; q2 < 8; ++q2) r[q2] = __bfloat162float(rp[q2]);
        }
#pragma unroll
        for (int q2 = 0; q2 < 8; q2 += 2) {
          float y0 = bf16_round(v[e + q2] + b[q2]), y1 = bf16_round(v[e + q2 + 1] + b[q2 + 1]);
          if (residual) {
            y0 = bf16_round(y0 + r[q2]);
            y1 = bf16_round(y1 + r[q2 + 1]);
          }
          pk[(e + q2) / 2] = pack_bf16(y0, y1);
        }
      }
    }
    uint4* d4 = reinterpret_cast<uint4*>(out + (long long)row * ldo + col);
#pragma unroll
    for (int q2 = 0; q2 < 4; ++q2) d4[q2] = make_uint4(pk[4 * q2], pk[4 * q2 + 1], pk[4 * q2 + 2], pk[4 * q2 + 3]);
    return 0.f;
  }
  LBW_DEV void tile_done(int, int, float) const {}
};

// The VAE ResidualBlock's first convolution fused with the RMS_norm + SiLU that follows it (vae2_1.py:189-192):
// y = bf16(acc + b), then silu(y / max(||y||, 1e-12) * sqrt(C) * gamma) over the row's N channels (the whole row
// lies in one tile), written straight into the second convolution's input; border rows are written as zeros.
struct EpiConvRms {
  static constexpr int WARP_SMEM = 0;  // no warp-cooperative chunk()
  static constexpr bool ROW_NORM = true;
  __nv_bfloat16* out;                // [M, ldo]
  long long ldo;
  const __nv_bfloat16* bias;         // [N] nullable
  const float* gamma;                // [N] (zero past the real channels)
  float scale_c;                     // sqrt(real channels)
  int P, W2, H2;

  LBW_DEV bool border(int row) const {
    const int q = row % P, hp = q / W2, wp = q - hp * W2;
    return hp == 0 || hp == H2 - 1 || wp == 0 || wp == W2 - 1;
  }
  LBW_DEV void rounded(int col, const float (&v)[32], float (&y)[32]) const {
#pragma unroll
    for (int e = 0; e < 32; e += 8) {
      float b[8];
      if (bias) {
        const uint4 bb = __ldg(reinterpret_cast<const uint4*>(bias + col + e));
        const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&bb);
#pragma unroll
        for (int q = 0; q < 8; ++q) b[q] = __bfloat162float(bp[q]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) b[q] = 0.f;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) y[e + q] = bf16_round(v[e + q] + b[q]);
    }
  }
  LBW_DEV float sumsq(int row, int col, const float (&v)[32]) const {
    if (border(row)) return 0.f;
    float y[32];
    rounded(col, v, y);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 32; ++e) ss += y[e] * y[e];
    return ss;
  }
  LBW_DEV void chunk_norm(int row, int col, const float (&v)[32], float ss) const {
    uint32_t pk[16];
    if (border(row)) {
#pragma unroll
      for (int e = 0; e < 16; ++e) pk[e] = 0u;
    } else {
      float y[32];
      rounded(col, v, y);
      const float inv = scale_c / fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float t0 = y[e] * inv * __ldg(gamma + col + e), t1 = y[e + 1] * inv * __ldg(gamma + col + e + 1);
        t0 = t0 / (1.f + __expf(-t0));
        t1 = t1 / (1.f + __expf(-t1));
        pk[e >> 1] = pack_bf16(t0, t1);
      }
    }
    uint4* d4 = reinterpret_cast<uint4*>(out + (long long)row * ldo + col);
#pragma unroll
    for (int q = 0; q < 4; ++q) d4[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  }
  LBW_DEV float chunk(int, int, const float (&)[32]) const { return 0.f; }
  LBW_DEV void tile_done(int, int, float) const {}
};

// fp32 store of the accumulator (attention scores of the VAE's mid-block attention)
struct EpiStoreF32 {
  static constexpr int WARP_SMEM = 0;  // no warp-cooperative chunk()
  float* out;
  long long ldo;
  LBW_DEV float chunk(int row, int col, const float (&v)[32]) const {
    float4* d4 = reinterpret_cast<float4*>(out + (long long)row * ldo + col);
#pragma unroll
    for (int q = 0; q < 8; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    return 0.f;
  }
  LBW_DEV void tile_done(int, int, float) const {}
};

}  // namespace lbw
