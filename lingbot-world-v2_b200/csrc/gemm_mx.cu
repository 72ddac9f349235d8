// Persistent tcgen05 block-scaled GEMM: MXFP8 (E4M3 elements, one E8M0 scale per 32 along K) x MXFP8
// -> fp32 (TMEM) -> fused epilogue. This is the FFN of the causal-fast block with LINGBOT_FFN_MX=1:
// ffn_mx.mm (kernels/ffn_mx.py:159-182), the bias + GELU(tanh) epilogue of ffn_epi.bias_gelu_pad
// (kernels/ffn_epi.py:15-37) and the gated residual x + y * e5 (wan/modules/model_fast.py:3110-3111).
// With LINGBOT_LIN_MX=1 the block's other Linears (q|k|v, o, cross q/k/v/o, camera FiLM MLP) run on it too.
//
//   A [M, K] codes + scales (activations),  W [N, K] codes + scales (nn.Linear layout), K % 128 == 0.
//   Scales use the tiled layout of lbw_mx_quantize: 512-byte atoms of 128 rows x 4 scales (row-block
//   major), which is exactly the 32-row x 16-byte core-matrix staging tcgen05.cp 32x128b.warpx4 expects.
//
// Tiles 128 x 256, K staged 128 codes (one 128-byte swizzled row) per stage through a 4-deep TMA ring;
// each stage also carries the tile's scales (1 atom for A, 2 for W) as plain bulk copies. The MMA thread
// copies the stage's scales into TMEM (columns 256..267) and issues 4 tcgen05.mma kind::mxf8f6f4
// (K = 32 each; the instruction's scale-id selects the byte of the 32-bit scale column). TMEM holds one
// 256-column accumulator (the other 256 columns would leave no room for the scales), so the 8 epilogue
// warps first pull the whole tile into registers (thread = row, 128 columns each), release the
// accumulator, and only then run the epilogue math while the next tile's MMAs proceed.
//   warp 0 TMA producer, warp 1 MMA issuer + TMEM owner, warps 2-9 epilogue.
#include <math.h>

#include "epilogues.cuh"
#include "host_common.cuh"
#include "lbw_common.cuh"
#include "mx_common.cuh"

namespace lbw {

namespace mxg {
constexpr int BM = 128, BK = 128;  // BK: bytes of one K block per row (one 128-byte swizzled TMA box row)
constexpr int A_BYTES = BM * BK;   // 16 KB
constexpr int SFA_BYTES = 512;
constexpr int THREADS = 320;
constexpr int EPI_WARPS = 8;
constexpr int SMEM_LIMIT = 232448;  // opt-in dynamic shared memory per CTA on sm_100
// Tile width TBN = 256 (default) or 128 (when 256-wide tiles would leave the last wave mostly idle).
// A 128-wide tile's MMAs take half as long as a 256-wide tile's, so its stages hold two K blocks (and
// their scale atoms): the lone MMA-issuing thread then waits once per 8 MMAs instead of once per 4.
// FMT: element format (MX_E4M3 / MX_E5M2: a K block is 128 elements, one byte each, one 512-byte scale atom per
// 128 rows; MX_E2M1: 256 elements as packed nibbles, two scale atoms per 128 rows).
template <int TBN, int FMT = MX_E4M3> struct Cfg {
  static constexpr int KSUB = TBN == 256 ? 1 : 2;                 // K blocks per stage
  static constexpr int KE = FMT == MX_E2M1 ? 256 : 128;           // elements of one K block
  static constexpr int SFPB = KE / 128;                           // scale atoms per K block and 128 rows
  static constexpr int B_SUB = TBN * BK;
  static constexpr int A_STAGE = A_BYTES * KSUB, B_STAGE = B_SUB * KSUB;
  static constexpr int B_BYTES = B_STAGE;
  static constexpr int SFA_STAGE = SFA_BYTES * SFPB * KSUB;
  static constexpr int SFB_STAGE = TBN / 128 * 512 * SFPB * KSUB;
  static constexpr int SF_BYTES = SFA_STAGE + SFB_STAGE;
  static constexpr int TX_BYTES = A_STAGE + B_STAGE + SF_BYTES;
  static constexpr int STAGES = TBN == 256 ? 4 : 3;
  static constexpr int SMEM_BYTES = STAGES * TX_BYTES + 1024;
  // scale columns right after the accumulator: 4 per scale atom for A (SFPB per K block), then the same per
  // 128-row W block
  static constexpr uint32_t SFA_COL = TBN, SFB_COL = TBN + 4 * SFPB * KSUB;
};
}  // namespace mxg

template <class Epi, int TBN = 256, int FMT = MX_E4M3>
__global__ void __launch_bounds__(mxg::THREADS, 1)
    gemm_mx_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfb, int M, int N, int K, int group_m,
                   Epi epi,
                   int* status) {
  using mxg::BM;
  using mxg::BK;
  using mxg::A_BYTES;
  using Cf = mxg::Cfg<TBN, FMT>;
  constexpr int SFPB = Cf::SFPB;
  constexpr int BN = TBN, STAGES = Cf::STAGES, B_BYTES = Cf::B_BYTES, SF_BYTES = Cf::SF_BYTES;
  constexpr int TX_BYTES = Cf::TX_BYTES;
  constexpr uint32_t SFA_COL = Cf::SFA_COL, SFB_COL = Cf::SFB_COL;
  constexpr int HALF_COLS = BN / 2;  // columns per epilogue warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int KSUB = Cf::KSUB, A_STAGE = Cf::A_STAGE;
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_STAGE;
  uint8_t* sSF = sB + STAGES * B_BYTES;
  __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], tfull_bar, tempty_bar, done_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&tfull_bar, 1);
    mbar_init(&tempty_bar, 256);
    mbar_init(&done_bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(&tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const Abort ab{status, &abort_flag};

  const int nM = (M + BM - 1) / BM, nN = (N + BN - 1) / BN, nK = K / Cf::KE, nS = nK / KSUB;
  const int nAtom = K / 128;  // scale atoms per 128 rows (4 scales of 32 elements each)
  const int n_sf_blocks = (N + 127) / 128;  // 128-row scale blocks of W that exist
  const int tiles = nM * nN;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      long long issued = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        int m_blk, n_blk;
        tile_coords(t, nM, nN, group_m, m_blk, n_blk);
        const int b0 = 2 * n_blk, b1 = (2 * n_blk + 1 < n_sf_blocks) ? 2 * n_blk + 1 : 2 * n_blk;
        bool ok = true;
        for (int ks = 0; ks < nS; ++ks) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1, ab, 0x51)) { ok = false; break; }
          uint8_t* sf = sSF + s * SF_BYTES;
          const int kb = ks * KSUB;  // first 128-code K block of the stage
          mbar_expect_tx(&full_bar[s], TX_BYTES);
#pragma unroll
          for (int u = 0; u < KSUB; ++u) {
            tma_load_2d(sA + s * A_STAGE + u * A_BYTES, &tmA, &full_bar[s], (kb + u) * BK, m_blk * BM);
            tma_load_2d(sB + s * B_BYTES + u * Cf::B_SUB, &tmB, &full_bar[s], (kb + u) * BK, n_blk * BN);
          }
          // scale atoms of consecutive K blocks are consecutive 512-byte atoms
          bulk_load(sf, sfa + ((long long)m_blk * nAtom + kb * SFPB) * 512, 512 * SFPB * KSUB, &full_bar[s]);
          if (BN == 256) {
            bulk_load(sf + Cf::SFA_STAGE, sfb + ((long long)b0 * nAtom + kb * SFPB) * 512, 512 * SFPB, &full_bar[s]);
            bulk_load(sf + Cf::SFA_STAGE + 512 * SFPB, sfb + ((long long)b1 * nAtom + kb * SFPB) * 512, 512 * SFPB,
                      &full_bar[s]);
          } else {
            bulk_load(sf + Cf::SFA_STAGE, sfb + ((long long)n_blk * nAtom + kb * SFPB) * 512, 512 * SFPB * KSUB,
                      &full_bar[s]);
          }
          ++issued;
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
      }
      for (long long i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i)
        mbar_wait_drain(&full_bar[i % STAGES], (uint32_t)((i / STAGES) & 1));
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // descriptors built once: a shared-memory byte offset o adds o >> 4 to the start-address field
      const uint64_t dA = sdesc_kmajor_sw128(smem_u32(sA)), dB = sdesc_kmajor_sw128(smem_u32(sB));
      const uint64_t dS = sdesc_sf(smem_u32(sSF));
      int s = 0;
      uint32_t ph = 0, aph = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        if (!mbar_wait(&tempty_bar, aph ^ 1, ab, 0x52)) break;
        tc_fence_after();
        bool ok = true;
        for (int ks = 0; ks < nS; ++ks) {
          if (!mbar_wait(&full_bar[s], ph, ab, 0x53)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = dA + (uint64_t)((s * A_STAGE) >> 4), db = dB + (uint64_t)((s * B_BYTES) >> 4);
          const uint64_t ds = dS + (uint64_t)((s * SF_BYTES) >> 4);
          // scale atoms into TMEM: A's atoms of the stage's K blocks, then per 128-row W block its atoms
#pragma unroll
          for (int a = 0; a < SFPB * KSUB; ++a)
            tmem_cp_32x128b_x4(tmem + SFA_COL + 4 * a, ds + (uint64_t)((a * 512) >> 4));
          // W: the stage holds each 128-row W block's atoms in turn; in TMEM the scales of one atom for all of
          // the tile's TBN rows are consecutive (4 columns per 128 rows), atom after atom
#pragma unroll
          for (int i = 0; i < Cf::SFB_STAGE / 512; ++i) {
            const int b = i / (SFPB * KSUB), t = i % (SFPB * KSUB);
            tmem_cp_32x128b_x4(tmem + SFB_COL + (BN / 128) * 4 * t + 4 * b,
                               ds + (uint64_t)((Cf::SFA_STAGE + i * 512) >> 4));
          }
          // 4 MMAs per 128-byte K block (32 bytes each: K = 32 E4M3 / E5M2 or K = 64 E2M1 elements). An MMA's
          // scales are consecutive bytes of a 32-bit TMEM scale column: FP8 reads byte kk of the block's atom,
          // E2M1 reads bytes 2 (kk % 2) .. +1 of atom kk / 2.
#pragma unroll
          for (int u = 0; u < KSUB; ++u)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const int atom = u * SFPB + (FMT == MX_E2M1 ? (kk >> 1) : 0);
              const uint32_t sf_id = FMT == MX_E2M1 ? 2 * (kk & 1) : kk;
              const uint64_t a_d = da + (uint64_t)((u * A_BYTES) >> 4) + (uint64_t)(kk * 2);
              const uint64_t b_d = db + (uint64_t)((u * Cf::B_SUB) >> 4) + (uint64_t)(kk * 2);
              const uint32_t acc = (ks | u | kk) != 0;
              if (FMT == MX_E2M1)
                mma_mxf4_ss(tmem, a_d, b_d, idesc_mxf4(BM, BN, sf_id), acc, tmem + SFA_COL + 4 * atom,
                            tmem + SFB_COL + (BN / 128) * 4 * atom);
              else
                mma_mxf8_ss(tmem, a_d, b_d, idesc_mxf8(BM, BN, sf_id, FMT == MX_E5M2 ? 1 : 0), acc,
                            tmem + SFA_COL + 4 * atom, tmem + SFB_COL + (BN / 128) * 4 * atom);
            }
          tc_commit(&empty_bar[s]);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull_bar);
        aph ^= 1;
      }
      tc_commit(&done_bar);
      mbar_wait_drain(&done_bar, 0);
    }
  } else {
    const int quarter = warp & 3;            // warps 2..9 -> lane quarters 2,3,0,1,2,3,0,1
    const int half = (warp - 2) >> 2;        // first or second half of the tile's columns
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      int m_blk, n_blk;
        tile_coords(t, nM, nN, group_m, m_blk, n_blk);
      if (!mbar_wait(&tfull_bar, aph, ab, 0x54)) break;
      tc_fence_after();
      const int row = m_blk * BM + quarter * 32 + lane;
      const int col0 = n_blk * BN + half * HALF_COLS;
      const uint32_t tb = tmem + ((uint32_t)(quarter * 32) << 16) + half * HALF_COLS;
      uint32_t r[HALF_COLS];
#pragma unroll
      for (int c = 0; c < HALF_COLS / 32; ++c) tmem_ld32(tb + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&tempty_bar);  // the accumulator may be overwritten from here on
      aph ^= 1;
      // Every epilogue of this GEMM starts from the accumulator rounded to bf16 (the bf16 matmul result of the
      // reference's MX matmul): rounding it here, two values per register, halves what the epilogue warps hold
      // while they work through the column slices (the rounding there is then exact).
      uint32_t pk[HALF_COLS / 2];
#pragma unroll
      for (int i = 0; i < HALF_COLS / 2; ++i) pk[i] = pack_bf16(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
      auto slice = [&](int c, float (&v)[32]) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v[2 * i] = __uint_as_float(pk[c * 16 + i] << 16);
          v[2 * i + 1] = __uint_as_float(pk[c * 16 + i] & 0xFFFF0000u);
        }
      };
      float stat = 0.f;
      if constexpr (Epi::WARP_SMEM > 0) {
        // warp-cooperative epilogue (all lanes; rows >= M are skipped inside), staged past the operand ring
        float* sm = reinterpret_cast<float*>(smem + STAGES * TX_BYTES + (warp - 2) * Epi::WARP_SMEM);
#pragma unroll
        for (int c = 0; c < HALF_COLS / 32; ++c) {
          const int col = col0 + c * 32;
          if (col < N) {
            float v[32];
            slice(c, v);
            epi.chunk_warp(m_blk * BM + quarter * 32, lane, col, v, M, sm);
          }
        }
      } else if (row < M) {
#pragma unroll
        for (int c = 0; c < HALF_COLS / 32; ++c) {
          const int col = col0 + c * 32;
          if (col < N) {
            float v[32];
            slice(c, v);
            stat += epi.chunk(row, col, v);
          }
        }
        epi.tile_done(row, col0, stat);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

template <class Epi, int TBN, int FMT = MX_E4M3>
static int launch_gemm_mx_t(const CUtensorMap& tmA, const void* a_scales, const void* w, const void* w_scales, int M,
                            int N, int K, const Epi& epi, cudaStream_t stream, int* st) {
  using C = mxg::Cfg<TBN, FMT>;
  constexpr int smem_bytes = C::SMEM_BYTES + mxg::EPI_WARPS * Epi::WARP_SMEM;
  static_assert(smem_bytes <= mxg::SMEM_LIMIT, "operand ring + epilogue staging exceed the shared memory of a CTA");
  const int row_bytes = K / 32 * mx_block_bytes(FMT);
  CUtensorMap tmB;
  int err = make_tmap_2d(&tmB, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, row_bytes, row_bytes, mxg::BK, TBN);
  if (err) return err;
  static bool attr_set[64] = {};  // per instantiation and device
  const int dix = device_index();
  if (dix < 0) return set_error(LBW_ERR_CUDA, "mx gemm: cudaGetDevice failed");
  if (!attr_set[dix]) {
    err = cuda_check(cudaFuncSetAttribute(gemm_mx_kernel<Epi, TBN, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          smem_bytes),
                     "mx gemm smem attribute");
    if (err) return err;
    attr_set[dix] = true;
  }
  const int tiles = ((M + mxg::BM - 1) / mxg::BM) * ((N + TBN - 1) / TBN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  gemm_mx_kernel<Epi, TBN, FMT><<<grid, mxg::THREADS, smem_bytes, stream>>>(
      tmA, tmB, reinterpret_cast<const uint8_t*>(a_scales), reinterpret_cast<const uint8_t*>(w_scales), M, N, K,
      group_rows(M, row_bytes, 1), epi, st);
  return cuda_check(cudaGetLastError(), "mx gemm launch");
}

// fmt: MX_E4M3 (the reference's default), MX_E5M2 (LINGBOT_MX_FP8=float8_e5m2) or MX_E2M1 (MXFP4). A and W hold
// K / 32 blocks per row: 32 bytes each for the FP8 formats, 16 (packed nibbles) for E2M1.
template <class Epi, int FMT = MX_E4M3>
static int launch_gemm_mx(const void* a, const void* a_scales, const void* w, const void* w_scales, int M, int N, int K,
                          const Epi& epi, cudaStream_t stream) {
  using namespace mxg;
  constexpr int fmt = FMT;
  const int ke = fmt == MX_E2M1 ? 256 : 128;  // elements of one 128-byte K block
  if (M <= 0 || N <= 0 || K <= 0) return set_error(LBW_ERR_SHAPE, "mx gemm: empty problem %d x %d x %d", M, N, K);
  if (K % ke) return set_error(LBW_ERR_SHAPE, "mx gemm: K=%d must be a multiple of %d", K, ke);
  if (N % 128) return set_error(LBW_ERR_SHAPE, "mx gemm: N=%d must be a multiple of 128", N);
  if (!a || !w || !a_scales || !w_scales) return set_error(LBW_ERR_INVALID, "mx gemm: null operand");
  if (!aligned(a_scales, 16) || !aligned(w_scales, 16)) return set_error(LBW_ERR_ALIGN, "mx gemm: scales alignment");
  int err = 0;
  int* st = device_status(&err);
  if (!st) return err;
  const int row_bytes = K / 32 * mx_block_bytes(fmt);
  CUtensorMap tmA;
  if ((err = make_tmap_2d(&tmA, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, row_bytes, row_bytes, BK, BM))) return err;
  const long long mt = (M + BM - 1) / BM;
  const bool can128 = (K / ke) % 2 == 0;  // 128-wide tiles stage two K blocks
  const int force = tile_n_override();
  const bool narrow = can128 && (force ? force == 128 : prefer_narrow_tiles(mt, N));
  return narrow ? launch_gemm_mx_t<Epi, 128, FMT>(tmA, a_scales, w, w_scales, M, N, K, epi, stream, st)
                : launch_gemm_mx_t<Epi, 256, FMT>(tmA, a_scales, w, w_scales, M, N, K, epi, stream, st);
}

static bool ok16mx(const void* p) { return p == nullptr || aligned(p, 16); }

// The MXFP8 element formats of the block Linears (LINGBOT_MX_FP8): E4M3 or E5M2.
static int mx_fp8_fmt_ok(int fmt, const char* who) {
  if (fmt == MX_E4M3 || fmt == MX_E5M2) return LBW_OK;
  return set_error(LBW_ERR_INVALID, "%s: element format %d (E4M3 or E5M2)", who, fmt);
}
template <class Epi>
static int launch_gemm_mx_fp8(int fmt, const void* a, const void* a_scales, const void* w, const void* w_scales, int M,
                              int N, int K, const Epi& epi, cudaStream_t stream) {
  if (fmt == MX_E5M2) return launch_gemm_mx<Epi, MX_E5M2>(a, a_scales, w, w_scales, M, N, K, epi, stream);
  return launch_gemm_mx<Epi, MX_E4M3>(a, a_scales, w, w_scales, M, N, K, epi, stream);
}

}  // namespace lbw

using namespace lbw;

extern "C" {

int lbw_mx_linear(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias, int m,
                  int n, int k, void* out, void* stream) {
  if (!out) return set_error(LBW_ERR_INVALID, "lbw_mx_linear: null output");
  if (!ok16mx(out) || !ok16mx(bias)) return set_error(LBW_ERR_ALIGN, "lbw_mx_linear: alignment");
  EpiStore e{};
  e.out[0] = e.out[1] = e.out[2] = reinterpret_cast<__nv_bfloat16*>(out);
  e.ld[0] = e.ld[1] = e.ld[2] = n;
  e.region_cols = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.round_acc = 1;
  return launch_gemm_mx(a, a_scales, w, w_scales, m, n, k, e, reinterpret_cast<cudaStream_t>(stream));
}

int lbw_mx_linear_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                      int m, int n, int k, int fmt, void* out, void* stream) {
  if (!out) return set_error(LBW_ERR_INVALID, "lbw_mx_linear_fmt: null output");
  if (!ok16mx(out) || !ok16mx(bias)) return set_error(LBW_ERR_ALIGN, "lbw_mx_linear_fmt: alignment");
  EpiStore e{};
  e.out[0] = e.out[1] = e.out[2] = reinterpret_cast<__nv_bfloat16*>(out);
  e.ld[0] = e.ld[1] = e.ld[2] = n;
  e.region_cols = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.round_acc = 1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (fmt == MX_E4M3) return launch_gemm_mx<EpiStore, MX_E4M3>(a, a_scales, w, w_scales, m, n, k, e, s);
  if (fmt == MX_E5M2) return launch_gemm_mx<EpiStore, MX_E5M2>(a, a_scales, w, w_scales, m, n, k, e, s);
  if (fmt == MX_E2M1) return launch_gemm_mx<EpiStore, MX_E2M1>(a, a_scales, w, w_scales, m, n, k, e, s);
  return set_error(LBW_ERR_INVALID, "lbw_mx_linear_fmt: element format %d", fmt);
}

int lbw_mx_linear_gelu(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                       int m, int n, int k, void* out, void* out_scales, void* stream) {
  return lbw_mx_linear_gelu_fmt(a, a_scales, w, w_scales, bias, m, n, k, MX_E4M3, out, out_scales, stream);
}

int lbw_mx_linear_gelu_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                           int m, int n, int k, int fmt, void* out, void* out_scales, void* stream) {
  if (!out || !out_scales || !bias) return set_error(LBW_ERR_INVALID, "lbw_mx_linear_gelu: null pointer");
  if (fmt != MX_E4M3 && fmt != MX_E5M2)
    return set_error(LBW_ERR_INVALID, "lbw_mx_linear_gelu: element format %d (E4M3 or E5M2)", fmt);
  if (!ok16mx(out) || !ok16mx(bias)) return set_error(LBW_ERR_ALIGN, "lbw_mx_linear_gelu: alignment");
  EpiGeluMX e{};
  e.data = reinterpret_cast<uint8_t*>(out);
  e.scales = reinterpret_cast<uint8_t*>(out_scales);
  e.ld = n;
  e.sf_cols = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.fmt = fmt;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (fmt == MX_E5M2) return launch_gemm_mx<EpiGeluMX, MX_E5M2>(a, a_scales, w, w_scales, m, n, k, e, s);
  return launch_gemm_mx(a, a_scales, w, w_scales, m, n, k, e, s);
}

int lbw_mx_linear_residual(const void* a, const void* a_scales, const void* w, const void* w_scales,
                           const void* bias, int m, int n, int k, float* x, const float* gate, void* stream) {
  return lbw_mx_linear_residual_fmt(a, a_scales, w, w_scales, bias, m, n, k, MX_E4M3, x, gate, stream);
}

int lbw_mx_linear_residual_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales,
                               const void* bias, int m, int n, int k, int fmt, float* x, const float* gate,
                               void* stream) {
  if (!x) return set_error(LBW_ERR_INVALID, "lbw_mx_linear_residual: null residual");
  if (fmt != MX_E4M3 && fmt != MX_E5M2)
    return set_error(LBW_ERR_INVALID, "lbw_mx_linear_residual: element format %d (E4M3 or E5M2)", fmt);
  if (!ok16mx(x) || !ok16mx(gate) || !ok16mx(bias)) return set_error(LBW_ERR_ALIGN, "lbw_mx_linear_residual: alignment");
  EpiResidualT<false, 16> e{};
  e.x = x;
  e.ldx = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.gate = gate;
  e.round_acc = 1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (fmt == MX_E5M2) return launch_gemm_mx<EpiResidualT<false, 16>, MX_E5M2>(a, a_scales, w, w_scales, m, n, k, e, s);
  return launch_gemm_mx(a, a_scales, w, w_scales, m, n, k, e, s);
}

// ---- the other block Linears in MXFP8 (LINGBOT_LIN_MX, wan/modules/model_fast.py:1266-1269, :1442-1494): each is
// y = bf16(mm(x, W)) + b in bf16 (_mx_matmul :1403-1410), so every epilogue below rounds the accumulator first.

int lbw_mx_qkv_proj(const void* h, const void* h_scales, const void* w_qkv, const void* w_qkv_scales,
                    const void* b_qkv, int m, int c, void* q_raw, void* k_raw, float* ss_q, float* ss_k, void* v_out,
                    long long ldv, int v_row_off, void* stream) {
  return lbw_mx_qkv_proj_fmt(h, h_scales, w_qkv, w_qkv_scales, b_qkv, m, c, MX_E4M3, q_raw, k_raw, ss_q, ss_k, v_out,
                             ldv, v_row_off, stream);
}

int lbw_mx_qkv_proj_fmt(const void* h, const void* h_scales, const void* w_qkv, const void* w_qkv_scales,
                        const void* b_qkv, int m, int c, int fmt, void* q_raw, void* k_raw, float* ss_q, float* ss_k,
                        void* v_out, long long ldv, int v_row_off, void* stream) {
  if (int err = mx_fp8_fmt_ok(fmt, "lbw_mx_qkv_proj")) return err;
  if (!q_raw || !k_raw || !v_out || !ss_q || !ss_k) return set_error(LBW_ERR_INVALID, "lbw_mx_qkv_proj: null pointer");
  if (c % mxg::BK) return set_error(LBW_ERR_SHAPE, "lbw_mx_qkv_proj: dim %d must be a multiple of %d", c, mxg::BK);
  if (!ok16mx(q_raw) || !ok16mx(k_raw) || !ok16mx(v_out) || !ok16mx(b_qkv) || ldv % 8 || v_row_off < 0)
    return set_error(LBW_ERR_ALIGN, "lbw_mx_qkv_proj: alignment");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int err = cuda_check(cudaMemsetAsync(ss_q, 0, sizeof(float) * m, s), "ss clear");
  if (!err) err = cuda_check(cudaMemsetAsync(ss_k, 0, sizeof(float) * m, s), "ss clear");
  if (err) return err;
  EpiStore e{};
  e.out[0] = reinterpret_cast<__nv_bfloat16*>(q_raw);
  e.out[1] = reinterpret_cast<__nv_bfloat16*>(k_raw);
  e.out[2] = reinterpret_cast<__nv_bfloat16*>(v_out);
  e.ld[0] = c; e.ld[1] = c; e.ld[2] = ldv;
  e.row_off[2] = v_row_off;
  e.ss[0] = ss_q; e.ss[1] = ss_k; e.ss[2] = nullptr;
  e.region_cols = c;
  e.ss_per_chunk = (c % 256) != 0;   // a region boundary inside a 256-column tile: sums per 32-column chunk
  e.bias = reinterpret_cast<const __nv_bfloat16*>(b_qkv);
  e.round_acc = 1;
  return launch_gemm_mx_fp8(fmt, h, h_scales, w_qkv, w_qkv_scales, m, 3 * c, c, e, s);
}

int lbw_mx_linear_rowss(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                        int m, int n, int k, void* out, float* ss, void* stream) {
  return lbw_mx_linear_rowss_fmt(a, a_scales, w, w_scales, bias, m, n, k, MX_E4M3, out, ss, stream);
}

int lbw_mx_linear_rowss_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                            int m, int n, int k, int fmt, void* out, float* ss, void* stream) {
  if (int err = mx_fp8_fmt_ok(fmt, "lbw_mx_linear_rowss")) return err;
  if (!out || !ss) return set_error(LBW_ERR_INVALID, "lbw_mx_linear_rowss: null pointer");
  if (!ok16mx(out) || !ok16mx(bias)) return set_error(LBW_ERR_ALIGN, "lbw_mx_linear_rowss: alignment");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int err = cuda_check(cudaMemsetAsync(ss, 0, sizeof(float) * m, s), "ss clear");
  if (err) return err;
  EpiStore e{};
  e.out[0] = e.out[1] = e.out[2] = reinterpret_cast<__nv_bfloat16*>(out);
  e.ld[0] = e.ld[1] = e.ld[2] = n;
  e.ss[0] = ss;
  e.region_cols = n;
  e.ss_per_chunk = (n % 256) != 0;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.round_acc = 1;
  return launch_gemm_mx_fp8(fmt, a, a_scales, w, w_scales, m, n, k, e, s);
}

int lbw_mx_linear_residual_film(const void* a, const void* a_scales, const void* w, const void* w_scales,
                                const void* bias, int m, int n, int k, float* x, const float* gate,
                                const void* film_scale, const void* film_shift, void* stream) {
  return lbw_mx_linear_residual_film_fmt(a, a_scales, w, w_scales, bias, m, n, k, MX_E4M3, x, gate, film_scale,
                                         film_shift, stream);
}

int lbw_mx_linear_residual_film_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales,
                                    const void* bias, int m, int n, int k, int fmt, float* x, const float* gate,
                                    const void* film_scale, const void* film_shift, void* stream) {
  if (int err = mx_fp8_fmt_ok(fmt, "lbw_mx_linear_residual_film")) return err;
  if (!x) return set_error(LBW_ERR_INVALID, "lbw_mx_linear_residual_film: null residual");
  if ((film_scale == nullptr) != (film_shift == nullptr))
    return set_error(LBW_ERR_INVALID, "lbw_mx_linear_residual_film: FiLM needs both scale and shift");
  if (!ok16mx(x) || !ok16mx(gate) || !ok16mx(bias) || !ok16mx(film_scale) || !ok16mx(film_shift))
    return set_error(LBW_ERR_ALIGN, "lbw_mx_linear_residual_film: alignment");
  EpiResidualT<true, 16> e{};
  e.x = x;
  e.ldx = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.gate = gate;
  e.film_scale = reinterpret_cast<const __nv_bfloat16*>(film_scale);
  e.film_shift = reinterpret_cast<const __nv_bfloat16*>(film_shift);
  e.ldf = n;
  e.round_acc = 1;
  return launch_gemm_mx_fp8(fmt, a, a_scales, w, w_scales, m, n, k, e, reinterpret_cast<cudaStream_t>(stream));
}

int lbw_mx_linear_act(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                      const void* addend, int silu, int m, int n, int k, void* out, void* stream) {
  return lbw_mx_linear_act_fmt(a, a_scales, w, w_scales, bias, addend, silu, m, n, k, MX_E4M3, out, stream);
}

int lbw_mx_linear_act_fmt(const void* a, const void* a_scales, const void* w, const void* w_scales, const void* bias,
                          const void* addend, int silu, int m, int n, int k, int fmt, void* out, void* stream) {
  if (int err = mx_fp8_fmt_ok(fmt, "lbw_mx_linear_act")) return err;
  if (!out) return set_error(LBW_ERR_INVALID, "lbw_mx_linear_act: null output");
  if (!ok16mx(out) || !ok16mx(bias) || !ok16mx(addend)) return set_error(LBW_ERR_ALIGN, "lbw_mx_linear_act: alignment");
  EpiAct e{};
  e.out = reinterpret_cast<__nv_bfloat16*>(out);
  e.ldo = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.addend = reinterpret_cast<const __nv_bfloat16*>(addend);
  e.silu = silu;
  e.round_acc = 1;
  return launch_gemm_mx_fp8(fmt, a, a_scales, w, w_scales, m, n, k, e, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
