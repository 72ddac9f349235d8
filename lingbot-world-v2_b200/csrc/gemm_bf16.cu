// Persistent tcgen05 GEMM, bf16 x bf16 -> fp32 (TMEM) -> fused epilogue.
//
//   out[m, n] = epilogue( sum_k A[m, k] * W[n, k] )      A: [M, K] activations, W: [N, K] = nn.Linear weight
//
// Tiles: 128 x 256 output per tile (one UMMA M=128, N=256 per K step of 16), K staged 64 at a time
// (one 128-byte swizzled row per M/N row) through a 4-deep TMA ring. Warp roles:
//   warp 0   TMA producer (one elected lane)
//   warp 1   UMMA issuer (one elected lane) and TMEM owner (2 x 256 fp32 accumulator columns)
//   warps 2-9 epilogue: tcgen05.ld of the accumulator (thread = output row), fused math, global stores;
//            warps w and w+4 share TMEM lane quarter w % 4 and take the left / right half of the tile's columns.
// The two accumulators let the epilogue of tile i run while the MMAs of tile i+1 proceed.
//
// Epilogues used by the block forward (CausalWanAttentionBlock, wan/modules/model_fast.py:2912-3116):
//   EpiStore     bias + bf16 store into up to three column regions (the fused q|k|v projection writes
//                q and k to scratch and v straight into the KV-cache destination chunk), optionally
//                accumulating each row's sum of squares of the rounded outputs for the RMSNorm that
//                follows (WanRMSNorm, wan/modules/model.py:126-143).
//   EpiResidual  x += bf16(acc + b) * gate, then optional FiLM x = (1 + s) * x + t (model_fast.py:3063-3089,
//                :3110-3111) on the fp32 residual stream.
//   EpiGelu      GELU_tanh(bf16(acc) + b), optionally followed by an MXFP8 quantise-dequantise of each
//                32-column block (the FFN-up epilogue, kernels/ffn_epi.py:15-37, and the activation
//                quantisation of kernels/ffn_mx.py:159-182) for the bf16-pipe MX FFN variant.
//
// The same kernel is the implicit-GEMM convolution of the VAE decoder (ConvA): the activations are frames
// stored channels-last with a one-pixel zero border, [frames][H + 2][W + 2][C], so that every tap (kt, kh, kw)
// of a (kt x kh x kw) kernel reads the same rows shifted by a constant: the A tile of a 64-channel K block of
// tap t is one TMA load at row m0 + off[t] (rows before the tensor or past its end read as zeros).
#include <math.h>

#include <mutex>

#include "host_common.cuh"
#include "lbw_common.cuh"
#include "mx_common.cuh"
#include "epilogues.cuh"

namespace lbw {

namespace gemm {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = BN * BK * 2;   // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
constexpr int THREADS = 320;
constexpr int EPI_THREADS = THREADS - 64;
constexpr int EPI_WARPS = EPI_THREADS / 32;
// Tile width TBN (256, or 128 when 256-wide tiles would leave the last wave mostly idle; the VAE convolutions also
// use 192 for 192 / 384 / 768 output channels, 96 for 96 and 64 for the 3-channel head): ring depth and shared
// memory per tile width.
// A 128-wide tile's MMAs (N = 128) take half as long as a 256-wide tile's, so its stages hold two 64-wide K
// blocks: the MMA thread then waits once per 8 MMAs instead of once per 4 (each wait leaves the tensor pipe
// idle for ~100 cycles, because the lone issuing thread has nothing else in flight).
template <int TBN> struct Cfg {
  static_assert(TBN == 64 || TBN == 96 || TBN == 128 || TBN == 192 || TBN == 256, "tile widths 64, 96, 128, 192, 256");
  static constexpr int KSUB = TBN >= 192 ? 1 : 2;           // 64-wide K blocks per stage
  static constexpr int BKS = BK * KSUB;                      // K per stage
  static constexpr int A_SUB = BM * BK * 2, B_SUB = TBN * BK * 2;
  static constexpr int A_STAGE = A_SUB * KSUB, B_STAGE = B_SUB * KSUB;
  static constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
  static constexpr int STAGES = TBN == 128 ? 3 : 4;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
  // two accumulators of TBN columns, the second at column ACC (96 columns are kept 128 apart); the allocation is
  // a power of two
  static constexpr uint32_t ACC = TBN == 96 ? 128 : TBN;
  static constexpr uint32_t TMEM_COLS = 2 * ACC <= 128 ? 128 : (2 * ACC <= 256 ? 256 : 512);
  static constexpr int NCHUNK = TBN / 32;                 // 32-column epilogue chunks per tile row
  static constexpr int NCH = (NCHUNK + 1) / 2;            // per warp of a lane-quarter pair (the second may get fewer)
};
}  // namespace gemm

// ------------------------------------------------------------------------------------------
// A-operand addressing: the (column, row) TMA coordinates of the 64-wide K block starting at column k0 for the
// tile rows starting at row0.
// ------------------------------------------------------------------------------------------
struct PlainA {
  LBW_DEV void coords(int k0, int row0, int& x, int& y) const { x = k0; y = row0; }
};
constexpr int CONV_MAX_TAPS = 27;
struct ConvA {
  int cblocks;               // 64-channel blocks per tap
  int off[CONV_MAX_TAPS];    // row offset of each tap's input rows (negative: reads before the tensor = 0)
  LBW_DEV void coords(int k0, int row0, int& x, int& y) const {
    const int kb = k0 >> 6, tap = kb / cblocks;
    x = (kb - tap * cblocks) << 6;
    y = row0 + off[tap];
  }
};

// ------------------------------------------------------------------------------------------
// kernel
// ------------------------------------------------------------------------------------------
template <class Epi, int TBN = 256, class AMap = PlainA>
__global__ void __launch_bounds__(gemm::THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                     int K, int group_m, Epi epi, int* status, const __grid_constant__ AMap amap) {
  using gemm::BM;
  using gemm::BK;
  using C = gemm::Cfg<TBN>;
  constexpr int BN = TBN;
  constexpr int STAGES = C::STAGES;
  constexpr int STAGE_BYTES = C::STAGE_BYTES;
  constexpr uint32_t TMEM_COLS = C::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], tfull_bar[2], tempty_bar[2], done_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], gemm::EPI_THREADS);
    }
    mbar_init(&done_bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(&tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const Abort ab{status, &abort_flag};

  const int nM = (M + BM - 1) / BM, nN = (N + BN - 1) / BN, nK = K / C::BKS;
  const int tiles = nM * nN;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      long long issued = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        int m_blk, n_blk;
        tile_coords(t, nM, nN, group_m, m_blk, n_blk);
        bool ok = true;
        for (int kb = 0; kb < nK; ++kb) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1, ab, 1)) { ok = false; break; }
          uint8_t* sa = smem + s * STAGE_BYTES;
          mbar_expect_tx(&full_bar[s], STAGE_BYTES);
#pragma unroll
          for (int u = 0; u < C::KSUB; ++u) {
            int ax, ay;
            amap.coords(kb * C::BKS + u * BK, m_blk * BM, ax, ay);
            tma_load_2d(sa + u * C::A_SUB, &tmA, &full_bar[s], ax, ay);
            tma_load_2d(sa + C::A_STAGE + u * C::B_SUB, &tmB, &full_bar[s], kb * C::BKS + u * BK, n_blk * BN);
          }
          ++issued;
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
      }
      // Drain: every load issued into the ring must have landed before the CTA exits.
      for (long long i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i)
        mbar_wait_drain(&full_bar[i % STAGES], (uint32_t)((i / STAGES) & 1));
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(BM, BN, 0, 0);
      // descriptors built once: a shared-memory byte offset o adds o >> 4 to the start-address field
      const uint64_t d0 = sdesc_kmajor_sw128(smem_u32(smem));
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        if (!mbar_wait(&tempty_bar[acc], aph ^ 1, ab, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * C::ACC;
        bool ok = true;
        for (int kb = 0; kb < nK; ++kb) {
          if (!mbar_wait(&full_bar[s], ph, ab, 3)) { ok = false; break; }
          tc_fence_after();
          const uint64_t da = d0 + (uint64_t)((s * STAGE_BYTES) >> 4), db = da + (uint64_t)(C::A_STAGE >> 4);
#pragma unroll
          for (int u = 0; u < C::KSUB; ++u)
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              mma_f16_ss(d, da + (uint64_t)((u * C::A_SUB) >> 4) + (uint64_t)(kk * 2),
                         db + (uint64_t)((u * C::B_SUB) >> 4) + (uint64_t)(kk * 2), idesc, (kb | u | kk) != 0);
          tc_commit(&empty_bar[s]);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull_bar[acc]);
        acc ^= 1;
        if (acc == 0) aph ^= 1;
      }
      // All MMAs issued by this thread complete before TMEM is released.
      tc_commit(&done_bar);
      mbar_wait_drain(&done_bar, 0);
    }
  } else {
    const int quarter = warp & 3;          // warps 2..9 -> TMEM lane quarters 2,3,0,1,2,3,0,1
    constexpr int NCH = C::NCH;            // 32-column chunks per warp
    const int c0 = ((warp - 2) >> 2) * NCH;
    int acc = 0;
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      int m_blk, n_blk;
        tile_coords(t, nM, nN, group_m, m_blk, n_blk);
      if (!mbar_wait(&tfull_bar[acc], aph, ab, 4)) break;
      tc_fence_after();
      const int row = m_blk * BM + quarter * 32 + lane;
      const uint32_t tb = tmem + ((uint32_t)(quarter * 32) << 16) + acc * C::ACC;
      float stat = 0.f;
      if constexpr (row_norm<Epi>::value) {
        // the row's sum of squares over every column chunk of the tile (both warps of the pair read all of them),
        // then this warp's half of the columns normalised and written
        float ss = 0.f;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          const int col = n_blk * BN + c * 32;
          if (col >= N) break;  // warp-uniform
          uint32_t r[32];
          tmem_ld32(tb + c * 32, r);
          tmem_ld_wait();
          if (row < M) ss += epi.sumsq(row, col, reinterpret_cast<const float(&)[32]>(r));
        }
#pragma unroll 1
        for (int c = c0; c < c0 + NCH && c < C::NCHUNK; ++c) {
          const int col = n_blk * BN + c * 32;
          if (col >= N) break;  // warp-uniform
          uint32_t r[32];
          tmem_ld32(tb + c * 32, r);
          tmem_ld_wait();
          if (row < M) epi.chunk_norm(row, col, reinterpret_cast<const float(&)[32]>(r), ss);
        }
      }
#pragma unroll 1
      for (int c = c0; c < c0 + NCH && c < C::NCHUNK && !row_norm<Epi>::value; ++c) {
        const int col = n_blk * BN + c * 32;
        if (col >= N) break;  // warp-uniform
        uint32_t r[32];
        tmem_ld32(tb + c * 32, r);
        tmem_ld_wait();
        if constexpr (Epi::WARP_SMEM > 0) {
          float* sm = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + (warp - 2) * Epi::WARP_SMEM);
          epi.chunk_warp(m_blk * BM + quarter * 32, lane, col, reinterpret_cast<const float(&)[32]>(r), M, sm);
        } else if (row < M) {
          stat += epi.chunk(row, col, reinterpret_cast<const float(&)[32]>(r));
        }
      }
      if (row < M) epi.tile_done(row, n_blk * BN, stat);
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      acc ^= 1;
      if (acc == 0) aph ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

inline void fit_epi(EpiStore& e, int tbn) { e.ss_per_chunk = (e.region_cols % tbn) != 0; }
template <class Epi>
inline void fit_epi(Epi&, int) {}

template <class Epi, int TBN, class AMap = PlainA>
static int launch_gemm_t(const CUtensorMap& tmA, const void* W, long long ldw, int M, int N, int K, Epi epi,
                         cudaStream_t stream, int* st, const AMap& amap = AMap{}, int a_cols = 0) {
  using C = gemm::Cfg<TBN>;
  CUtensorMap tmB;
  int err = make_tmap_2d(&tmB, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, ldw, gemm::BK, TBN);
  if (err) return err;
  fit_epi(epi, TBN);
  static bool attr_set[64] = {};  // per instantiation and device
  const int dix = device_index();
  if (dix < 0) return set_error(LBW_ERR_CUDA, "gemm: cudaGetDevice failed");
  if (!attr_set[dix]) {
    err = cuda_check(cudaFuncSetAttribute(gemm_bf16_kernel<Epi, TBN, AMap>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          C::SMEM_BYTES + gemm::EPI_WARPS * Epi::WARP_SMEM),
                     "gemm smem attribute");
    if (err) return err;
    attr_set[dix] = true;
  }
  const int tiles = ((M + gemm::BM - 1) / gemm::BM) * ((N + TBN - 1) / TBN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  // tile groups keep ~40 MB of A rows in L2: A's row width is K for a GEMM, the channel count for a convolution
  const int group = group_rows(M, a_cols > 0 ? a_cols : K, 2);
  gemm_bf16_kernel<Epi, TBN, AMap><<<grid, gemm::THREADS, C::SMEM_BYTES + gemm::EPI_WARPS * Epi::WARP_SMEM, stream>>>(
      tmA, tmB, M, N, K, group, epi, st, amap);
  return cuda_check(cudaGetLastError(), "gemm launch");
}

template <class Epi>
static int launch_gemm(const void* A, long long lda, const void* W, long long ldw, int M, int N, int K, const Epi& epi,
                       cudaStream_t stream) {
  using namespace gemm;
  if (M <= 0 || N <= 0 || K <= 0) return set_error(LBW_ERR_SHAPE, "gemm: empty problem %d x %d x %d", M, N, K);
  if (K % BK) return set_error(LBW_ERR_SHAPE, "gemm: K=%d must be a multiple of %d", K, BK);
  if (N % 32) return set_error(LBW_ERR_SHAPE, "gemm: N=%d must be a multiple of 32", N);
  if (!A || !W) return set_error(LBW_ERR_INVALID, "gemm: null operand");
  int err = 0;
  int* st = device_status(&err);
  if (!st) return err;
  CUtensorMap tmA;
  if ((err = make_tmap_2d(&tmA, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, lda, BK, BM))) return err;
  // 128-wide tiles when 256-wide ones would leave the last round of tiles mostly idle (few rows per rank)
  const long long mt = (M + BM - 1) / BM;
  const bool can128 = K % gemm::Cfg<128>::BKS == 0;
  const int force = tile_n_override();
  const bool use128 = can128 && (force ? force == 128 : prefer_narrow_tiles(mt, N));
  if (use128) return launch_gemm_t<Epi, 128>(tmA, W, ldw, M, N, K, epi, stream, st);
  return launch_gemm_t<Epi, 256>(tmA, W, ldw, M, N, K, epi, stream, st);
}

static bool ok16(const void* p) { return p == nullptr || aligned(p, 16); }

}  // namespace lbw

using namespace lbw;

extern "C" {

int lbw_gemm_bf16(const void* a, long long lda, const void* w, long long ldw, const void* bias, void* out,
                  long long ldo, int m, int n, int k, void* stream) {
  if (!out) return set_error(LBW_ERR_INVALID, "lbw_gemm_bf16: null output");
  if (!ok16(bias) || !ok16(out) || ldo % 8) return set_error(LBW_ERR_ALIGN, "lbw_gemm_bf16: output/bias alignment");
  EpiStore e{};
  e.out[0] = e.out[1] = e.out[2] = reinterpret_cast<__nv_bfloat16*>(out);
  e.ld[0] = e.ld[1] = e.ld[2] = ldo;
  e.region_cols = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  return launch_gemm(a, lda, w, ldw, m, n, k, e, reinterpret_cast<cudaStream_t>(stream));
}

int lbw_qkv_proj(const void* h, const void* w_qkv, const void* b_qkv, int m, int c, void* q_raw, void* k_raw,
                 float* ss_q, float* ss_k, void* v_out, long long ldv, int v_row_off, void* stream) {
  if (!q_raw || !k_raw || !v_out || !ss_q || !ss_k) return set_error(LBW_ERR_INVALID, "lbw_qkv_proj: null pointer");
  if (c % 128) return set_error(LBW_ERR_SHAPE, "lbw_qkv_proj: dim %d must be a multiple of 128", c);
  if (!ok16(q_raw) || !ok16(k_raw) || !ok16(v_out) || !ok16(b_qkv) || ldv % 8)
    return set_error(LBW_ERR_ALIGN, "lbw_qkv_proj: alignment");
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
  e.ss_per_chunk = (c % gemm::BN) != 0;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(b_qkv);
  return launch_gemm(h, c, w_qkv, c, m, 3 * c, c, e, s);
}

int lbw_linear_rowss(const void* a, const void* w, const void* bias, int m, int n, int k, void* out, float* ss,
                     void* stream) {
  if (!out || !ss) return set_error(LBW_ERR_INVALID, "lbw_linear_rowss: null pointer");
  if (!ok16(out) || !ok16(bias)) return set_error(LBW_ERR_ALIGN, "lbw_linear_rowss: alignment");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int err = cuda_check(cudaMemsetAsync(ss, 0, sizeof(float) * m, s), "ss clear");
  if (err) return err;
  EpiStore e{};
  e.out[0] = e.out[1] = e.out[2] = reinterpret_cast<__nv_bfloat16*>(out);
  e.ld[0] = e.ld[1] = e.ld[2] = n;
  e.ss[0] = ss;
  e.region_cols = n;
  e.ss_per_chunk = (n % gemm::BN) != 0;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  return launch_gemm(a, k, w, k, m, n, k, e, s);
}

int lbw_linear_residual(const void* a, const void* w, const void* bias, int m, int n, int k, float* x,
                        const float* gate, const void* film_scale, const void* film_shift, void* stream) {
  if (!x) return set_error(LBW_ERR_INVALID, "lbw_linear_residual: null residual");
  if ((film_scale == nullptr) != (film_shift == nullptr))
    return set_error(LBW_ERR_INVALID, "lbw_linear_residual: FiLM needs both scale and shift");
  if (!ok16(x) || !ok16(gate) || !ok16(bias) || !ok16(film_scale) || !ok16(film_shift))
    return set_error(LBW_ERR_ALIGN, "lbw_linear_residual: alignment");
  EpiResidual e{};
  e.x = x; e.ldx = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.gate = gate;
  e.film_scale = reinterpret_cast<const __nv_bfloat16*>(film_scale);
  e.film_shift = reinterpret_cast<const __nv_bfloat16*>(film_shift);
  e.ldf = n;
  return launch_gemm(a, k, w, k, m, n, k, e, reinterpret_cast<cudaStream_t>(stream));
}

int lbw_linear_gelu(const void* a, const void* w, const void* bias, int m, int n, int k, void* out, int mx_qdq,
                    void* stream) {
  if (!out || !bias) return set_error(LBW_ERR_INVALID, "lbw_linear_gelu: null pointer");
  if (!ok16(out) || !ok16(bias)) return set_error(LBW_ERR_ALIGN, "lbw_linear_gelu: alignment");
  EpiGelu e{};
  e.out = reinterpret_cast<__nv_bfloat16*>(out);
  e.ldo = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.qdq = mx_qdq;
  return launch_gemm(a, k, w, k, m, n, k, e, reinterpret_cast<cudaStream_t>(stream));
}

int lbw_gemm_f32(const void* a, long long lda, const void* w, long long ldw, float* out, long long ldo, int m, int n,
                 int k, void* stream) {
  if (!out) return set_error(LBW_ERR_INVALID, "lbw_gemm_f32: null output");
  if (!ok16(out) || ldo % 4 || lda % 8 || ldw % 8) return set_error(LBW_ERR_ALIGN, "lbw_gemm_f32: alignment");
  EpiStoreF32 e{};
  e.out = out;
  e.ldo = ldo;
  return launch_gemm(a, lda, w, ldw, m, n, k, e, reinterpret_cast<cudaStream_t>(stream));
}

int lbw_vae_conv(const void* x, long long in_rows, int c_in, const void* w, const void* bias, int c_out, int kt, int kh,
                 int kw, int frames, int h, int wd, const void* residual, void* out, void* stream) {
  using namespace gemm;
  if (!x || !w || !out) return set_error(LBW_ERR_INVALID, "lbw_vae_conv: null pointer");
  if ((kt != 1 && kt != 3) || kh != kw || (kh != 1 && kh != 3))
    return set_error(LBW_ERR_SHAPE, "lbw_vae_conv: kernel %dx%dx%d (kt 1 or 3, kh = kw 1 or 3)", kt, kh, kw);
  if (c_in <= 0 || c_in % 8 || c_out <= 0 || c_out % 32 || frames <= 0 || h <= 0 || wd <= 0)
    return set_error(LBW_ERR_SHAPE, "lbw_vae_conv: channels %d -> %d (multiples of 8 / 32), %d frames of %dx%d",
                     c_in, c_out, frames, h, wd);
  const long long P = (long long)(h + 2) * (wd + 2);
  const long long M = (long long)frames * P;
  if (in_rows < (long long)(frames + kt - 1) * P)
    return set_error(LBW_ERR_SHAPE, "lbw_vae_conv: %lld input rows, need %lld (%d history frames)", in_rows,
                     (long long)(frames + kt - 1) * P, kt - 1);
  if (M > (1LL << 30) || in_rows > (1LL << 31) - 1)
    return set_error(LBW_ERR_SHAPE, "lbw_vae_conv: %lld rows exceed the kernel's int indexing", M);
  if (!aligned(x, 16) || !aligned(w, 16) || !ok16(out) || !ok16(bias) || !ok16(residual))
    return set_error(LBW_ERR_ALIGN, "lbw_vae_conv: alignment");
  int err = 0;
  int* st = device_status(&err);
  if (!st) return err;
  // K blocks of 64 channels per tap; the channels past c_in of the last block lie outside the tensor map's
  // columns, so TMA fills them with zeros (and the packed weights hold zeros there)
  ConvA amap{};
  amap.cblocks = (c_in + 63) / 64;
  int t = 0;
  for (int a = 0; a < kt; ++a)
    for (int b = 0; b < kh; ++b)
      for (int c = 0; c < kw; ++c)
        amap.off[t++] = (int)(a * P + (b - kh / 2) * (long long)(wd + 2) + (c - kw / 2));
  const int K = t * amap.cblocks * 64;
  CUtensorMap tmA;
  if ((err = make_tmap_2d(&tmA, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, in_rows, c_in, c_in, BK, BM))) return err;
  EpiConv e{};
  e.out = reinterpret_cast<__nv_bfloat16*>(out);
  e.ldo = c_out;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  e.ldr = c_out;
  e.P = (int)P;
  e.W2 = wd + 2;
  e.H2 = h + 2;
  const long long mt = (M + BM - 1) / BM;
  const bool can128 = K % gemm::Cfg<128>::BKS == 0;
  const int force = tile_n_override();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // tiles exactly as wide as the channels where a width divides them: no zero columns computed
  if (!force && c_out % 192 == 0)
    return launch_gemm_t<EpiConv, 192, ConvA>(tmA, w, K, (int)M, c_out, K, e, s, st, amap, c_in);
  if (!force && c_out == 96 && K % gemm::Cfg<96>::BKS == 0)
    return launch_gemm_t<EpiConv, 96, ConvA>(tmA, w, K, (int)M, c_out, K, e, s, st, amap, c_in);
  if (!force && c_out <= 64 && K % gemm::Cfg<64>::BKS == 0)
    return launch_gemm_t<EpiConv, 64, ConvA>(tmA, w, K, (int)M, c_out, K, e, s, st, amap, c_in);
  if (can128 && (force ? force == 128 : prefer_narrow_tiles(mt, c_out)))
    return launch_gemm_t<EpiConv, 128, ConvA>(tmA, w, K, (int)M, c_out, K, e, s, st, amap, c_in);
  return launch_gemm_t<EpiConv, 256, ConvA>(tmA, w, K, (int)M, c_out, K, e, s, st, amap, c_in);
}

int lbw_vae_conv_rms(const void* x, long long in_rows, int c_in, const void* w, const void* bias, int c_out, int kt,
                     int kh, int kw, int frames, int h, int wd, const float* gamma, int c_real, void* out, void* stream) {
  using namespace gemm;
  if (!x || !w || !out || !gamma) return set_error(LBW_ERR_INVALID, "lbw_vae_conv_rms: null pointer");
  if ((kt != 1 && kt != 3) || kh != kw || (kh != 1 && kh != 3))
    return set_error(LBW_ERR_SHAPE, "lbw_vae_conv_rms: kernel %dx%dx%d (kt 1 or 3, kh = kw 1 or 3)", kt, kh, kw);
  if (c_in <= 0 || c_in % 8 || c_out <= 0 || c_out % 32 || c_out > 256 || c_real <= 0 || c_real > c_out ||
      frames <= 0 || h <= 0 || wd <= 0)
    return set_error(LBW_ERR_SHAPE, "lbw_vae_conv_rms: channels %d -> %d (%d real; the row must fit one tile)", c_in,
                     c_out, c_real);
  const long long P = (long long)(h + 2) * (wd + 2);
  const long long M = (long long)frames * P;
  if (in_rows < (long long)(frames + kt - 1) * P || M > (1LL << 30) || in_rows > (1LL << 31) - 1)
    return set_error(LBW_ERR_SHAPE, "lbw_vae_conv_rms: %lld input rows for %d frames", in_rows, frames);
  if (!aligned(x, 16) || !aligned(w, 16) || !ok16(out) || !ok16(bias) || !aligned(gamma, 16))
    return set_error(LBW_ERR_ALIGN, "lbw_vae_conv_rms: alignment");
  int err = 0;
  int* st = device_status(&err);
  if (!st) return err;
  ConvA amap{};
  amap.cblocks = (c_in + 63) / 64;
  int t = 0;
  for (int a = 0; a < kt; ++a)
    for (int b = 0; b < kh; ++b)
      for (int c = 0; c < kw; ++c)
        amap.off[t++] = (int)(a * P + (b - kh / 2) * (long long)(wd + 2) + (c - kw / 2));
  const int K = t * amap.cblocks * 64;
  CUtensorMap tmA;
  if ((err = make_tmap_2d(&tmA, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, in_rows, c_in, c_in, BK, BM))) return err;
  EpiConvRms e{};
  e.out = reinterpret_cast<__nv_bfloat16*>(out);
  e.ldo = c_out;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.gamma = gamma;
  e.scale_c = sqrtf((float)c_real);
  e.P = (int)P;
  e.W2 = wd + 2;
  e.H2 = h + 2;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // one tile holds the whole row
  if (c_out == 192) return launch_gemm_t<EpiConvRms, 192, ConvA>(tmA, w, K, (int)M, c_out, K, e, s, st, amap, c_in);
  if (c_out == 96 && K % gemm::Cfg<96>::BKS == 0)
    return launch_gemm_t<EpiConvRms, 96, ConvA>(tmA, w, K, (int)M, c_out, K, e, s, st, amap, c_in);
  if (c_out <= 128 && K % gemm::Cfg<128>::BKS == 0)
    return launch_gemm_t<EpiConvRms, 128, ConvA>(tmA, w, K, (int)M, c_out, K, e, s, st, amap, c_in);
  return launch_gemm_t<EpiConvRms, 256, ConvA>(tmA, w, K, (int)M, c_out, K, e, s, st, amap, c_in);
}

int lbw_linear_act(const void* a, const void* w, const void* bias, const void* addend, int silu, int m, int n, int k,
                   void* out, void* stream) {
  if (!out) return set_error(LBW_ERR_INVALID, "lbw_linear_act: null output");
  if (!ok16(out) || !ok16(bias) || !ok16(addend) || n % 8) return set_error(LBW_ERR_ALIGN, "lbw_linear_act: alignment");
  EpiAct e{};
  e.out = reinterpret_cast<__nv_bfloat16*>(out);
  e.ldo = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  e.addend = reinterpret_cast<const __nv_bfloat16*>(addend);
  e.silu = silu;
  return launch_gemm(a, k, w, k, m, n, k, e, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ------------------------------------------------------------------------------------------
// Allocation-free variant of the linear + RMSNorm pair (lbw_linear_rowss followed by
// lbw_rmsnorm_rope without RoPE). Some hosts cannot hand this library a scratch buffer or let it
// call cudaMalloc: runtimes that reserve the whole device memory for their own pool up front (a
// serving engine sizing its KV cache to fill HBM) and plugins loaded by another framework that
// exposes no allocator to them. For those callers the row sums of squares, and the status word
// that records a timed-out wait of the GEMM, live in the fixed arrays below, which every GPU that
// loads the library keeps until the process exits.
// ------------------------------------------------------------------------------------------
namespace lbw {

constexpr int NOALLOC_MAX_ROWS = 65536;  // 256 KB of fp32 row sums per device
static __device__ __align__(256) float g_noalloc_rowss[NOALLOC_MAX_ROWS];
// Bounded-wait timeouts of the call's GEMM (LBW_DEV_TIMEOUT | site); read and cleared by lbw_check_device_status.
static __device__ int g_noalloc_status;

// y[row, :] = bf16(bf16(y * rsqrt(ss[row] / C + eps)) * gamma), in place (the same rounding points as
// rmsnorm_rope_kernel without the rotation). Each thread reads and rewrites its own 8 values. Nothing is
// written when the GEMM before it recorded a timeout (its output is incomplete).
__global__ void __launch_bounds__(128) rms_gamma_inplace_kernel(__nv_bfloat16* y, const float* ss,
                                                                const __nv_bfloat16* __restrict__ gamma, int C,
                                                                float eps, long long ldy, const int* status) {
  if (*(volatile const int*)status != 0) return;
  const long long row = blockIdx.x;
  const float r = 1.f / sqrtf(ss[row] / (float)C + eps);
  __nv_bfloat16* yr = y + row * ldy;
  for (int g = threadIdx.x; g < (C >> 3); g += 128) {
    uint4 xv = *reinterpret_cast<const uint4*>(yr + g * 8);
    uint4 gv = *reinterpret_cast<const uint4*>(gamma + g * 8);
    const __nv_bfloat16* xp = reinterpret_cast<const __nv_bfloat16*>(&xv);
    const __nv_bfloat16* gp = reinterpret_cast<const __nv_bfloat16*>(&gv);
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = bf16_round(bf16_round(__bfloat162float(xp[e]) * r) * __bfloat162float(gp[e]));
    *reinterpret_cast<uint4*>(yr + g * 8) =
        make_uint4(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]), pack_bf16(o[6], o[7]));
  }
}

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// Device addresses of the two arrays in the CUDA context current on this thread, looked up once per context
// (a module's globals have a different address in every context that loads it).
struct NoallocSlot {
  CUcontext ctx = nullptr;
  int dev = -1;
  float* rowss = nullptr;
  int* status = nullptr;
};
static std::mutex g_noalloc_mu;
static NoallocSlot g_noalloc_slots[64];

static CUcontext current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext c = nullptr;
  if (fn) fn(&c);
  return c;
}

static const NoallocSlot* noalloc_slot(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
    *err = set_error(LBW_ERR_CUDA, "lbw_linear_rmsnorm_noalloc: cudaGetDevice failed");
    return nullptr;
  }
  CUcontext ctx = current_context();
  if (!ctx) {  // no context on this thread yet: bind the device's primary context, as the runtime would
    if (cudaSetDevice(dev) != cudaSuccess || !(ctx = current_context())) {
      *err = set_error(LBW_ERR_CUDA, "lbw_linear_rmsnorm_noalloc: no CUDA context");
      return nullptr;
    }
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  for (auto& s : g_noalloc_slots)
    if (s.rowss && s.ctx == ctx && s.dev == dev) {
      *err = LBW_OK;
      return &s;
    }
  for (auto& s : g_noalloc_slots) {
    if (s.rowss) continue;
    void* pr = nullptr;
    void* ps = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&pr, g_noalloc_rowss);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&ps, g_noalloc_status);
    if (e != cudaSuccess || !pr || !ps) {
      *err = set_error(LBW_ERR_CUDA, "lbw_linear_rmsnorm_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
      return nullptr;
    }
    s.ctx = ctx;
    s.dev = dev;
    s.rowss = static_cast<float*>(pr);
    s.status = static_cast<int*>(ps);
    *err = LBW_OK;
    return &s;
  }
  *err = set_error(LBW_ERR_UNSUPPORTED, "lbw_linear_rmsnorm_noalloc: more than 64 device contexts");
  return nullptr;
}

// The allocation-free status word of the current device and context, or null when the entry point has not been
// used there (lbw_check_device_status reads it without looking anything up).
int* noalloc_status_peek() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  for (auto& s : g_noalloc_slots)
    if (s.rowss && s.ctx == ctx && s.dev == dev) return s.status;
  return nullptr;
}

}  // namespace lbw

extern "C" int lbw_linear_rmsnorm_noalloc(const void* a, const void* w, const void* bias, const void* gamma, int m,
                                          int n, int k, float eps, void* out, void* stream) {
  using namespace lbw;
  using namespace lbw::gemm;
  if (!a || !w || !gamma || !out) return set_error(LBW_ERR_INVALID, "lbw_linear_rmsnorm_noalloc: null pointer");
  if (m <= 0 || m > NOALLOC_MAX_ROWS)
    return set_error(LBW_ERR_SHAPE, "lbw_linear_rmsnorm_noalloc: %d rows; the built-in scratch holds at most %d rows",
                     m, NOALLOC_MAX_ROWS);
  if (n <= 0 || n % 32 || k <= 0 || k % BK)
    return set_error(LBW_ERR_SHAPE, "lbw_linear_rmsnorm_noalloc: N=%d must be a multiple of 32 and K=%d of %d", n, k, BK);
  if (!aligned(a, 16) || !aligned(w, 16) || !ok16(out) || !ok16(bias) || !ok16(gamma))
    return set_error(LBW_ERR_ALIGN, "lbw_linear_rmsnorm_noalloc: alignment");
  int err = 0;
  const NoallocSlot* slot = noalloc_slot(&err);
  if (!slot) return err;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The array keeps the previous call's sums: clear this call's rows first.
  if ((err = cuda_check(cudaMemsetAsync(slot->rowss, 0, sizeof(float) * (size_t)m, s), "noalloc scratch clear")))
    return err;
  CUtensorMap tmA;
  if ((err = make_tmap_2d(&tmA, a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, k, k, BK, BM))) return err;
  EpiStore e{};
  e.out[0] = e.out[1] = e.out[2] = reinterpret_cast<__nv_bfloat16*>(out);
  e.ld[0] = e.ld[1] = e.ld[2] = n;
  e.ss[0] = slot->rowss;
  e.region_cols = n;
  e.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  // the 256-wide tile launch of the allocating GEMMs (its shared-memory attribute is set once per device), with
  // the library's own status word replaced by the fixed one
  if ((err = launch_gemm_t<EpiStore, 256>(tmA, w, k, m, n, k, e, s, slot->status))) return err;
  rms_gamma_inplace_kernel<<<m, 128, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(out), slot->rowss,
                                             reinterpret_cast<const __nv_bfloat16*>(gamma), n, eps, n, slot->status);
  return cuda_check(cudaGetLastError(), "noalloc rms launch");
}
