// Chunk attention on tcgen05: softmax(scale * Q Kᵀ + bias) V over a list of KV-cache chunks.
//
// This is the exact (online-softmax) attention of the causal-fast block: the query chunk attends
// every key of the rolling window, which arrives as separate per-chunk cache tensors ordered
// (leading..., destination) -- wan/modules/chunked_kv_cache.py:47-76 and
// wan/modules/attention.py:1048-1058 (exact_attention_chunks -> SDPA over torch.cat of the
// chunks). There is no token mask: causality is what the cache holds (model_fast.py:2551-2568).
// With a per-key additive bias the same kernel is the deduplicated text cross-attention
// (attention.py:516-554).
//
// CTA = 2 query tiles x 128 rows of one head; head_dim 128; KV streamed 128 keys per tile.
//   warps 0-3 / 4-7  softmax of query tile 0 / 1 (thread = query row = TMEM lane)
//   warp 8           TMA producer: Q once, then K/V tiles through a 2-deep ring
//   warp 9           UMMA issuer, TMEM owner (512 columns: S0 | S1 | O0 | O1, 128 each)
//   warp 10          watches the K/V ring for the issuer: its arrivals fold "V(j) landed" into p_ready[0][0] and
//                    "K(j + 1) landed" into p_ready[0][1], so the issuing thread waits on four barriers per key
//                    tile instead of six (every shared-memory read of the issuing thread, an mbarrier test
//                    included, first waits for the MMAs it has issued to be taken by the tensor pipe)
// S_i = Q_i Kᵀ lands in TMEM; the softmax warps read it (tcgen05.ld), write bf16 P_i back over
// the first 64 columns of S_i (tcgen05.st, signalled per half tile so that P V on keys 0..63 starts
// while the exponentials of keys 64..127 are computed) and the MMA warp accumulates O_i += P_i V from TMEM
// (A operand) and shared memory (V, MN-major). The running max is only raised when a row's max
// grows by more than 2^8 (so P <= 256); O_i is then rescaled in TMEM by its own row's thread.
// Softmax is one tcgen05.ld pass per tile (the row's 128 scores stay in registers), packed fp32x2
// arithmetic, and a quarter of the exponentials on the FMA pipe (exp2_poly2) so that the SFU, whose
// rate is exactly one exp per 512 MMA flops, does not bound the loop.
// MMAs of one CTA execute in issue order, and every tcgen05.commit covers all earlier MMAs:
// when softmax i sees S_i(j+1) complete, PV_i(j) has completed too, so O_i is stable and P_i(j)
// has been consumed.
// Launch shapes (AttnSched): a grid of (query-tile pairs, heads, uniform KV splits), or the tail schedule the block
// uses -- whole windows in full waves of CTAs, then the windows of the last, partial wave cut into key ranges that
// fill the SMs it would leave idle, merged by attn_merge_tail_kernel.
#include <math.h>

#include "host_common.cuh"
#include "lbw_common.cuh"

namespace lbw {

#ifndef LBW_ATTN_POLY_EIGHTHS
#define LBW_ATTN_POLY_EIGHTHS 2  // eighths of the exponentials computed on the FMA pipe (exp2_poly2)
#endif

namespace attn {
constexpr int POLY = LBW_ATTN_POLY_EIGHTHS;
static_assert(POLY >= 0 && POLY <= 8, "LBW_ATTN_POLY_EIGHTHS must lie in [0, 8]");
constexpr int BM = 128, BN = 128, D = 128, QT = 2, STAGES = 2, MAX_CHUNKS = 8;
constexpr int HALF = 128 * 64 * 2;  // 128 rows x 64 bf16 (one 128-byte swizzled box)
constexpr int TILE = 2 * HALF;      // 128 rows x 128 bf16
constexpr int SMEM_BYTES = (QT + 2 * STAGES) * TILE + 1024;
constexpr int THREADS = 352;
}  // namespace attn

struct KVMaps {
  CUtensorMap k[attn::MAX_CHUNKS];
  CUtensorMap v[attn::MAX_CHUNKS];
  int rows[attn::MAX_CHUNKS];
  int n;
  int n_tiles;  // 128-key tiles over all chunks (each chunk's last tile may be ragged)
};

// Work schedule of one launch.
//   pieces == 0: grid (query-tile pairs, heads, KV splits); split z attends the key tiles [z n / Z, (z + 1) n / Z)
//                of its window and, when a workspace is given, writes slot slot0 + z of [slot][row][head][128].
//   pieces > 0:  1-D grid over windows w = head * qpairs + pair (a window is one head's pair of query tiles
//                against every key). Blocks [0, n_dp) attend whole windows and write the output. The last n_tail
//                windows (the final, partial wave of whole windows) are cut into `pieces` key ranges each: block
//                n_dp + p * n_tail + t attends range p of window n_dp + t and writes its unnormalised rows to
//                [p][t][256 rows][128] and (m, l) to [p][t][256][2], which attn_merge_tail_kernel combines. The
//                pieces run after every whole window has been dispatched and fill the SMs the last wave leaves.
struct AttnSched {
  int qpairs, heads, n_dp, n_tail, pieces;
};

// Combines split-KV partials: out = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s, M = max_s m_s.
// One warp per (row, head); each lane owns 4 of the 128 head dims.
__global__ void attn_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int n_slots,
                                  int q_rows, int heads, __nv_bfloat16* __restrict__ out, long long ldo) {
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (long long)q_rows * heads) return;
  const long long row = wid / heads;
  const int head = (int)(wid % heads);
  float M = -INFINITY;
  for (int s = 0; s < n_slots; ++s) M = fmaxf(M, part_ml[((s * (long long)q_rows + row) * heads + head) * 2]);
  float L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < n_slots; ++s) {
    const long long base = (s * (long long)q_rows + row) * heads + head;
    const float2 ml = *reinterpret_cast<const float2*>(part_ml + base * 2);
    const float w = (ml.x == -INFINITY) ? 0.f : exp2f(ml.x - M);
    L += w * ml.y;
    const float4 o = *reinterpret_cast<const float4*>(part_o + base * attn::D + lane * 4);
    acc[0] += w * o.x; acc[1] += w * o.y; acc[2] += w * o.z; acc[3] += w * o.w;
  }
  const float inv = 1.f / L;
  uint2 pk = make_uint2(pack_bf16(acc[0] * inv, acc[1] * inv), pack_bf16(acc[2] * inv, acc[3] * inv));
  *reinterpret_cast<uint2*>(out + row * ldo + (long long)head * attn::D + lane * 4) = pk;
}

// The same combination for the cut windows of a pieces > 0 schedule: one warp per (cut window, row).
__global__ void attn_merge_tail_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                       const AttnSched sc, int q_rows, __nv_bfloat16* __restrict__ out, long long ldo) {
  constexpr int WR = attn::QT * attn::BM;  // rows of a window
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (long long)sc.n_tail * WR) return;
  const int t = (int)(wid / WR), r = (int)(wid % WR);
  const int w = sc.n_dp + t;
  const int head = w / sc.qpairs;
  const long long row = (long long)(w % sc.qpairs) * WR + r;
  if (row >= q_rows) return;
  float M = -INFINITY;
  for (int p = 0; p < sc.pieces; ++p) M = fmaxf(M, part_ml[(((long long)p * sc.n_tail + t) * WR + r) * 2]);
  float L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int p = 0; p < sc.pieces; ++p) {
    const long long base = ((long long)p * sc.n_tail + t) * WR + r;
    const float2 ml = *reinterpret_cast<const float2*>(part_ml + base * 2);
    const float wgt = (ml.x == -INFINITY) ? 0.f : exp2f(ml.x - M);
    L += wgt * ml.y;
    const float4 o = *reinterpret_cast<const float4*>(part_o + base * attn::D + lane * 4);
    acc[0] += wgt * o.x; acc[1] += wgt * o.y; acc[2] += wgt * o.z; acc[3] += wgt * o.w;
  }
  const float inv = 1.f / L;
  uint2 pk = make_uint2(pack_bf16(acc[0] * inv, acc[1] * inv), pack_bf16(acc[2] * inv, acc[3] * inv));
  *reinterpret_cast<uint2*>(out + row * ldo + (long long)head * attn::D + lane * 4) = pk;
}

// Bounded wait until *flag has reached value (wrap-safe), for K/V rows that a stream memory operation on
// another stream announces once its copy engines have written them; then order the TMA loads that follow
// after the flag. The limit is in nanoseconds of the global timer (set by the host: a peer may legitimately be
// late by more than the mbarrier limit, and the exchange's own watchdog, which opens this gate when a peer is
// lost, acts after its timeout).
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool gate_wait(const unsigned int* flag, unsigned int value, long long limit_ns,
                                          const Abort& ab, int site) {
  const unsigned long long t0 = global_ns();
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if ((int)(v - value) >= 0) break;
    if (*ab.flag) return false;
    if ((long long)(global_ns() - t0) > limit_ns) {
      *ab.flag = 1;
      if (ab.status) atomicCAS(ab.status, 0, LBW_DEV_TIMEOUT | site);
      return false;
    }
    __nanosleep(256);
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

template <bool HAS_BIAS>
__global__ void __launch_bounds__(attn::THREADS, 1)
    chunk_attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ KVMaps kv, int q_rows,
                      float scale_log2, const float* __restrict__ key_bias, __nv_bfloat16* __restrict__ out,
                      long long ldo, float* __restrict__ part_o, float* __restrict__ part_ml, int slot0,
                      const AttnSched sc, const unsigned int* gate_flag, unsigned int gate_value, int gate_chunk,
                      long long gate_limit_ns, int* status) {
  using namespace attn;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + QT * TILE;
  uint8_t* sV = sK + STAGES * TILE;
  __shared__ __align__(8) uint64_t q_full, k_full[STAGES], k_empty[STAGES], v_full[STAGES], v_empty[STAGES],
      s_full[QT], p_ready[QT][2], o_done, done_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // This CTA attends its window's 128-key tiles [g_begin, g_end) (see AttnSched).
  int head, pair, g_begin, g_end;
  long long part_row0 = -1;  // pieces > 0: first workspace row of this block's partial; -1: write the output
  if (sc.pieces == 0) {
    pair = blockIdx.x;
    head = blockIdx.y;
    g_begin = (int)((long long)blockIdx.z * kv.n_tiles / gridDim.z);
    g_end = (int)((long long)(blockIdx.z + 1) * kv.n_tiles / gridDim.z);
  } else {
    int w = blockIdx.x;
    g_begin = 0;
    g_end = kv.n_tiles;
    if (w >= sc.n_dp) {
      const int t = (w - sc.n_dp) % sc.n_tail, p = (w - sc.n_dp) / sc.n_tail;
      w = sc.n_dp + t;
      g_begin = (int)((long long)p * kv.n_tiles / sc.pieces);
      g_end = (int)((long long)(p + 1) * kv.n_tiles / sc.pieces);
      part_row0 = ((long long)p * sc.n_tail + t) * (QT * BM);
    }
    head = w / sc.qpairs;
    pair = w % sc.qpairs;
  }
  const bool to_part = sc.pieces == 0 ? part_o != nullptr : part_row0 >= 0;
  const int q0 = pair * (QT * BM);
  const bool two = q0 + BM < q_rows;  // false when the block's second query tile lies past the last row

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < QT; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i][0], 128 + (i == 0));  // P of keys 0..63 written (+ V(j) landed, for tile 0)
      mbar_init(&p_ready[i][1], 128 + (i == 0));  // P of keys 64..127 written (+ K(j + 1) landed, for tile 0)
    }
    mbar_init(&o_done, 1);
    mbar_init(&done_bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) tmem_alloc(&tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const Abort ab{status, &abort_flag};
  const int n_chunks = kv.n;

  if (warp == 8) {
    // ---------------- producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      mbar_expect_tx(&q_full, QT * TILE);
      for (int i = 0; i < QT; ++i)
        for (int h = 0; h < 2; ++h)
          tma_load_2d(sQ + i * TILE + h * HALF, &tmQ, &q_full, head * D + h * 64, q0 + i * BM);
      int j = 0, g = 0;
      bool ok = true, gated = false;
      for (int c = 0; c < n_chunks && ok && g < g_end; ++c) {
        const int rows = kv.rows[c];
        for (int t0 = 0; t0 < rows && g < g_end; t0 += BN, ++g) {
          if (g < g_begin) continue;
          if (c >= gate_chunk && !gated) {  // chunks from gate_chunk on are still being filled by copy engines
            if (!gate_wait(gate_flag, gate_value, gate_limit_ns, ab, 0x23)) { ok = false; break; }
            gated = true;
          }
          const int s = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(&k_empty[s], ph ^ 1, ab, 0x21)) { ok = false; break; }
          mbar_expect_tx(&k_full[s], TILE);
          for (int h = 0; h < 2; ++h) tma_load_2d(sK + s * TILE + h * HALF, &kv.k[c], &k_full[s], head * D + h * 64, t0);
          if (!mbar_wait(&v_empty[s], ph ^ 1, ab, 0x22)) { ok = false; ++j; break; }
          mbar_expect_tx(&v_full[s], TILE);
          for (int h = 0; h < 2; ++h) tma_load_2d(sV + s * TILE + h * HALF, &kv.v[c], &v_full[s], head * D + h * 64, t0);
          ++j;
        }
      }
      // Let the last loads of each ring slot land before the CTA can exit.
      mbar_wait_drain(&q_full, 0);
      for (int i = (j > STAGES ? j - STAGES : 0); i < j; ++i) {
        mbar_wait_drain(&k_full[i & 1], (i >> 1) & 1);
        mbar_wait_drain(&v_full[i & 1], (i >> 1) & 1);
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16(BM, BN, 0, 0);  // S = Q Kᵀ: both K-major (head_dim contiguous)
      const uint32_t idesc_o = idesc_bf16(BM, D, 0, 1);   // O += P V: P from TMEM, V MN-major
      const int n_tiles = g_end - g_begin;

      // Descriptors are built once; a byte offset o inside shared memory moves the 14-bit start-address
      // field by o >> 4 (shared addresses stay below 2^18 bytes, so the field never carries). The issuing
      // thread is alone on its warp, so every instruction between two MMAs is latency the tensor pipe sees.
      const uint64_t dQ = sdesc_kmajor_sw128(smem_u32(sQ));
      const uint64_t dK = sdesc_kmajor_sw128(smem_u32(sK));
      const uint64_t dV = sdesc_mnmajor_sw128(smem_u32(sV), HALF);
      auto issue_s = [&](int i, int stage) {
        const uint64_t q = dQ + (uint64_t)((i * TILE) >> 4), k = dK + (uint64_t)((stage * TILE) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = (uint64_t)(((kk >> 2) * HALF + (kk & 3) * 32) >> 4);
          mma_f16_ss(tmem + i * 128, q + off, k + off, idesc_s, kk > 0);
        }
      };
      // O_i += P_i V over one half of the tile's keys (half 0: keys 0..63, half 1: keys 64..127)
      auto issue_pv = [&](int i, int stage, bool first, int half) {
        const uint64_t v = dV + (uint64_t)((stage * TILE) >> 4);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int kk = half * 4 + q;
          mma_f16_ts(tmem + 256 + i * 128, tmem + i * 128 + kk * 8, v + (uint64_t)((kk * 2048) >> 4), idesc_o,
                     !(first && kk == 0));
        }
      };

      bool ok = mbar_wait(&q_full, 0, ab, 0x31) && mbar_wait(&k_full[0], 0, ab, 0x32);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        tc_commit(&s_full[0]);
        if (two) {
          issue_s(1, 0);
          tc_commit(&s_full[1]);
        }
        tc_commit(&k_empty[0]);
        for (int j = 0; j < n_tiles && ok; ++j) {
          const int s = j & 1;
          const bool more = j + 1 < n_tiles;
          const int s1 = (j + 1) & 1;
          // p_ready[0][0] also means V(j) landed, p_ready[0][1] also K(j + 1) (the watcher's arrivals)
          if (!mbar_wait(&p_ready[0][0], j & 1, ab, 0x34)) { ok = false; break; }
          tc_fence_after();
          issue_pv(0, s, j == 0, 0);
          if (!mbar_wait(&p_ready[0][1], j & 1, ab, 0x37)) { ok = false; break; }
          tc_fence_after();
          issue_pv(0, s, j == 0, 1);
          if (more) {
            issue_s(0, s1);
            tc_commit(&s_full[0]);
          }
          if (two) {
            if (!mbar_wait(&p_ready[1][0], j & 1, ab, 0x36)) { ok = false; break; }
            tc_fence_after();
            issue_pv(1, s, j == 0, 0);
            if (!mbar_wait(&p_ready[1][1], j & 1, ab, 0x38)) { ok = false; break; }
            tc_fence_after();
            issue_pv(1, s, j == 0, 1);
          }
          tc_commit(&v_empty[s]);
          if (more) {
            if (two) {
              issue_s(1, s1);
              tc_commit(&s_full[1]);
            }
            tc_commit(&k_empty[s1]);
          }
        }
        if (ok) tc_commit(&o_done);
      }
      tc_commit(&done_bar);
      mbar_wait_drain(&done_bar, 0);
    }
  } else if (warp == 10) {
    // ---------------- K/V watcher ----------------
    // Observes every landing in order (K(0) first), so none of its parity waits runs a phase ahead, and waits for
    // each p_ready[0][h] phase to complete before arriving for the next key tile: an early arrival would count
    // toward the current phase and release P V before every softmax thread had written its part of P.
    if (lane == 0) {
      const int n_tiles = g_end - g_begin;
      bool ok = mbar_wait(&k_full[0], 0, ab, 0x60);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1, ab, 0x61)) break;
        mbar_arrive(&p_ready[0][0]);
        if (j + 1 < n_tiles && !mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, ab, 0x62)) break;
        mbar_arrive(&p_ready[0][1]);
        if (!mbar_wait(&p_ready[0][0], j & 1, ab, 0x63) || !mbar_wait(&p_ready[0][1], j & 1, ab, 0x64)) break;
      }
    }
  } else {
    // ---------------- softmax / correction / epilogue ----------------
    const int wg = warp >> 2;
    const int quarter = warp & 3;
    const bool active = wg == 0 || two;  // an all-padding second tile has no softmax to do
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + wg * 128;
    const uint32_t tO = tmem + lane_off + 256 + wg * 128;
    const float LOG2E = 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    int j = 0;
    bool ok = true;
    long long key_base = 0;
    int g = 0;
    for (int c = 0; c < n_chunks && ok && active && g < g_end; ++c) {
      const int rows = kv.rows[c];
      for (int t0 = 0; t0 < rows && g < g_end; t0 += BN, ++g) {
        if (g < g_begin) continue;
        const int valid = rows - t0 < BN ? rows - t0 : BN;
        if (!mbar_wait(&s_full[wg], j & 1, ab, 0x40 + wg)) { ok = false; break; }
        tc_fence_after();
        const float* kb = HAS_BIAS ? key_bias + key_base + t0 : nullptr;
        // One pass over S: all 128 scores of this row into registers (4 loads, one wait).
        uint32_t r[128];
        tmem_ld32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(&r[64]));
        tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(&r[96]));
        tmem_ld_wait();
        float* sv = reinterpret_cast<float*>(r);
        float a = scale_log2;  // p = exp2(a * s - m); with a key bias the scores are pre-scaled (a = 1)
        if (HAS_BIAS) {
#pragma unroll
          for (int e = 0; e < BN; ++e) sv[e] = sv[e] * scale_log2 + kb[e < valid ? e : 0] * LOG2E;
          a = 1.f;
        }
        if (valid < BN) {  // ragged last tile of a chunk (warp-uniform)
#pragma unroll
          for (int e = 0; e < BN; ++e)
            if (e >= valid) sv[e] = -INFINITY;
        }
        // row max: 8 independent chains of 3-input max
        float t8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t8[q] = sv[q];
#pragma unroll
        for (int e = 8; e < 120; e += 16)
#pragma unroll
          for (int q = 0; q < 8; ++q) t8[q] = fmax3(t8[q], sv[e + q], sv[e + 8 + q]);
#pragma unroll
        for (int q = 0; q < 8; ++q) t8[q] = fmaxf(t8[q], sv[120 + q]);
        const float mx = fmaxf(fmax3(t8[0], t8[1], t8[2]), fmax3(fmax3(t8[3], t8[4], t8[5]), t8[6], t8[7])) * a;
        const float m_new = fmaxf(m, mx);
        // The running max only moves when a row's max grew by more than 2^8; O is then rescaled by
        // alpha before PV(j) accumulates onto it (below, after P is written and the scores are dead,
        // but before p_ready releases PV(j)).
        float alpha = 1.f;
        bool rescale = false;
        if (j == 0) {
          m = m_new;
        } else {
          const bool need = m_new > m + 8.f;
          rescale = __any_sync(0xffffffffu, need);
          if (need) {
            alpha = fast_exp2(m - m_new);
            l *= alpha;
            m = m_new;
          }
        }
        // P = exp2(a*s - m): 3 of every 4 pairs on the SFU (ex2.approx), 1 on the FMA pipe (exp2_poly2),
        // which keeps the SFU from being the limit (one exp per 512 MMA flops is exactly its rate).
        // Scaling, subtraction and the row sum use packed fp32x2 instructions.
        const uint64_t a2 = f2_pack(a, a), b2 = f2_pack(-m, -m);
        uint64_t lsum[4] = {0ull, 0ull, 0ull, 0ull};
        if (valid == BN) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            if (cc == 2 && !rescale) {  // keys 0..63 are in TMEM: let P V start on them (warp-uniform branch)
              tmem_st_wait();
              tc_fence_before();
              mbar_arrive(&p_ready[wg][0]);
            }
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const int col = cc * 32 + e;
              float x0, x1, p0, p1;
              f2_unpack(f2_fma(f2_pack(sv[col], sv[col + 1]), a2, b2), x0, x1);
              if ((((e >> 1) * POLY) & 7) >= 8 - POLY) {  // spreads POLY of every 8 pairs evenly
                exp2_poly2(x0, x1, p0, p1);
              } else {
                p0 = fast_exp2(x0);
                p1 = fast_exp2(x1);
              }
              lsum[(e >> 1) & 3] = f2_add(lsum[(e >> 1) & 3], f2_pack(p0, p1));
              pk[e >> 1] = pack_bf16(p0, p1);
            }
            tmem_st16(tS + cc * 16, pk);
          }
        } else {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const int col = cc * 32 + e;
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(sv[col], sv[col + 1]), a2, b2), x0, x1);
              const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);  // masked scores are -inf -> 0
              lsum[(e >> 1) & 3] = f2_add(lsum[(e >> 1) & 3], f2_pack(p0, p1));
              pk[e >> 1] = pack_bf16(p0, p1);
            }
            tmem_st16(tS + cc * 16, pk);
          }
        }
        float l0, l1, l2, l3;
        f2_unpack(f2_add(lsum[0], lsum[1]), l0, l1);
        f2_unpack(f2_add(lsum[2], lsum[3]), l2, l3);
        l += (l0 + l1) + (l2 + l3);
        if (rescale) {  // warp-uniform
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t o[32];
            tmem_ld32(tO + cc * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + cc * 32, o);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        if (rescale || valid != BN) mbar_arrive(&p_ready[wg][0]);  // (O rescaled first, or ragged tile)
        mbar_arrive(&p_ready[wg][1]);
        ++j;
      }
      key_base += rows;
    }
    const int row = q0 + wg * BM + quarter * 32 + lane;
    if (!active) {
      // nothing to write: every row of this tile is past q_rows
    } else if (to_part && ok && mbar_wait(&o_done, 0, ab, 0x49)) {
      // split-KV partial: unnormalised O (fp32) and this row's (m, l), merged by attn_merge(_tail)_kernel
      tc_fence_after();
      const long long prow = sc.pieces == 0 ? ((slot0 + (long long)blockIdx.z) * q_rows + row) * sc.heads + head
                                            : part_row0 + wg * BM + quarter * 32 + lane;
      float* orow = part_o + prow * (long long)D;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t r[32];
        tmem_ld32(tO + cc * 32, r);
        tmem_ld_wait();
        if (row < q_rows) {
          float4* d4 = reinterpret_cast<float4*>(orow + cc * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            d4[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                                __uint_as_float(r[4 * q + 3]));
        }
      }
      if (row < q_rows) *reinterpret_cast<float2*>(part_ml + prow * 2) = make_float2(m, l);
    } else if (!to_part && ok && mbar_wait(&o_done, 0, ab, 0x48)) {
      tc_fence_after();
      const float inv = 1.f / l;
      __nv_bfloat16* orow = out + (long long)row * ldo + (long long)head * D;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t r[32];
        tmem_ld32(tO + cc * 32, r);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) pk[e >> 1] = pack_bf16(__uint_as_float(r[e]) * inv, __uint_as_float(r[e + 1]) * inv);
        if (row < q_rows) {
          uint4* d4 = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) d4[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, 512);
}

}  // namespace lbw

using namespace lbw;

// Limit of the gate wait: LBW_GATE_TIMEOUT_S seconds (default 120, more than the exchange watchdog's default
// 60 s, so that a lost peer is reported as PeerLost by the host rather than as a device timeout), read per call.
static long long gate_timeout_ns() {
  double s = 120.0;
  if (const char* e = getenv("LBW_GATE_TIMEOUT_S")) {
    const double v = atof(e);
    if (v > 0) s = v;
  }
  if (s > 3600.0) s = 3600.0;
  return (long long)(s * 1e9);
}

// Per-piece cost of a cut window in key-tile periods (the block's prologue and pipeline fill, its partial write and
// its share of the merge), used to choose the number of pieces: on B200 each further wave of pieces measured
// ~35 us, about 18 periods (c4 window, 1,350 and 2,700 query rows, 2 to 16 pieces).
#ifndef LBW_ATTN_PIECE_COST_TILES
#define LBW_ATTN_PIECE_COST_TILES 18
#endif

// Tail schedule of n_windows whole windows of n_tiles key tiles each on `sms` SMs: the windows past the last
// full wave are cut into `pieces` key ranges (0: the count that minimises the modelled time of the cut part,
// waves of pieces x (n_tiles / pieces + LBW_ATTN_PIECE_COST_TILES)). n_tail = 0 when nothing is cut.
static void tail_plan(long long n_windows, int n_tiles, int pieces, int sms, int* n_tail, int* pieces_out) {
  const long long tail = n_windows % sms;
  if (pieces == 0) {
    double best = 1e300;
    pieces = 1;
    for (int k = 1; k <= 16 && k <= n_tiles; ++k) {
      const double waves = (double)((tail * k + sms - 1) / sms);
      const double cost = waves * ((double)n_tiles / k + LBW_ATTN_PIECE_COST_TILES);
      if (cost < best - 1e-9) {
        best = cost;
        pieces = k;
      }
    }
  }
  if (tail == 0 || pieces <= 1) {
    *n_tail = 0;
    *pieces_out = 1;
    return;
  }
  *n_tail = (int)tail;
  *pieces_out = pieces;
}

static int launch_attention(const void* q, long long ldq, int q_rows, int heads, const void* const* k_chunks,
                            const void* const* v_chunks, const int* chunk_rows, int n_chunks, long long ldkv,
                            const float* key_bias, float softmax_scale, void* out, long long ldo, int n_splits,
                            float* part_o, float* part_ml, int slot0, const unsigned int* gate_flag,
                            unsigned int gate_value, int gate_chunk, cudaStream_t s, int pieces = -1,
                            long long ws_blocks = 0) {
  using namespace attn;
  if (!q || !k_chunks || !v_chunks || !chunk_rows) return set_error(LBW_ERR_INVALID, "chunk_attention: null pointer");
  if (!out && !part_o) return set_error(LBW_ERR_INVALID, "chunk_attention: null output");
  if (q_rows <= 0 || heads <= 0) return set_error(LBW_ERR_SHAPE, "chunk_attention: empty query");
  if (n_chunks < 1 || n_chunks > MAX_CHUNKS)
    return set_error(LBW_ERR_SHAPE, "chunk_attention: %d chunks (1..%d supported)", n_chunks, MAX_CHUNKS);
  if (ldq % 8 || ldkv % 8 || (out && (ldo % 8 || !aligned(out, 16))))
    return set_error(LBW_ERR_ALIGN, "chunk_attention: row strides must be multiples of 8 elements");
  if (ldq < (long long)heads * D || ldkv < (long long)heads * D || (out && ldo < (long long)heads * D))
    return set_error(LBW_ERR_SHAPE, "chunk_attention: row stride smaller than heads*128");
  if (key_bias && !aligned(key_bias, 4)) return set_error(LBW_ERR_ALIGN, "chunk_attention: key_bias alignment");
  if (part_o && (!part_ml || !aligned(part_o, 16) || !aligned(part_ml, 8) || slot0 < 0))
    return set_error(LBW_ERR_INVALID, "chunk_attention: partial buffers missing or misaligned");
  if (!part_o && n_splits != 1 && pieces < 0)
    return set_error(LBW_ERR_INVALID, "chunk_attention: KV splits need partial buffers");
  if (pieces >= 0 && (!out || n_splits != 1 || slot0 != 0))
    return set_error(LBW_ERR_INVALID, "chunk_attention: a tail schedule writes out (one split, slot 0)");
  if (gate_chunk < n_chunks && (!gate_flag || !aligned(gate_flag, 4)))
    return set_error(LBW_ERR_INVALID, "chunk_attention: gated chunks need a 4-byte aligned gate flag");
  if (gate_chunk < 0) gate_chunk = 0;
  int err = 0;
  int* st = device_status(&err);
  if (!st) return err;
  CUtensorMap tmQ;
  KVMaps kv;
  memset(&kv, 0, sizeof(kv));
  const uint64_t cols = (uint64_t)heads * D;
  if ((err = make_tmap_2d(&tmQ, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q_rows, cols, ldq, 64, BM))) return err;
  int n_tiles = 0;
  for (int c = 0; c < n_chunks; ++c) {
    if (chunk_rows[c] <= 0) return set_error(LBW_ERR_SHAPE, "chunk_attention: chunk %d is empty", c);
    if (!k_chunks[c] || !v_chunks[c]) return set_error(LBW_ERR_INVALID, "chunk_attention: null chunk %d", c);
    if ((err = make_tmap_2d(&kv.k[c], k_chunks[c], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, chunk_rows[c], cols, ldkv, 64, BN)))
      return err;
    if ((err = make_tmap_2d(&kv.v[c], v_chunks[c], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, chunk_rows[c], cols, ldkv, 64, BN)))
      return err;
    kv.rows[c] = chunk_rows[c];
    n_tiles += (chunk_rows[c] + BN - 1) / BN;
  }
  kv.n = n_chunks;
  kv.n_tiles = n_tiles;
  if (n_splits < 1 || n_splits > n_tiles)
    return set_error(LBW_ERR_SHAPE, "chunk_attention: %d KV splits for %d key tiles", n_splits, n_tiles);
  AttnSched sc{(q_rows + QT * BM - 1) / (QT * BM), heads, 0, 0, 0};
  dim3 grid(sc.qpairs, heads, n_splits);
  if (pieces >= 0) {
    if (pieces > n_tiles)
      return set_error(LBW_ERR_SHAPE, "chunk_attention: %d pieces for %d key tiles", pieces, n_tiles);
    const long long n_windows = (long long)sc.qpairs * heads;
    tail_plan(n_windows, n_tiles, pieces, num_sms(), &sc.n_tail, &sc.pieces);
    sc.n_dp = (int)(n_windows - sc.n_tail);
    if (sc.n_tail > 0 && (!part_o || !part_ml || !aligned(part_o, 16) || !aligned(part_ml, 8) ||
                          ws_blocks < (long long)sc.n_tail * sc.pieces))
      return set_error(LBW_ERR_INVALID, "chunk_attention: the tail schedule needs %lld workspace blocks (%lld given)",
                       (long long)sc.n_tail * sc.pieces, ws_blocks);
    grid = dim3((unsigned)(sc.n_dp + (long long)sc.n_tail * sc.pieces));
  }
  static bool attr[64][2] = {};  // per device and variant
  const int hb = key_bias ? 1 : 0;
  const int dix = device_index();
  if (dix < 0) return set_error(LBW_ERR_CUDA, "chunk_attention: cudaGetDevice failed");
  if (!attr[dix][hb]) {
    err = cuda_check(cudaFuncSetAttribute(hb ? chunk_attn_kernel<true> : chunk_attn_kernel<false>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES),
                     "attention smem attribute");
    if (err) return err;
    attr[dix][hb] = true;
  }
  const float scale_log2 = softmax_scale * 1.4426950408889634f;
  const long long gate_ns = gate_chunk < n_chunks ? gate_timeout_ns() : 0;
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
  if (hb)
    chunk_attn_kernel<true><<<grid, THREADS, SMEM_BYTES, s>>>(tmQ, kv, q_rows, scale_log2, key_bias, o, ldo, part_o,
                                                              part_ml, slot0, sc, gate_flag, gate_value, gate_chunk,
                                                              gate_ns, st);
  else
    chunk_attn_kernel<false><<<grid, THREADS, SMEM_BYTES, s>>>(tmQ, kv, q_rows, scale_log2, nullptr, o, ldo, part_o,
                                                               part_ml, slot0, sc, gate_flag, gate_value, gate_chunk,
                                                               gate_ns, st);
  if ((err = cuda_check(cudaGetLastError(), "attention launch"))) return err;
  if (sc.n_tail > 0) {
    const long long threads = (long long)sc.n_tail * QT * BM * 32;
    attn_merge_tail_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(part_o, part_ml, sc, q_rows, o, ldo);
    err = cuda_check(cudaGetLastError(), "attention tail merge launch");
  }
  return err;
}

extern "C" {

int lbw_chunk_attention(const void* q, long long ldq, int q_rows, int heads, const void* const* k_chunks,
                        const void* const* v_chunks, const int* chunk_rows, int n_chunks, long long ldkv,
                        const float* key_bias, float softmax_scale, void* out, long long ldo, void* stream) {
  if (!out) return set_error(LBW_ERR_INVALID, "chunk_attention: null output");
  return launch_attention(q, ldq, q_rows, heads, k_chunks, v_chunks, chunk_rows, n_chunks, ldkv, key_bias,
                          softmax_scale, out, ldo, 1, nullptr, nullptr, 0, nullptr, 0, n_chunks,
                          reinterpret_cast<cudaStream_t>(stream));
}

int lbw_chunk_attention_partial(const void* q, long long ldq, int q_rows, int heads, const void* const* k_chunks,
                                const void* const* v_chunks, const int* chunk_rows, int n_chunks, long long ldkv,
                                const float* key_bias, float softmax_scale, int n_splits, float* part_o,
                                float* part_ml, int slot0, void* stream) {
  if (!part_o || !part_ml) return set_error(LBW_ERR_INVALID, "chunk_attention_partial: null workspace");
  return launch_attention(q, ldq, q_rows, heads, k_chunks, v_chunks, chunk_rows, n_chunks, ldkv, key_bias,
                          softmax_scale, nullptr, 0, n_splits, part_o, part_ml, slot0, nullptr, 0, n_chunks,
                          reinterpret_cast<cudaStream_t>(stream));
}

int lbw_chunk_attention_gated(const void* q, long long ldq, int q_rows, int heads, const void* const* k_chunks,
                              const void* const* v_chunks, const int* chunk_rows, int n_chunks, long long ldkv,
                              float softmax_scale, void* out, long long ldo, int n_splits, float* part_o,
                              float* part_ml, int slot0, const unsigned int* gate_flag, unsigned int gate_value,
                              int gate_chunk, void* stream) {
  if (gate_chunk < 0 || gate_chunk >= n_chunks)
    return set_error(LBW_ERR_SHAPE, "chunk_attention_gated: gate chunk %d of %d", gate_chunk, n_chunks);
  if (!out && !part_o) return set_error(LBW_ERR_INVALID, "chunk_attention_gated: null output");
  if (out && part_o) return set_error(LBW_ERR_INVALID, "chunk_attention_gated: give out or the partial buffers");
  return launch_attention(q, ldq, q_rows, heads, k_chunks, v_chunks, chunk_rows, n_chunks, ldkv, nullptr,
                          softmax_scale, out, ldo, n_splits, part_o, part_ml, slot0, gate_flag, gate_value, gate_chunk,
                          reinterpret_cast<cudaStream_t>(stream));
}

int lbw_attention_tail_plan(int q_rows, int heads, const int* chunk_rows, int n_chunks, int pieces, int* n_tail,
                            int* pieces_used) {
  using namespace attn;
  if (!chunk_rows || !n_tail || !pieces_used) return set_error(LBW_ERR_INVALID, "attention_tail_plan: null pointer");
  if (q_rows <= 0 || heads <= 0 || n_chunks < 1 || n_chunks > MAX_CHUNKS || pieces < 0)
    return set_error(LBW_ERR_SHAPE, "attention_tail_plan: bad shape");
  int n_tiles = 0;
  for (int c = 0; c < n_chunks; ++c) {
    if (chunk_rows[c] <= 0) return set_error(LBW_ERR_SHAPE, "attention_tail_plan: chunk %d is empty", c);
    n_tiles += (chunk_rows[c] + BN - 1) / BN;
  }
  if (pieces > n_tiles) return set_error(LBW_ERR_SHAPE, "attention_tail_plan: %d pieces for %d key tiles", pieces, n_tiles);
  const long long n_windows = (long long)((q_rows + QT * BM - 1) / (QT * BM)) * heads;
  tail_plan(n_windows, n_tiles, pieces, num_sms(), n_tail, pieces_used);
  return LBW_OK;
}

int lbw_chunk_attention_tail(const void* q, long long ldq, int q_rows, int heads, const void* const* k_chunks,
                             const void* const* v_chunks, const int* chunk_rows, int n_chunks, long long ldkv,
                             const float* key_bias, float softmax_scale, void* out, long long ldo, int pieces,
                             float* part_o, float* part_ml, long long ws_blocks, const unsigned int* gate_flag,
                             unsigned int gate_value, int gate_chunk, void* stream) {
  if (!out) return set_error(LBW_ERR_INVALID, "chunk_attention_tail: null output");
  if (pieces < 0) return set_error(LBW_ERR_SHAPE, "chunk_attention_tail: pieces %d", pieces);
  if (gate_chunk < 0 || gate_chunk > n_chunks)
    return set_error(LBW_ERR_SHAPE, "chunk_attention_tail: gate chunk %d of %d", gate_chunk, n_chunks);
  if (gate_chunk < n_chunks && key_bias)
    return set_error(LBW_ERR_INVALID, "chunk_attention_tail: a gated launch takes no key bias");
  return launch_attention(q, ldq, q_rows, heads, k_chunks, v_chunks, chunk_rows, n_chunks, ldkv, key_bias,
                          softmax_scale, out, ldo, 1, part_o, part_ml, 0, gate_flag, gate_value, gate_chunk,
                          reinterpret_cast<cudaStream_t>(stream), pieces, ws_blocks);
}

int lbw_attention_merge(const float* part_o, const float* part_ml, int n_slots, int q_rows, int heads, void* out,
                        long long ldo, void* stream) {
  using namespace attn;
  if (!part_o || !part_ml || !out) return set_error(LBW_ERR_INVALID, "attention_merge: null pointer");
  if (n_slots < 1 || q_rows <= 0 || heads <= 0) return set_error(LBW_ERR_SHAPE, "attention_merge: empty");
  if (ldo % 8 || ldo < (long long)heads * D || !aligned(out, 16) || !aligned(part_o, 16) || !aligned(part_ml, 8))
    return set_error(LBW_ERR_ALIGN, "attention_merge: alignment");
  const long long threads = (long long)q_rows * heads * 32;
  attn_merge_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      part_o, part_ml, n_slots, q_rows, heads, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return cuda_check(cudaGetLastError(), "attention_merge launch");
}

}  // extern "C"
