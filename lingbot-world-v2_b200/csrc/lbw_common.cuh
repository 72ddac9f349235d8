// Device-side building blocks shared by every sm_100a kernel of the block forward:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (UMMA) issue, TMEM alloc/load/store
// and the shared-memory matrix descriptors the tensor core reads.
//
// Every wait on an mbarrier is bounded by LBW_WAIT_CYCLES SM clocks. A wait that runs out
// records LBW_ERR_TIMEOUT (plus a site code) in the device status word passed to the kernel,
// raises the CTA-wide abort flag and returns false; the caller then leaves its loop, so a
// pipeline bug shows up as an error status on the host instead of a hung GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#define LBW_DEV __device__ __forceinline__

// ~1.1 s at the B200's 1965 MHz boost clock.
#ifndef LBW_WAIT_CYCLES
#define LBW_WAIT_CYCLES (1ll << 31)
#endif

// Device status codes (the host maps them to lbw_status values; see lbw.h).
#define LBW_DEV_OK 0
#define LBW_DEV_TIMEOUT 0x100  // | site

namespace lbw {

LBW_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
LBW_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
LBW_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
LBW_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
LBW_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
LBW_DEV bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// CTA-wide error state: a pointer to the device status word and a shared abort flag.
struct Abort {
  int* status;            // global, may be null
  volatile int* flag;     // shared
};

// Wait until phase `parity` of `bar` has completed. Bounded: returns false on timeout or when
// another thread of the CTA already aborted.
LBW_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, const Abort& ab, int site) {
  uint32_t a = smem_u32(bar);
  if (mbar_test(a, parity)) return true;
  long long t0 = clock64();
  while (true) {
    if (mbar_test(a, parity)) return true;
    if (*ab.flag) return false;
    if (clock64() - t0 > LBW_WAIT_CYCLES) {
      *ab.flag = 1;
      if (ab.status) atomicCAS(ab.status, 0, LBW_DEV_TIMEOUT | site);
      return false;
    }
  }
}

// Bounded wait that ignores the abort flag and records nothing: used on the way out of a kernel
// so that copies and MMAs already in flight land before shared memory and TMEM are released.
LBW_DEV bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  uint32_t a = smem_u32(bar);
  long long t0 = clock64();
  while (!mbar_test(a, parity)) {
    if (clock64() - t0 > LBW_WAIT_CYCLES) return false;
  }
  return true;
}

// Persistent GEMM tile order: tile t of an nM x nN grid of output tiles, walked in groups of gm row blocks
// with the row block varying fastest inside a group. The tiles in flight then share a few weight column
// blocks, and the group's activation rows stay in L2 while the weights stream past once per group (a plain
// row-major walk re-reads every weight block from DRAM on every wave once the weights exceed L2).
LBW_DEV void tile_coords(int t, int nM, int nN, int gm, int& m, int& n) {
  const int per = gm * nN;
  const int grp = t / per;
  const int m0 = grp * gm;
  const int rows = nM - m0 < gm ? nM - m0 : gm;
  const int loc = t - grp * per;
  m = m0 + loc % rows;
  n = loc / rows;
}

// ------------------------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ------------------------------------------------------------------------------------------
LBW_DEV void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
LBW_DEV void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// Plain bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
LBW_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA issue, commit, TMEM <-> registers
// ------------------------------------------------------------------------------------------
LBW_DEV void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
LBW_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
LBW_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LBW_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on `bar` once every tcgen05 op issued so far by this thread has completed.
LBW_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (bf16 inputs, fp32 accumulate).
LBW_DEV void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem desc), kind::f16.
LBW_DEV void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D(tmem) (+)= (A * SFA) * (B * SFB), kind::mxf8f6f4 with E8M0 scales in TMEM (one per 32 K).
LBW_DEV void mma_mxf8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate,
                         uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// D(tmem) (+)= (A * SFA) * (B * SFB), kind::mxf4 (E2M1 pairs per byte) with E8M0 scales, two per MMA (K = 64).
LBW_DEV void mma_mxf4_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate,
                         uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// Shared memory (32 rows x 16 bytes) -> TMEM, broadcast to the four 32-lane quarters.
LBW_DEV void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

#define LBW_R4(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3])
// 32 lanes x 32 columns of 32 bit: thread t of the warp gets lane (warp%4)*32+t, columns c..c+31.
LBW_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : LBW_R4(0), LBW_R4(4), LBW_R4(8), LBW_R4(12), LBW_R4(16), LBW_R4(20), LBW_R4(24), LBW_R4(28)
      : "r"(taddr));
}
LBW_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : LBW_R4(0), LBW_R4(4), LBW_R4(8), LBW_R4(12)
      : "r"(taddr));
}
#undef LBW_R4
#define LBW_W4(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3])
LBW_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      LBW_W4(0), LBW_W4(4), LBW_W4(8), LBW_W4(12)
      : "memory");
}
LBW_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      LBW_W4(0), LBW_W4(4), LBW_W4(8), LBW_W4(12), LBW_W4(16), LBW_W4(20), LBW_W4(24), LBW_W4(28)
      : "memory");
}
#undef LBW_W4
LBW_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
LBW_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------------------------------
// Shared-memory matrix descriptors (tcgen05 "version 1" format)
//   bits [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1, [61,64) layout (2 = 128-byte swizzle).
// ------------------------------------------------------------------------------------------
LBW_DEV uint64_t sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(layout & 7) << 61;
  return d;
}
// K-major operand tile written by TMA with 128-byte swizzle: rows of 128 bytes, 8-row groups
// 1024 bytes apart. Advancing along K inside the 128-byte row = adding bytes to the start.
LBW_DEV uint64_t sdesc_kmajor_sw128(uint32_t saddr) { return sdesc(saddr, 16, 1024, 2); }
// MN-major operand, 128-byte swizzle: each K row holds 64 16-bit MN elements (128 bytes),
// 8-row K groups 1024 bytes apart, consecutive 64-element MN blocks `mn_block_bytes` apart.
LBW_DEV uint64_t sdesc_mnmajor_sw128(uint32_t saddr, uint32_t mn_block_bytes) {
  return sdesc(saddr, mn_block_bytes, 1024, 2);
}
// Scale-factor staging for tcgen05.cp (no swizzle; 8 rows x 16 bytes per core matrix).
LBW_DEV uint64_t sdesc_sf(uint32_t saddr) { return sdesc(saddr, 0, 128, 0); }

// Instruction descriptor, kind::f16: bf16 x bf16 -> fp32, M x N, A/B major-ness.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                      // D format f32
         | (1u << 7)                    // A bf16
         | (1u << 10)                   // B bf16
         | ((uint32_t)a_mn_major << 15) // A major
         | ((uint32_t)b_mn_major << 16) // B major
         | ((uint32_t)(N >> 3) << 17)   // N
         | ((uint32_t)(M >> 4) << 24);  // M
}
// Instruction descriptor, kind::mxf8f6f4 block-scaled: both operands E4M3 (fmt 0) or both E5M2 (fmt 1) with UE8M0
// scales, K-major operands; sf_id selects the byte of the 32-bit TMEM scale column.
__host__ __device__ constexpr uint32_t idesc_mxf8(int M, int N, uint32_t sf_id, uint32_t fmt = 0) {
  return (sf_id << 4)                  // B scale-factor id
         | (fmt << 7) | (fmt << 10)    // A, B element format (0 = E4M3, 1 = E5M2)
         | ((uint32_t)(N >> 3) << 17)  // N
         | (1u << 23)                  // scale format UE8M0
         | ((uint32_t)(M >> 4) << 24)  // M
         | (sf_id << 29);              // A scale-factor id
}
// Instruction descriptor, kind::mxf4 block-scaled (E2M1 x E2M1, packed two per byte, one UE8M0 scale per 32
// elements, K = 64 per MMA): sf_id is the first of the two consecutive scale bytes the MMA reads (0 or 2).
__host__ __device__ constexpr uint32_t idesc_mxf4(int M, int N, uint32_t sf_id) {
  return (sf_id << 4)                  // B scale-factor id
         | (1u << 7) | (1u << 10)      // A, B element format E2M1 (the kind::mxf4 encoding)
         | ((uint32_t)(N >> 3) << 17)  // N
         | (1u << 23)                  // scale format UE8M0
         | ((uint32_t)(M >> 4) << 24)  // M
         | (sf_id << 29);              // A scale-factor id; bit 31 = 0: K = 64
}

// ------------------------------------------------------------------------------------------
// small numeric helpers
// ------------------------------------------------------------------------------------------
LBW_DEV uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
LBW_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
LBW_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Packed fp32x2 arithmetic (one instruction for the two lanes of a register pair) and 3-input max.
LBW_DEV uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
LBW_DEV void f2_unpack(uint64_t v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
LBW_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
LBW_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
LBW_DEV float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// Two 2^x on the FMA/ALU pipes (x finite; results below 2^-126 are flushed up to 2^-126).
// Cody-Waite style range reduction x = n + f with n = round(x) (adding 1.5 * 2^23 leaves n in the
// low mantissa bits) and f in [-0.5, 0.5]; 2^f by a cubic whose coefficients were fitted for this
// library by relative-error least squares on [-0.5, 0.5] (max relative error 1.8e-4, below the 2^-9
// rounding of a bf16 result); the result's exponent field is then raised by n.
LBW_DEV void exp2_poly2(float x0, float x1, float& y0, float& y1) {
  const uint64_t x = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t t = f2_add(x, f2_pack(12582912.f, 12582912.f));
  const uint64_t n = f2_add(t, f2_pack(-12582912.f, -12582912.f));  // round(x), exact
  const uint64_t f = f2_fma(n, f2_pack(-1.f, -1.f), x);             // x - round(x), exact
  uint64_t p = f2_fma(f2_pack(0.054602623f, 0.054602623f), f, f2_pack(0.24192412f, 0.24192412f));
  p = f2_fma(p, f, f2_pack(0.69331646f, 0.69331646f));
  p = f2_fma(p, f, f2_pack(1.f, 1.f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  y0 = __int_as_float(__float_as_int(p0) + ((__float_as_int(t0) - 0x4B400000) << 23));
  y1 = __int_as_float(__float_as_int(p1) + ((__float_as_int(t1) - 0x4B400000) << 23));
}

}  // namespace lbw
