// Host-side helpers shared by the C-ABI entry points: status/error reporting, the per-device
// status word, TMA tensor-map encoding and launch configuration.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "../../include/lbw.h"

namespace lbw {

// Records `code` and a formatted message as this thread's last error; returns `code`.
int set_error(int code, const char* fmt, ...);

// Device status word of the current device (zeroed on first use). Kernels that wait on
// mbarriers record timeouts there; lbw_check_device_status() reads and clears it.
int* device_status(int* err);
// The status word of the current device if device_status() has created it, else null (allocates nothing).
int* device_status_peek();
// The status word of lbw_linear_rmsnorm_noalloc in the current device and context, or null when that entry
// point has not run there.
int* noalloc_status_peek();
// Creates the current device's peer pull streams and events now (lbw_init); they are otherwise made on the first
// exchange.
int pull_streams_init();
// Destroys device `dev`'s pull streams and events (lbw_destroy); the next exchange creates them again.
void pull_streams_release(int dev);

// cudaError_t -> LBW_ERR_CUDA with the CUDA error string.
inline int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LBW_OK;
  return set_error(LBW_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Encodes a 2-D row-major tensor map: `rows` x `cols` elements of `elem_bytes` each, row pitch
// `row_stride_elems`, box `box_cols` x `box_rows`, 128-byte swizzle (box_cols * elem_bytes
// must be 128). Out-of-bounds rows of a box are zero-filled by the TMA unit.
int make_tmap_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows);

int num_sms();
// Row blocks (of 128) per tile group of the persistent GEMMs (see tile_coords): about 40 MB of activation rows
// (K elements of elem_bytes each) so that a group stays in the 126 MB L2 with the weights streaming past.
inline int group_rows(int M, int K, int elem_bytes) {
  const long long per = 128LL * K * elem_bytes;
  long long g = (40LL << 20) / (per > 0 ? per : 1);
  const long long nm = (M + 127) / 128;
  if (g < 1) g = 1;
  if (g > nm) g = nm;
  return (int)g;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Tile width of the persistent GEMMs (128 x TBN tiles, one CTA per SM walking its share of them): the time is
// set by the most tiles any CTA runs, and a 128-wide tile costs ~0.6 of a 256-wide one (B200, the block's bf16
// and MXFP8 GEMMs at 1,350 / 2,700 / 10,800 rows: 0.58-0.63), so 128 wins when 0.6 x its per-CTA tile count
// stays below 256's.
inline bool prefer_narrow_tiles(long long m_tiles, long long n) {
  const long long sms = num_sms();
  const long long w256 = (m_tiles * ((n + 255) / 256) + sms - 1) / sms;
  const long long w128 = (m_tiles * ((n + 127) / 128) + sms - 1) / sms;
  return 3 * w128 < 5 * w256;
}

// Index of the current device for per-device caches (function attributes such as a kernel's dynamic shared
// memory limit belong to one device's context), or -1.
inline int device_index() {
  int d = 0;
  return (cudaGetDevice(&d) == cudaSuccess && d >= 0 && d < 64) ? d : -1;
}

// Tile-width override of the persistent GEMMs for tuning sweeps: LBW_GEMM_TILE_N=128 or 256 forces that width
// where the shape allows it; unset (or any other value) keeps the automatic choice.
inline int tile_n_override() {
  const char* s = getenv("LBW_GEMM_TILE_N");
  if (!s) return 0;
  const int v = atoi(s);
  return (v == 128 || v == 256) ? v : 0;
}

}  // namespace lbw
