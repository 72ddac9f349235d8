// Library-wide C-ABI plumbing: version, last-error string, device status word, tensor maps.
#include <stdarg.h>
#include <string.h>

#include <mutex>

#include "host_common.cuh"

namespace lbw {

static thread_local char g_last_error[1024] = {0};

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

static std::mutex g_mu;
static int* g_status[64] = {nullptr};

int* device_status(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = set_error(LBW_ERR_CUDA, "cudaGetDevice failed");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, 64) != cudaSuccess || cudaMemset(p, 0, 64) != cudaSuccess) {
      *err = set_error(LBW_ERR_CUDA, "status word allocation failed");
      return nullptr;
    }
    g_status[dev] = p;
  }
  *err = LBW_OK;
  return g_status[dev];
}

int* device_status_peek() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  return g_status[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(LBW_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (!aligned(base, 16)) return set_error(LBW_ERR_ALIGN, "TMA base address not 16-byte aligned");
  if ((row_stride_elems * elem_bytes) % 16 != 0) return set_error(LBW_ERR_ALIGN, "TMA row pitch not a multiple of 16 bytes");
  if (box_cols * elem_bytes != 128) return set_error(LBW_ERR_INVALID, "TMA box inner extent must be 128 bytes");
  if (rows == 0 || cols == 0) return set_error(LBW_ERR_SHAPE, "empty TMA tensor");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * (cuuint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(LBW_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LBW_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

}  // namespace lbw

extern "C" {

int lbw_version(void) { return LBW_VERSION; }

int lbw_last_error(char* buf, size_t n) {
  if (!buf || n == 0) return LBW_ERR_INVALID;
  strncpy(buf, lbw::g_last_error, n - 1);
  buf[n - 1] = 0;
  return LBW_OK;
}

const char* lbw_status_string(int code) {
  switch (code) {
    case LBW_OK: return "ok";
    case LBW_ERR_INVALID: return "invalid argument";
    case LBW_ERR_SHAPE: return "unsupported shape";
    case LBW_ERR_ALIGN: return "misaligned pointer or stride";
    case LBW_ERR_CUDA: return "CUDA error";
    case LBW_ERR_TIMEOUT: return "device wait timed out";
    case LBW_ERR_UNSUPPORTED: return "unsupported configuration";
    default: return "unknown status";
  }
}

// The per-device state is keyed by device ordinal and is made on first use; lbw_init / lbw_destroy create and
// release it at a time the caller picks. Both switch to `device` for the call and then make the caller's
// context current again (cudaSetDevice alone would leave the device's primary context current, which is not
// the caller's when it runs in a context of its own).
typedef CUresult (*CtxGetFn)(CUcontext*);
typedef CUresult (*CtxSetFn)(CUcontext);

static void* driver_entry(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return p;
}

struct DeviceScope {
  CUcontext prev = nullptr;
  CtxSetFn set = nullptr;
  int err = LBW_OK;
  explicit DeviceScope(int device, const char* who) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
      err = lbw::set_error(LBW_ERR_CUDA, "%s: cudaGetDeviceCount failed", who);
      return;
    }
    if (device < 0 || device >= n || device >= 64) {
      err = lbw::set_error(LBW_ERR_INVALID, "%s: device %d out of range (%d devices)", who, device, n);
      return;
    }
    auto get = reinterpret_cast<CtxGetFn>(driver_entry("cuCtxGetCurrent"));
    set = reinterpret_cast<CtxSetFn>(driver_entry("cuCtxSetCurrent"));
    if (!get || !set || get(&prev) != CUDA_SUCCESS) {
      err = lbw::set_error(LBW_ERR_CUDA, "%s: driver context entry points unavailable", who);
      return;
    }
    err = lbw::cuda_check(cudaSetDevice(device), "cudaSetDevice");
  }
  ~DeviceScope() {
    if (set && prev) set(prev);
  }
};

int lbw_init(int device) {
  DeviceScope scope(device, "lbw_init");
  if (scope.err) return scope.err;
  int err = LBW_OK;
  lbw::device_status(&err);
  if (err) return err;
  return lbw::pull_streams_init();
}

int lbw_destroy(int device) {
  DeviceScope scope(device, "lbw_destroy");
  if (scope.err) return scope.err;
  int err = lbw::cuda_check(cudaDeviceSynchronize(), "lbw_destroy: device synchronize");
  {
    std::lock_guard<std::mutex> lk(lbw::g_mu);
    if (lbw::g_status[device]) {
      const int e = lbw::cuda_check(cudaFree(lbw::g_status[device]), "lbw_destroy: status word free");
      if (!err) err = e;
      lbw::g_status[device] = nullptr;
    }
  }
  lbw::pull_streams_release(device);
  return err;
}

int lbw_check_device_status(void* stream, int* device_code) {
  // Reads the library's status word and the allocation-free entry point's one; allocates neither.
  int* words[2] = {lbw::device_status_peek(), lbw::noalloc_status_peek()};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int v[2] = {0, 0};
  for (int i = 0; i < 2; ++i) {
    if (!words[i]) continue;
    int rc = lbw::cuda_check(cudaMemcpyAsync(&v[i], words[i], sizeof(int), cudaMemcpyDeviceToHost, s), "status read");
    if (rc) return rc;
  }
  int rc = lbw::cuda_check(cudaStreamSynchronize(s), "status sync");
  if (rc) return rc;
  const int code = v[0] ? v[0] : v[1];
  if (device_code) *device_code = code;
  if (code != 0) {
    for (int i = 0; i < 2; ++i)
      if (v[i]) cudaMemsetAsync(words[i], 0, sizeof(int), s);
    cudaStreamSynchronize(s);
    return lbw::set_error(LBW_ERR_TIMEOUT, "a kernel wait timed out (device code 0x%x)", code);
  }
  return LBW_OK;
}

}  // extern "C"
