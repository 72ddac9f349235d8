// Sequence-parallel K/V exchange over NVLink without streaming multiprocessors.
//
// The reference all-gathers the new chunk's K and V shards into every rank's destination cache chunk
// (wan/modules/model_fast.py:2066-2108, tensor_parallel.py:106-139). Here each rank stages its shard in a
// CUDA-IPC-shared buffer and pulls the other ranks' shards with copy-engine memcpys; ranks signal each other
// with stream memory operations (cuStreamWriteValue32 on the peer's flag word, cuStreamWaitValue32 on its
// own). Nothing of the exchange occupies an SM, so it runs under the attention of the cached chunks instead
// of competing with it for SMs the way a collective kernel does.
//
// Buffer layout (one per rank, same size on every rank, in device memory shared through CUDA IPC):
//   [512, 516)    gathered:  epoch of the last exchange whose rows have all landed in this rank's destination
//                 (read by the gated attention kernel, lbw_chunk_attention_gated)
//   [4096, ...)   K shard [rows, cols] bf16, then V shard [rows, cols] bf16
// Flag blocks (one per rank, LBW_SP_FLAG_BLOCK bytes each, in host memory that every rank of the node maps and
// registers with CUDA, so that the host can also write them):
//   [0, 256)      ready[64]: ready[p] = epoch when rank p has staged its shard for that epoch
//   [256, 512)    done[64]:  done[p]  = epoch when rank p has finished pulling this rank's shard
//   [512, 516)    gathered, as above (a copy the host's watchdog reads)
// A rank's streams wait only on words of its own flag block, so a host thread can always release them (by
// writing the awaited epochs there) when a peer stops taking part: the waits have a limit even though stream
// memory operations have none.
// Epochs count the exchanges on a buffer (1, 2, ...); every rank runs the same sequence of exchanges.
#include <string.h>

#include <mutex>

#include "host_common.cuh"

namespace lbw {

constexpr int PEER_MAX = 64;
constexpr size_t PEER_FLAGS = 4096;
constexpr size_t FLAG_BLOCK = LBW_SP_FLAG_BLOCK;

typedef CUresult (*StreamValueFn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

static StreamValueFn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
    return reinterpret_cast<StreamValueFn>(p);
  return nullptr;
}

static StreamValueFn write_fn() {
  static StreamValueFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] { fn = driver_fn("cuStreamWriteValue32"); });
  return fn;
}

static StreamValueFn wait_fn() {
  static StreamValueFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] { fn = driver_fn("cuStreamWaitValue32"); });
  return fn;
}

// Helper streams for the concurrent peer pulls (one per peer, created once per device) and their events.
struct PullStreams {
  cudaStream_t s[PEER_MAX] = {};
  cudaEvent_t ev[PEER_MAX + 1] = {};
  bool ready = false;
};

static std::mutex g_pull_mu;
static PullStreams g_pull[64];

static int pull_streams(PullStreams** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return set_error(LBW_ERR_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lk(g_pull_mu);
  PullStreams& p = g_pull[dev];
  if (!p.ready) {
    int lo = 0, hi = 0;
    if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess) return set_error(LBW_ERR_CUDA, "stream priority range");
    for (int i = 0; i < PEER_MAX; ++i)
      if (!p.s[i] && cudaStreamCreateWithPriority(&p.s[i], cudaStreamNonBlocking, hi) != cudaSuccess)
        return set_error(LBW_ERR_CUDA, "peer pull stream creation failed");
    for (int i = 0; i <= PEER_MAX; ++i)
      if (!p.ev[i] && cudaEventCreateWithFlags(&p.ev[i], cudaEventDisableTiming) != cudaSuccess)
        return set_error(LBW_ERR_CUDA, "peer pull event creation failed");
    p.ready = true;
  }
  *out = &p;
  return LBW_OK;
}

int pull_streams_init() {
  PullStreams* p = nullptr;
  return pull_streams(&p);
}

void pull_streams_release(int dev) {
  if (dev < 0 || dev >= 64) return;
  std::lock_guard<std::mutex> lk(g_pull_mu);
  PullStreams& p = g_pull[dev];
  for (int i = 0; i < PEER_MAX; ++i)
    if (p.s[i]) {
      cudaStreamDestroy(p.s[i]);
      p.s[i] = nullptr;
    }
  for (int i = 0; i <= PEER_MAX; ++i)
    if (p.ev[i]) {
      cudaEventDestroy(p.ev[i]);
      p.ev[i] = nullptr;
    }
  p.ready = false;
}

}  // namespace lbw

using namespace lbw;

extern "C" {

int lbw_peer_buffer_create(long long bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes <= (long long)PEER_FLAGS) return set_error(LBW_ERR_INVALID, "peer_buffer_create: bad arguments");
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return set_error(LBW_ERR_CUDA, "peer_buffer_create: cudaMalloc of %lld bytes failed", bytes);
  if (cudaMemset(p, 0, PEER_FLAGS) != cudaSuccess) {
    cudaFree(p);
    return set_error(LBW_ERR_CUDA, "peer_buffer_create: flag reset failed");
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return set_error(LBW_ERR_CUDA, "peer_buffer_create: cudaIpcGetMemHandle failed");
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return LBW_OK;
}

int lbw_peer_buffer_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return set_error(LBW_ERR_INVALID, "peer_buffer_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(LBW_ERR_CUDA, "peer_buffer_open: %s", cudaGetErrorString(e));
  return LBW_OK;
}

int lbw_peer_buffer_close(void* ptr, int owned) {
  if (!ptr) return LBW_OK;
  cudaError_t e = owned ? cudaFree(ptr) : cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return set_error(LBW_ERR_CUDA, "peer_buffer_close: %s", cudaGetErrorString(e));
  return LBW_OK;
}

int lbw_host_flags_register(void* host, long long bytes, void** dev) {
  if (!host || !dev || bytes <= 0) return set_error(LBW_ERR_INVALID, "host_flags_register: bad arguments");
  if (!aligned(host, 4096) || bytes % 4096) return set_error(LBW_ERR_ALIGN, "host_flags_register: page alignment");
  cudaError_t e = cudaHostRegister(host, (size_t)bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (e != cudaSuccess) return set_error(LBW_ERR_CUDA, "host_flags_register: %s", cudaGetErrorString(e));
  e = cudaHostGetDevicePointer(dev, host, 0);
  if (e != cudaSuccess) {
    cudaHostUnregister(host);
    return set_error(LBW_ERR_CUDA, "host_flags_register: device pointer: %s", cudaGetErrorString(e));
  }
  return LBW_OK;
}

int lbw_host_flags_unregister(void* host) {
  if (!host) return LBW_OK;
  cudaError_t e = cudaHostUnregister(host);
  if (e != cudaSuccess) return set_error(LBW_ERR_CUDA, "host_flags_unregister: %s", cudaGetErrorString(e));
  return LBW_OK;
}

}  // extern "C"

namespace lbw {

// Shared argument checks and setup of the two halves of an exchange.
struct Exchange {
  StreamValueFn wr = nullptr, wt = nullptr;
  cudaStream_t s = nullptr;
  CUstream cs = nullptr;
  size_t row = 0, pitch = 0, shard = 0;
  uint8_t *mine = nullptr, *kd = nullptr, *vd = nullptr;
  uint8_t* flags = nullptr;  // device address (this process's mapping) of rank 0's flag block
};

static int exchange_setup(Exchange* x, void* const* bufs, void* flags, int rank, int world, unsigned int epoch,
                          void* k_dest, void* v_dest, long long ld, int local_rows, int cols, void* stream,
                          const char* who) {
  if (!bufs || !flags || !k_dest || !v_dest) return set_error(LBW_ERR_INVALID, "%s: null pointer", who);
  if (world < 2 || world > PEER_MAX || rank < 0 || rank >= world || epoch == 0 || local_rows <= 0 || cols <= 0 ||
      ld < cols)
    return set_error(LBW_ERR_SHAPE, "%s: rank %d of %d, epoch %u, %d x %d rows (ld %lld)", who, rank, world, epoch,
                     local_rows, cols, ld);
  for (int p = 0; p < world; ++p)
    if (!bufs[p]) return set_error(LBW_ERR_INVALID, "%s: no buffer for rank %d", who, p);
  x->wr = write_fn();
  x->wt = wait_fn();
  if (!x->wr || !x->wt) return set_error(LBW_ERR_UNSUPPORTED, "%s: stream memory operations unavailable", who);
  x->s = reinterpret_cast<cudaStream_t>(stream);
  x->cs = reinterpret_cast<CUstream>(x->s);
  x->row = (size_t)cols * 2;
  x->pitch = (size_t)ld * 2;
  x->shard = x->row * (size_t)local_rows;
  x->mine = static_cast<uint8_t*>(bufs[rank]);
  x->flags = static_cast<uint8_t*>(flags);
  x->kd = static_cast<uint8_t*>(k_dest);
  x->vd = static_cast<uint8_t*>(v_dest);
  return LBW_OK;
}

// word `p` of region `which` (0 ready, 1 done, 2 gathered) of rank `owner`'s flag block
static CUdeviceptr flag_at(const Exchange& x, int owner, int which, int p) {
  return reinterpret_cast<CUdeviceptr>(x.flags + (size_t)owner * FLAG_BLOCK + which * 256 + 4 * p);
}
// the gathered word the gated attention reads, in this rank's device buffer
static CUdeviceptr gathered_at(const Exchange& x) { return reinterpret_cast<CUdeviceptr>(x.mine + 512); }

static int ck(CUresult r, const char* what) {
  return r == CUDA_SUCCESS ? LBW_OK : set_error(LBW_ERR_CUDA, "sp_kv exchange: %s (%d)", what, (int)r);
}

static int copy_rows(uint8_t* dst, size_t dpitch, const uint8_t* src, size_t spitch, size_t row, int rows,
                     cudaStream_t s) {
  cudaError_t e = (dpitch == row && spitch == row)
                      ? cudaMemcpyAsync(dst, src, row * (size_t)rows, cudaMemcpyDefault, s)
                      : cudaMemcpy2DAsync(dst, dpitch, src, spitch, row, rows, cudaMemcpyDefault, s);
  return e == cudaSuccess ? LBW_OK : set_error(LBW_ERR_CUDA, "sp_kv exchange: copy failed (%s)", cudaGetErrorString(e));
}

}  // namespace lbw

extern "C" {

int lbw_sp_kv_stage(void* const* bufs, void* flags, int rank, int world, unsigned int epoch, void* k_dest,
                    void* v_dest, long long ld, int local_rows, int cols, void* stream) {
  Exchange x;
  int err = exchange_setup(&x, bufs, flags, rank, world, epoch, k_dest, v_dest, ld, local_rows, cols, stream,
                           "sp_kv_stage");
  if (err) return err;
  // every peer has finished pulling this rank's previous shard before it is overwritten
  if (epoch > 1)
    for (int p = 0; p < world; ++p)
      if (p != rank &&
          (err = ck(x.wt(x.cs, flag_at(x, rank, 1, p), epoch - 1, CU_STREAM_WAIT_VALUE_GEQ), "wait done")))
        return err;
  const size_t own = (size_t)rank * local_rows * x.pitch;
  if ((err = copy_rows(x.mine + PEER_FLAGS, x.row, x.kd + own, x.pitch, x.row, local_rows, x.s))) return err;
  if ((err = copy_rows(x.mine + PEER_FLAGS + x.shard, x.row, x.vd + own, x.pitch, x.row, local_rows, x.s))) return err;
  return cuda_check(cudaGetLastError(), "sp_kv_stage");
}

int lbw_sp_kv_gather(void* const* bufs, void* flags, int rank, int world, unsigned int epoch, void* k_dest,
                     void* v_dest, long long ld, int local_rows, int cols, void* stream) {
  Exchange x;
  int err = exchange_setup(&x, bufs, flags, rank, world, epoch, k_dest, v_dest, ld, local_rows, cols, stream,
                           "sp_kv_gather");
  if (err) return err;
  PullStreams* ps = nullptr;
  if ((err = pull_streams(&ps))) return err;
  for (int p = 0; p < world; ++p)
    if (p != rank && (err = ck(x.wr(x.cs, flag_at(x, p, 0, rank), epoch, CU_STREAM_WRITE_VALUE_DEFAULT), "signal ready")))
      return err;
  for (int p = 0; p < world; ++p)
    if (p != rank && (err = ck(x.wt(x.cs, flag_at(x, rank, 0, p), epoch, CU_STREAM_WAIT_VALUE_GEQ), "wait ready")))
      return err;
  // pull every peer's shard on its own stream (copy engines in parallel), join, then release the peers' buffers
  if (cudaEventRecord(ps->ev[PEER_MAX], x.s) != cudaSuccess) return set_error(LBW_ERR_CUDA, "sp_kv_gather: event record");
  for (int p = 0; p < world; ++p) {
    if (p == rank) continue;
    cudaStream_t h = ps->s[p];
    const uint8_t* src = static_cast<const uint8_t*>(bufs[p]) + PEER_FLAGS;
    const size_t off = (size_t)p * local_rows * x.pitch;
    if (cudaStreamWaitEvent(h, ps->ev[PEER_MAX], 0) != cudaSuccess)
      return set_error(LBW_ERR_CUDA, "sp_kv_gather: stream wait failed");
    if ((err = copy_rows(x.kd + off, x.pitch, src, x.row, x.row, local_rows, h))) return err;
    if ((err = copy_rows(x.vd + off, x.pitch, src + x.shard, x.row, x.row, local_rows, h))) return err;
    if (cudaEventRecord(ps->ev[p], h) != cudaSuccess || cudaStreamWaitEvent(x.s, ps->ev[p], 0) != cudaSuccess)
      return set_error(LBW_ERR_CUDA, "sp_kv_gather: join of the pull from rank %d failed", p);
  }
  for (int p = 0; p < world; ++p)
    if (p != rank && (err = ck(x.wr(x.cs, flag_at(x, p, 1, rank), epoch, CU_STREAM_WRITE_VALUE_DEFAULT), "signal done")))
      return err;
  if ((err = ck(x.wr(x.cs, gathered_at(x), epoch, CU_STREAM_WRITE_VALUE_DEFAULT), "signal gathered"))) return err;
  if ((err = ck(x.wr(x.cs, flag_at(x, rank, 2, 0), epoch, CU_STREAM_WRITE_VALUE_DEFAULT), "signal gathered (host)")))
    return err;
  return cuda_check(cudaGetLastError(), "sp_kv_gather");
}

}  // extern "C"
