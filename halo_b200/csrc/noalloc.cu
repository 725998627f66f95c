// halo_chunked_decode_noalloc: the split-KV decode + merge with its scratch
// in a fixed, library-owned device array instead of a caller workspace.
//
// Why: some callers cannot allocate device memory at the moment they need
// attention -- e.g. code running inside a framework that owns every device
// allocation through its own pool, a plugin host that forbids cudaMalloc on
// its hot path (cudaMalloc may synchronise the device), or a C/FFI caller
// with no allocator of its own.  They still pass their own inputs and
// outputs; only the partial (m, l, o) scratch moves into this file.
//
// Limits and rules (also stated in include/halo_b200.h):
//  * The scratch holds kNoAllocScratchBytes (8 MiB).  A problem whose
//    partials need more is rejected with HALO_ERR_WORKSPACE before any work
//    is enqueued; use halo_chunked_decode with a caller workspace instead.
//  * Every GPU that loads the library keeps this array until process exit.
//  * All calls on a device share the one array and it keeps the last call's
//    contents.  Its first 4096 bytes are the split-KV scheduler's counters,
//    which must be zero when a call starts: each call clears them on its
//    stream (cudaMemsetAsync, no allocation) before the kernels, so a call
//    that ended early (a timed-out wait) cannot leave stale counters for the
//    next.  The partials after them are written before they are read.
//    Calls whose work overlaps on the GPU (other streams, other host
//    threads) race on the array; serialise them.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current).  Make that first call
//    before any stream capture.  The address is cached for the life of the
//    process: after cudaDeviceReset (or any teardown of the device's primary
//    context) it is stale, so this entry point must not be used on that
//    device again in the same process.
//  * No cudaMalloc, cudaFree or other device allocation happens here.
#include <mutex>

#include "halo_common.cuh"

namespace halo {

constexpr int64_t kNoAllocScratchBytes = 8ll << 20;

// File-scope scratch.  In host code this name is only a stand-in for the
// symbol: its device address must be looked up per device (below) and passed
// to the kernels, never taken directly.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);

// Device address of g_noalloc_scratch on the current device, looked up once
// per device with that device current.  Returns nullptr on failure (the
// error string is set).
static void* scratch_ptr() {
  static std::mutex mu;
  static void* cache[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cuda_fail(e, "cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    fail(HALO_ERR_UNSUPPORTED, "device index %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
      return nullptr;
    }
    cache[dev] = ptr;
  }
  return cache[dev];
}

}  // namespace halo

extern "C" int32_t halo_chunked_decode_noalloc(const halo_decode_problem_t* problem,
                                               const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                               const halo_merge_args_t* merge,
                                               halo_stream_t stream) {
  const int64_t need = halo_decode_workspace_bytes(problem, chunks, n_chunks);
  if (need < 0) return static_cast<int32_t>(need);
  if (need > halo::kNoAllocScratchBytes)
    return halo::fail(HALO_ERR_WORKSPACE,
                      "problem needs %lld bytes of scratch but the no-alloc entry point has a "
                      "fixed %lld; call halo_chunked_decode with a workspace instead",
                      (long long)need, (long long)halo::kNoAllocScratchBytes);
  void* ptr = halo::scratch_ptr();
  if (!ptr) return HALO_ERR_CUDA;
  cudaError_t e = cudaMemsetAsync(ptr, 0, halo::kCtrlBytes,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return halo::cuda_fail(e, "clear no-alloc scratch counters");
  return halo_chunked_decode(problem, chunks, n_chunks, ptr, halo::kNoAllocScratchBytes, merge,
                             stream);
}
