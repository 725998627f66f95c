// Shared device helpers for the HALO B200 kernels (sm_100a).
//
// Everything here is hand-written inline PTX for the async-copy engine
// (cp.async.bulk + mbarrier transaction counts), warp-level tensor-core
// fragments (ldmatrix + mma.sync) and bounded waits.  Every spin-wait has a
// wall-clock limit: on expiry it records an error code in the device error
// word and the caller unwinds instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/halo_b200.h"

namespace halo {

// ---------------------------------------------------------------- errors
// Device-side error word (one per device that loads the library, defined in
// decode.cu).  Kernels receive its address as a parameter and set it with
// atomicCAS so the first error wins; the host reads and clears it through
// halo_device_error().  device_error_ptr() returns the current device's copy.
unsigned int* device_error_ptr();

// Process-wide count of kernels this library has launched (halo_launch_count).
void count_launches(int n = 1);

__device__ __forceinline__ void set_device_error(unsigned int* err, unsigned int code) {
  if (err) atomicCAS(err, 0u, code);
}

// exp2 on the special-function unit (relative error ~2^-22; subnormal
// results flush to zero).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wall-clock limit of every bounded wait (nanoseconds).
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Control block at the start of every decode workspace: the dynamic
// schedule's per-pair piece counters and its exit counter.  It must be zero
// before a workspace's first use; every call that completes leaves it zero.
constexpr int64_t kCtrlBytes = 4096;

// System-scope relaxed 64-bit accesses (peer GPU memory through NVLink): an
// aligned 64-bit access is single-copy atomic.
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Named CTA barrier `id` (1..15) over `threads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with launch_dependent() may be scheduled before the
// kernel ahead of it in the stream has finished (once every CTA of that
// kernel has called grid_dep_trigger() or exited); it must call
// grid_dep_wait() before touching anything the earlier kernel writes, which
// returns once that kernel has completed and its memory is visible.  For a
// kernel launched normally grid_dep_wait() returns at once.
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive_n(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(n)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the given phase parity.  Returns false (and records
// HALO_ERR_TIMEOUT in *err) when the wall-clock limit expires.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_device_error(err, static_cast<unsigned int>(-HALO_ERR_TIMEOUT));
      return false;
    }
  }
}

// The same bounded wait with mbarrier.try_wait's suspend-time hint: each
// poll may block the thread in the barrier unit for up to `hint_ns` and
// returns as soon as the phase completes, so a long wait takes fewer polls
// (and fewer issue slots) than back-to-back polls.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity,
                                                   uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_hint(uint64_t* bar, uint32_t parity, unsigned int* err,
                                               uint32_t hint_ns) {
  if (mbar_try_wait_hint(bar, parity, hint_ns)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 8; ++i)
      if (mbar_try_wait_hint(bar, parity, hint_ns)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_device_error(err, static_cast<unsigned int>(-HALO_ERR_TIMEOUT));
      return false;
    }
  }
}

// ---------------------------------------------------------------- bulk copy
// One-dimensional bulk copy global -> shared through the async-copy (TMA)
// engine; completion is signalled as transaction bytes on `bar`.  `src` and
// `dst` must be 16-byte aligned and `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Tiled 4-D tensor load (TMA) into shared memory; completion counted as
// transaction bytes on `bar`.  Coordinates are {inner, row, head, batch};
// the inner coordinate times the element size must be a multiple of 16.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
        "r"(c3), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
        "r"(smem_addr(bar))
      : "memory");
}

// Byte offset of 16-byte chunk `c16` (along the row) of row `row` in a tile
// written by swizzled TMA boxes of BOX_ROWS rows x INNER bytes (INNER = 32,
// 64 or 128 with the matching 32B/64B/128B swizzle mode; boxes stacked along
// the row).  The TMA swizzle XORs address bits [4, 4+b) with bits [7, 7+b),
// b = log2(INNER/16); with INNER-byte rows that is chunk j of row r stored at
// j ^ ((r >> (7 - log2 INNER)) % (INNER/16)).  The tile base must be
// 1024-byte aligned.
template <int INNER = 128, int BOX_ROWS = 64>
__device__ __forceinline__ uint32_t swz(int row, int c16) {
  constexpr int kCpb = INNER / 16;
  constexpr int kShift = INNER == 128 ? 0 : (INNER == 64 ? 1 : 2);
  const int box = c16 / kCpb, c = c16 % kCpb;
  const int x = (row >> kShift) & (kCpb - 1);
  return static_cast<uint32_t>(box * (BOX_ROWS * INNER) + row * INNER + ((c ^ x) << 4));
}

// ---------------------------------------------------------------- fragments
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Transpose of an 8x8 matrix of 16-bit values held one row pair per thread
// (thread t: row t/4, columns 2(t%4), 2(t%4)+1) across the warp.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
struct Elem;

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kDtype = HALO_DTYPE_BF16;
  // Round a pair of floats to one packed register (lo -> bits 0..15).
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ void unpack(uint32_t r, float& lo, float& hi) {
    lo = __uint_as_float(r << 16);
    hi = __uint_as_float(r & 0xFFFF0000u);
  }
};

template <>
struct Elem<__half> {
  static constexpr int kDtype = HALO_DTYPE_F16;
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f32(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ void unpack(uint32_t r, float& lo, float& hi) {
    __half2 h = *reinterpret_cast<__half2*>(&r);
    float2 f = __half22float2(h);
    lo = f.x;
    hi = f.y;
  }
};

// D[16x8] += A[16x16] * B[16x8], fp32 accumulate.
__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1,
                                          __nv_bfloat16*) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1,
                                          __half*) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__host__ __device__ __forceinline__ int64_t ceil_div64(int64_t a, int64_t b) {
  return (a + b - 1) / b;
}

}  // namespace halo
