// Cross-GPU LSE merge over NVLink peer memory, fused into one kernel.
//
// Sequence-sharded decode leaves each rank with P local split partials
// (m, l, o) per (b, h) row.  halo_sharded_merge replaces "local merge ->
// all-gather of (o, lse) -> merge of the gathered parts" (three launches and
// a collective) with one kernel per rank: CTA r merges row r's local
// partials, stores the row's normalised (o, lse) straight into slot
// [rank][r] of every rank's exchange buffer (plain stores through peer
// pointers, i.e. NVLink P2P writes), publishes a per-row flag on each rank
// with a system-scope release, waits (bounded) for the flags of all ranks
// for row r in its own buffer, and folds the `world` parts into the output.
// The merge is the identity of halo/kv_cache_chunked.py:194-239 (lzbaclz/HALO)
// generalised to P parts; the reference is single-GPU, this exchange is new.
//
// Exchange buffer (one per rank, allocated with halo_ipc_alloc, mapped on
// every peer with halo_ipc_open), fp32 data then uint32 flags:
//   data[2][world][R][Dv + 1]   parity = epoch & 1; o then lse per row
//   flag[world][R]              last epoch whose row arrived from that rank
// Epochs increase by one per call.  A rank can only run one call ahead of
// any peer (it needs that peer's row of the current call first), so the
// parity slot it writes was last read two calls earlier, and readers wait
// for flag >= epoch.  No TMA, no multicast: plain loads and stores.
#include <cstdint>
#include <cstring>

#include "halo_common.cuh"
#include "merge_row.cuh"

namespace halo {

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
void count_launches(int n);

namespace exchange {

constexpr int kMaxWorld = 8;
constexpr int kWarps = 16;

struct Params {
  const float* m_parts;     // local split partials (as halo_lse_merge)
  const float* l_parts;     // may be NULL (every part normalised)
  const float* o_parts;
  int64_t ps, rs, ops, ors;
  int32_t R, H, P, Dv;
  int32_t world, rank;
  uint32_t epoch;
  char* bufs[kMaxWorld];    // every rank's exchange buffer, mapped here
  int32_t out_dtype;
  char* out;
  int64_t out_sb, out_sh;
  float* lse;
  unsigned int* err;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One CTA (kWarps warps) per (b, h) row; lane l owns the DPL consecutive
// columns [l*DPL, l*DPL + DPL) of the local merge.
template <int DPL, bool VEC>
__global__ void __launch_bounds__(kWarps * 32) kx_kernel(const __grid_constant__ Params p) {
  __shared__ float s_red[kWarps];
  __shared__ float s_l[kWarps];
  __shared__ __align__(16) float s_o[kWarps][DPL * 32];
  __shared__ float s_row[257];
  __shared__ int s_ok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x;
  const int Dv = p.Dv;
  const size_t row_floats = (size_t)Dv + 1;
  const size_t par_floats = (size_t)p.world * p.R * row_floats;
  float* const data_own = reinterpret_cast<float*>(p.bufs[p.rank]);
  uint32_t* const flags_own = reinterpret_cast<uint32_t*>(data_own + 2 * par_floats);
  const int par = p.epoch & 1u;

  // ---- 1. local merge of this rank's P partials
  const float* mr = p.m_parts + (int64_t)row * p.rs;
  const float* lr = p.l_parts ? p.l_parts + (int64_t)row * p.rs : nullptr;
  const float* orow = p.o_parts + (int64_t)row * p.ors;
  const float M = row_max<kWarps>(mr, p.ps, p.P, s_red);
  float L;
  float acc[DPL];
  fold_partials<DPL, kWarps, 8, VEC>(mr, lr, orow, p.ps, p.ops, p.P, Dv, M, L, acc);
  if (lane == 0) s_l[warp] = L;
  const int d0 = lane * DPL;
#pragma unroll
  for (int e = 0; e < DPL; ++e) s_o[warp][d0 + e] = acc[e];
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += s_l[w];
    s_row[Dv] = (t > 0.f) ? M + logf(t) : -INFINITY;   // lse of the local part
    s_red[0] = t;
  }
  __syncthreads();
  const float Lloc = s_red[0];
  for (int d = threadIdx.x; d < Dv; d += blockDim.x) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += s_o[w][d];
    s_row[d] = (Lloc > 0.f) ? v / Lloc : 0.f;          // normalised local output
  }
  __syncthreads();

  // ---- 2. push the row into slot [rank][row] of every rank's buffer
  for (int j = 0; j < p.world; ++j) {
    float* dst = reinterpret_cast<float*>(p.bufs[j]) + par * par_floats +
                 ((size_t)p.rank * p.R + row) * row_floats;
    for (int d = threadIdx.x; d <= Dv; d += blockDim.x) dst[d] = s_row[d];
  }
  __syncthreads();
  if (threadIdx.x < p.world) {
    __threadfence_system();
    uint32_t* f = reinterpret_cast<uint32_t*>(reinterpret_cast<float*>(p.bufs[threadIdx.x]) +
                                              2 * par_floats) +
                  (size_t)p.rank * p.R + row;
    st_release_sys(f, p.epoch);
  }

  // ---- 3. wait (bounded) for every rank's row
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < p.world) {
    const uint32_t* f = flags_own + (size_t)threadIdx.x * p.R + row;
    bool ok = (int32_t)(ld_acquire_sys(f) - p.epoch) >= 0;
    if (!ok) {
      const uint64_t t0 = globaltimer_ns();
      while (true) {
        for (int i = 0; i < 64 && !ok; ++i) ok = (int32_t)(ld_acquire_sys(f) - p.epoch) >= 0;
        if (ok) break;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          set_device_error(p.err, static_cast<unsigned int>(-HALO_ERR_TIMEOUT));
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (!s_ok) return;

  // ---- 4. fold the world parts (lse-weighted) and write the output
  const float* base = data_own + par * par_floats + (size_t)row * row_floats;
  const size_t rank_stride = (size_t)p.R * row_floats;
  float Mx = -INFINITY;
  for (int j = 0; j < p.world; ++j) Mx = fmaxf(Mx, __ldcg(base + j * rank_stride + Dv));
  float W = 0.f;
  for (int j = 0; j < p.world; ++j) {
    const float lj = __ldcg(base + j * rank_stride + Dv);
    W += (lj == -INFINITY) ? 0.f : expf(lj - Mx);
  }
  const int b = row / p.H, h = row % p.H;
  if (threadIdx.x == 0 && p.lse)
    p.lse[row] = (W > 0.f) ? Mx + logf(W) : -INFINITY;
  const float invW = (W > 0.f) ? 1.f / W : 0.f;
  for (int d = threadIdx.x; d < Dv; d += blockDim.x) {
    float v = 0.f;
    for (int j = 0; j < p.world; ++j) {
      const float lj = __ldcg(base + j * rank_stride + Dv);
      if (lj == -INFINITY) continue;
      v = fmaf(__ldcg(base + j * rank_stride + d), expf(lj - Mx), v);
    }
    v *= invW;
    const int64_t off = (int64_t)b * p.out_sb + (int64_t)h * p.out_sh + d;
    if (p.out_dtype == HALO_DTYPE_F32)
      reinterpret_cast<float*>(p.out)[off] = v;
    else if (p.out_dtype == HALO_DTYPE_BF16)
      reinterpret_cast<__nv_bfloat16*>(p.out)[off] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<__half*>(p.out)[off] = __float2half_rn(v);
  }
}

}  // namespace exchange
}  // namespace halo

using namespace halo;

extern "C" int64_t halo_exchange_bytes(int32_t world, int32_t rows, int32_t Dv) {
  if (world <= 0 || world > exchange::kMaxWorld || rows <= 0 || Dv <= 0 || Dv > 256)
    return fail(HALO_ERR_INVALID_ARG, "bad exchange shape (world %d, rows %d, Dv %d)", world,
                rows, Dv);
  const int64_t data = 2LL * world * rows * (Dv + 1) * 4;
  return data + (int64_t)world * rows * 4;
}

extern "C" int32_t halo_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle_out) {
  if (bytes <= 0 || !dev_ptr || !handle_out) return fail(HALO_ERR_INVALID_ARG, "bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (exchange buffer)");
  e = cudaMemset(p, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "exchange buffer setup");
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *dev_ptr = p;
  return HALO_OK;
}

extern "C" int32_t halo_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return fail(HALO_ERR_INVALID_ARG, "bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *dev_ptr = p;
  return HALO_OK;
}

extern "C" int32_t halo_ipc_close(void* dev_ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? HALO_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

extern "C" int32_t halo_ipc_free(void* dev_ptr) {
  cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? HALO_OK : cuda_fail(e, "cudaFree (exchange buffer)");
}

extern "C" int32_t halo_sharded_merge(int32_t B, int32_t H, int32_t Dv, int32_t P,
                                      const float* m_parts, const float* l_parts,
                                      const float* o_parts, int64_t part_stride,
                                      int64_t row_stride, int64_t o_part_stride,
                                      int64_t o_row_stride, int32_t world, int32_t rank,
                                      uint32_t epoch, void* const* bufs, int32_t out_dtype,
                                      void* out, int64_t out_stride_b, int64_t out_stride_h,
                                      float* lse, halo_stream_t stream) {
  if (B <= 0 || H <= 0 || P < 0 || Dv <= 0 || Dv > 256)
    return fail(HALO_ERR_INVALID_ARG, "bad merge shape");
  if (world <= 0 || world > exchange::kMaxWorld || rank < 0 || rank >= world)
    return fail(HALO_ERR_INVALID_ARG, "bad world %d / rank %d", world, rank);
  if ((P > 0 && (!m_parts || !o_parts)) || !bufs || !out)
    return fail(HALO_ERR_INVALID_ARG, "NULL pointer");
  if (out_dtype != HALO_DTYPE_F32 && out_dtype != HALO_DTYPE_BF16 && out_dtype != HALO_DTYPE_F16)
    return fail(HALO_ERR_INVALID_ARG, "bad out dtype %d", out_dtype);
  exchange::Params prm{};
  prm.m_parts = m_parts;
  prm.l_parts = l_parts;
  prm.o_parts = o_parts;
  prm.ps = part_stride;
  prm.rs = row_stride;
  prm.ops = o_part_stride;
  prm.ors = o_row_stride;
  prm.R = B * H;
  prm.H = H;
  prm.P = P;
  prm.Dv = Dv;
  prm.world = world;
  prm.rank = rank;
  prm.epoch = epoch;
  for (int j = 0; j < world; ++j) {
    if (!bufs[j]) return fail(HALO_ERR_INVALID_ARG, "exchange buffer %d is NULL", j);
    prm.bufs[j] = static_cast<char*>(bufs[j]);
  }
  prm.out_dtype = out_dtype;
  prm.out = static_cast<char*>(out);
  prm.out_sb = out_stride_b;
  prm.out_sh = out_stride_h;
  prm.lse = lse;
  prm.err = device_error_ptr();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(prm.R), block(exchange::kWarps * 32);
  const bool vec = (reinterpret_cast<uintptr_t>(o_parts) & 15) == 0 && o_part_stride % 4 == 0 &&
                   o_row_stride % 4 == 0;
  if (Dv <= 32) exchange::kx_kernel<1, false><<<grid, block, 0, st>>>(prm);
  else if (Dv <= 64) exchange::kx_kernel<2, false><<<grid, block, 0, st>>>(prm);
  else if (Dv <= 128 && Dv % 4 == 0 && vec) exchange::kx_kernel<4, true><<<grid, block, 0, st>>>(prm);
  else if (Dv <= 128) exchange::kx_kernel<4, false><<<grid, block, 0, st>>>(prm);
  else exchange::kx_kernel<8, false><<<grid, block, 0, st>>>(prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kx_kernel launch");
  count_launches(1);
  return HALO_OK;
}
