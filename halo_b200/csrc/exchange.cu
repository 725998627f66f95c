// Cross-GPU LSE merge over NVLink peer memory, fused into one kernel.
//
// Sequence-sharded decode leaves each rank with P local split partials
// (m, l, o) per (b, h) row.  halo_sharded_merge replaces "local merge ->
// all-gather of (o, lse) -> merge of the gathered parts" (three launches and
// a collective) with one kernel per rank: CTA r merges row r's local
// partials, stores the row's normalised (o, lse) straight into slot
// [rank][r] of every peer's exchange buffer (plain stores through peer
// pointers, i.e. NVLink P2P writes), waits (bounded) until the rows of all
// ranks for row r are in its own buffer, and folds the `world` parts into
// the output.  The merge is the identity of halo/kv_cache_chunked.py:194-239
// (lzbaclz/HALO) generalised to P parts; the reference is single-GPU, this
// exchange is new.
//
// Every value travels as one 64-bit word: the call's epoch in the high half,
// the fp32 bits in the low half.  An aligned 64-bit store is single-copy
// atomic, so a reader that sees the current epoch in a word also sees that
// word's value: no flags, no system-scope fences, one NVLink trip.
//
// Exchange buffer (one per rank, allocated with halo_ipc_alloc, mapped on
// every peer with halo_ipc_open), then control words only the owner touches:
//   word[2][world][R][Dv + 2]   parity = epoch & 1; o, lse, pad per row
//   ctrl[4]                     [0] epoch of the last completed call,
//                               [1] CTAs of the running call that finished
// The epoch lives on the device: each CTA reads ctrl[0] + 1 when it starts,
// and the last CTA to finish stores it back, so every rank advances by one
// per call without the host passing a counter, and a captured CUDA graph
// replays correctly.  A rank can only run one call ahead of any peer (it
// needs that peer's row of the current call first), so the parity slot it
// writes was last read two calls earlier.  No TMA, no multicast: plain
// loads and stores.
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
// Four warps and at most 88 registers a thread, so a CTA fits beside two
// split-KV CTAs on an SM: launched as a dependent, the merge's CTAs are
// resident (waiting) while the split-KV kernel drains and start the moment
// it completes.
constexpr int kWarps = 4;

struct Params {
  const float* m_parts;     // local split partials (as halo_lse_merge)
  const float* l_parts;     // may be NULL (every part normalised)
  const float* o_parts;
  int64_t ps, rs, ops, ors;
  int32_t R, H, P, Dv;
  int32_t world, rank;
  char* bufs[kMaxWorld];    // every rank's exchange buffer, mapped here
  int32_t out_dtype;
  char* out;
  int64_t out_sb, out_sh;
  float* lse;
  unsigned int* err;
};

// One CTA (kWarps warps) per (b, h) row; lane l owns the DPL consecutive
// columns [l*DPL, l*DPL + DPL) of the local merge.
template <int DPL, bool VEC>
__global__ void __maxnreg__(88) kx_kernel(const __grid_constant__ Params p) {
  __shared__ float s_red[kWarps];
  __shared__ float s_l[kWarps];
  __shared__ __align__(16) float s_o[kWarps][DPL * 32];
  __shared__ float s_row[257];
  __shared__ float s_w[kMaxWorld];
  extern __shared__ float s_x[];   // [world][Dv + 1]
  __shared__ int s_ok;
  __shared__ uint32_t s_epoch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x;
  const int Dv = p.Dv;
  const size_t row_words = (size_t)Dv + 2;   // o, lse, pad
  const size_t rank_words = (size_t)p.R * row_words;
  const size_t par_words = (size_t)p.world * rank_words;
  uint64_t* const data_own = reinterpret_cast<uint64_t*>(p.bufs[p.rank]);
  uint32_t* const ctrl = reinterpret_cast<uint32_t*>(data_own + 2 * par_words);
  grid_dep_trigger();   // the next split-KV launch may start its prologue
  grid_dep_wait();      // the partials' writer has finished (dependent launch)
  if (threadIdx.x == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(ctrl) + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int par = epoch & 1u;
  const uint64_t tag = (uint64_t)epoch << 32;

  // ---- 1. local merge of this rank's P partials (one round trip when
  // P <= 40, or 16 for rows wider than 128), normalised into s_row: o then lse
  const float* mr = p.m_parts + (int64_t)row * p.rs;
  const float* lr = p.l_parts ? p.l_parts + (int64_t)row * p.rs : nullptr;
  const float* orow = p.o_parts + (int64_t)row * p.ors;
  float M, L;
  float acc[DPL];
  merge_partials<DPL, kWarps, kMergeRound<DPL>, VEC>(mr, lr, orow, p.ps, p.ops, p.P, Dv, s_red,
                                                     s_l, s_o, M, L, acc);
  if (warp == 0) {
    const int d0 = lane * DPL;
#pragma unroll
    for (int e = 0; e < DPL; ++e)
      if (d0 + e < Dv) s_row[d0 + e] = (L > 0.f) ? acc[e] / L : 0.f;   // normalised local output
    if (lane == 0) s_row[Dv] = (L > 0.f) ? M + logf(L) : -INFINITY;     // lse of the local part
  }
  __syncthreads();

  // ---- 2. push the row into slot [rank][row] of every peer's buffer
  // (NVLink stores; pulling instead, with peer loads, measured slower: every
  // poll of a word not yet written is a remote round trip)
  for (int j = 0; j < p.world; ++j) {
    if (j == p.rank) continue;
    uint64_t* dst = reinterpret_cast<uint64_t*>(p.bufs[j]) + par * par_words +
                    (size_t)p.rank * rank_words + (size_t)row * row_words;
    for (int d = threadIdx.x; d <= Dv; d += blockDim.x)
      st_relaxed_sys(dst + d, tag | __float_as_uint(s_row[d]));
  }

  // ---- 3. collect every rank's row from this rank's buffer (bounded wait
  // on the epoch tags): a thread issues the loads of kBatch of its words
  // before checking any, so an 8-rank row costs one or two round trips
  // rather than eight
  constexpr int kBatch = 8;
  const uint64_t* src = data_own + par * par_words + (size_t)row * row_words;
  auto word = [&](int j, int d) -> const uint64_t* { return src + (size_t)j * rank_words + d; };
  const int n_words = p.world * (Dv + 1);   // o and lse words of every rank
  bool all_ok = true;
  for (int base = threadIdx.x; base < n_words && all_ok; base += kBatch * blockDim.x) {
    uint64_t v[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = base + u * blockDim.x;
      const int j = i / (Dv + 1), d = i - j * (Dv + 1);
      v[u] = (i < n_words && j != p.rank) ? ld_relaxed_sys(word(j, d)) : 0;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = base + u * blockDim.x;
      if (i >= n_words || !all_ok) continue;
      const int j = i / (Dv + 1), d = i - j * (Dv + 1);
      if (j == p.rank) {
        s_x[i] = s_row[d];
        continue;
      }
      uint64_t w = v[u];
      if ((uint32_t)(w >> 32) != epoch) {
        const uint64_t* a = word(j, d);
        const uint64_t t0 = globaltimer_ns();
        while ((uint32_t)(w >> 32) != epoch) {
          for (int k = 0; k < 64 && (uint32_t)(w >> 32) != epoch; ++k) w = ld_relaxed_sys(a);
          if ((uint32_t)(w >> 32) != epoch && globaltimer_ns() - t0 > kWaitLimitNs) {
            set_device_error(p.err, static_cast<unsigned int>(-HALO_ERR_TIMEOUT));
            s_ok = 0;
            all_ok = false;
            break;
          }
        }
        if (!all_ok) continue;
      }
      s_x[i] = __uint_as_float((uint32_t)w);   // i = j * (Dv + 1) + d
    }
  }
  __syncthreads();

  // ---- 4. fold the world parts (lse-weighted) and write the output
  if (s_ok) {
    float Mx = -INFINITY;
    for (int j = 0; j < p.world; ++j) Mx = fmaxf(Mx, s_x[j * (Dv + 1) + Dv]);
    if (threadIdx.x < p.world) {
      const float lj = s_x[threadIdx.x * (Dv + 1) + Dv];
      s_w[threadIdx.x] = (lj == -INFINITY) ? 0.f : expf(lj - Mx);
    }
    __syncthreads();
    float W = 0.f;
    for (int j = 0; j < p.world; ++j) W += s_w[j];
    const int b = row / p.H, h = row % p.H;
    if (threadIdx.x == 0 && p.lse) p.lse[row] = (W > 0.f) ? Mx + logf(W) : -INFINITY;
    const float invW = (W > 0.f) ? 1.f / W : 0.f;
    for (int d = threadIdx.x; d < Dv; d += blockDim.x) {
      float v = 0.f;
      for (int j = 0; j < p.world; ++j)
        if (s_w[j] != 0.f) v = fmaf(s_x[j * (Dv + 1) + d], s_w[j], v);
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
  // the last CTA of the call publishes its epoch for the next call (the
  // kernel boundary makes it visible to the next launch)
  if (threadIdx.x == 0) {
    if (atomicAdd(ctrl + 1, 1u) == (uint32_t)p.R - 1) {
      ctrl[1] = 0;
      *reinterpret_cast<volatile uint32_t*>(ctrl) = epoch;
    }
  }
}

}  // namespace exchange

// Host-side checks of a sharded merge's arguments, shared by
// halo_sharded_merge and halo_sharded_decode (which runs them before it
// launches the split-KV kernel).
int validate_exchange(int32_t B, int32_t H, int32_t Dv, int32_t P, const float* m_parts,
                      const float* o_parts, int32_t world, int32_t rank, void* const* bufs,
                      int32_t out_dtype, const void* out) {
  if (B <= 0 || H <= 0 || P < 0 || Dv <= 0 || Dv > 256)
    return fail(HALO_ERR_INVALID_ARG, "bad merge shape");
  if (world <= 0 || world > exchange::kMaxWorld || rank < 0 || rank >= world)
    return fail(HALO_ERR_INVALID_ARG, "bad world %d / rank %d", world, rank);
  if ((P > 0 && (!m_parts || !o_parts)) || !bufs || !out)
    return fail(HALO_ERR_INVALID_ARG, "NULL pointer");
  if (out_dtype != HALO_DTYPE_F32 && out_dtype != HALO_DTYPE_BF16 && out_dtype != HALO_DTYPE_F16)
    return fail(HALO_ERR_INVALID_ARG, "bad out dtype %d", out_dtype);
  for (int j = 0; j < world; ++j)
    if (!bufs[j]) return fail(HALO_ERR_INVALID_ARG, "exchange buffer %d is NULL", j);
  return HALO_OK;
}

}  // namespace halo

using namespace halo;

extern "C" int64_t halo_exchange_bytes(int32_t world, int32_t rows, int32_t Dv) {
  if (world <= 0 || world > exchange::kMaxWorld || rows <= 0 || Dv <= 0 || Dv > 256)
    return fail(HALO_ERR_INVALID_ARG, "bad exchange shape (world %d, rows %d, Dv %d)", world,
                rows, Dv);
  return 2LL * world * rows * (Dv + 2) * 8 + 16;   // tagged words + control words
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
                                      void* const* bufs, int32_t out_dtype,
                                      void* out, int64_t out_stride_b, int64_t out_stride_h,
                                      float* lse, halo_stream_t stream) {
  const int rc = validate_exchange(B, H, Dv, P, m_parts, o_parts, world, rank, bufs, out_dtype,
                                   out);
  if (rc != HALO_OK) return rc;
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
  for (int j = 0; j < world; ++j) prm.bufs[j] = static_cast<char*>(bufs[j]);
  prm.out_dtype = out_dtype;
  prm.out = static_cast<char*>(out);
  prm.out_sb = out_stride_b;
  prm.out_sh = out_stride_h;
  prm.lse = lse;
  prm.err = device_error_ptr();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(prm.R), block(exchange::kWarps * 32);
  const size_t xsm = (size_t)world * (Dv + 1) * sizeof(float);   // staged rows of every rank
  const bool vec = (reinterpret_cast<uintptr_t>(o_parts) & 15) == 0 && o_part_stride % 4 == 0 &&
                   o_row_stride % 4 == 0;
  // a dependent launch: scheduled while the split-KV kernel's last CTAs run
  cudaError_t e;
  if (Dv <= 32) e = launch_dependent(exchange::kx_kernel<1, false>, grid, block, xsm, st, prm);
  else if (Dv <= 64) e = launch_dependent(exchange::kx_kernel<2, false>, grid, block, xsm, st, prm);
  else if (Dv <= 128 && Dv % 4 == 0 && vec)
    e = launch_dependent(exchange::kx_kernel<4, true>, grid, block, xsm, st, prm);
  else if (Dv <= 128) e = launch_dependent(exchange::kx_kernel<4, false>, grid, block, xsm, st, prm);
  else e = launch_dependent(exchange::kx_kernel<8, false>, grid, block, xsm, st, prm);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kx_kernel launch");
  count_launches(1);
  return HALO_OK;
}
