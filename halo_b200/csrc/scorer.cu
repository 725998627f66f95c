// Chunk-hotness scorer (Quest upper bound) for B200.
//
// Replaces the torch ops of baselines/quest_path_d.py in lzbaclz/HALO:
//   * page_summary_kernel: per-page channel-wise min/max of K
//     (observe_keys, :125-150).  Exact (min/max of the stored values).
//   * page_score_kernel:   GQA mean-pooled query (fp32 sum over the group,
//     one division, one rounding to the query dtype -- how torch evaluates
//     `.mean(dim=2)` on 16-bit tensors, :166-172) and the Quest bound
//     sum_d max(q_d * kmin_d, q_d * kmax_d) in fp32 (:175-179).
//   * page_topk_kernel:    max over (batch, kv-head, query) per page
//     (:197), optional exclusion mask, and the top-k pages by score, largest
//     first, ties to the lower page index (one CTA, bitonic sort in shared
//     memory).
// All HBM-bound except top-k, which touches P floats.
//
// The HALOPress ablation scorer of baselines/scorer_ablations.py:184-268:
//   * page_mean_kernel:  per-page mean key (observe_keys, :208-218): fp32
//     sum over the page's rows in row order, one division by the page size,
//     one rounding to the key dtype.
//   * page_attn_kernel:  the attention proxy q_g . K_mean per (b, kv-head,
//     query, page), fp32 (:231-234), q_g the GQA mean as for Quest.
//   * press_topk_kernel: max over (b, kv-head, query), min-max
//     normalisation, the recency and sink terms, alpha*attn + beta*rec +
//     gamma*sink with one rounding per operation (:235-262), and the top-k
//     pages (one CTA).
#include <cstdint>
#include <mutex>

#include "halo_common.cuh"

namespace halo {

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p) {
  if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float*>(p);
  else return Elem<T>::to_f32(*p);
}

template <typename T>
__device__ __forceinline__ T st_elem(float x) {
  if constexpr (sizeof(T) == 4) return x;
  else return Elem<T>::from_f32(x);
}

// Round an fp32 value to T and back (identity for fp32).
template <typename T>
__device__ __forceinline__ float ld_f32_round(float x) {
  if constexpr (sizeof(T) == 4) return x;
  else return Elem<T>::to_f32(Elem<T>::from_f32(x));
}

// One warp per page; lane handles columns lane, lane+32, ...
struct SummaryParams {
  const char* k;
  int64_t sb, sh, st;         // element strides of K
  char* kmin;
  char* kmax;
  int64_t ob, oh, op;         // element strides of kmin/kmax (b, h, page)
  int32_t H_kv, D, page, page_begin, n_pages;
};

template <typename T>
__global__ void __launch_bounds__(128) page_summary_kernel(const SummaryParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pg = blockIdx.x * 4 + warp;
  if (pg >= p.n_pages) return;
  const int bh = blockIdx.y;
  const int b = bh / p.H_kv, h = bh % p.H_kv;
  const int page = p.page_begin + pg;
  const T* base = reinterpret_cast<const T*>(p.k) + b * p.sb + h * p.sh + (int64_t)page * p.page * p.st;
  T* mn_out = reinterpret_cast<T*>(p.kmin) + b * p.ob + h * p.oh + (int64_t)page * p.op;
  T* mx_out = reinterpret_cast<T*>(p.kmax) + b * p.ob + h * p.oh + (int64_t)page * p.op;
  for (int d = lane; d < p.D; d += 32) {
    float mn = INFINITY, mx = -INFINITY;
    for (int r = 0; r < p.page; ++r) {
      const float x = ld_f32(base + (int64_t)r * p.st + d);
      mn = fminf(mn, x);
      mx = fmaxf(mx, x);
    }
    mn_out[d] = st_elem<T>(mn);
    mx_out[d] = st_elem<T>(mx);
  }
}

// One warp per page; lane handles columns lane, lane+32, ...  kmin carries
// the output (kmax unused).
template <typename T>
__global__ void __launch_bounds__(128) page_mean_kernel(const SummaryParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pg = blockIdx.x * 4 + warp;
  if (pg >= p.n_pages) return;
  const int bh = blockIdx.y;
  const int b = bh / p.H_kv, h = bh % p.H_kv;
  const int page = p.page_begin + pg;
  const T* base = reinterpret_cast<const T*>(p.k) + b * p.sb + h * p.sh + (int64_t)page * p.page * p.st;
  T* out = reinterpret_cast<T*>(p.kmin) + b * p.ob + h * p.oh + (int64_t)page * p.op;
  const float n_rows = (float)p.page;
  for (int d = lane; d < p.D; d += 32) {
    float s = 0.f;
    for (int r = 0; r < p.page; ++r) s = __fadd_rn(s, ld_f32(base + (int64_t)r * p.st + d));
    out[d] = st_elem<T>(__fdiv_rn(s, n_rows));
  }
}

struct ScoreParams {
  const char* q;
  int64_t q_sb, q_sh, q_st;   // element strides of q (B, H, T_q, D)
  const char* kmin;
  const char* kmax;
  int64_t ob, oh, op;         // element strides of kmin/kmax
  float* scores;              // (B, H_kv, T_q, P) contiguous fp32
  int32_t B, H, H_kv, T_q, D, P;
};

// grid (ceil(P / 4), B * H_kv * T_q); one warp per page.
template <typename T>
__global__ void __launch_bounds__(128) page_score_kernel(const ScoreParams p) {
  extern __shared__ float qg[];  // D floats: the rounded GQA-mean query
  const int row = blockIdx.y;
  const int t = row % p.T_q;
  const int bh = row / p.T_q;
  const int b = bh / p.H_kv, h = bh % p.H_kv;
  const int G = p.H / p.H_kv;
  for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
    float s = 0.f;
    for (int g = 0; g < G; ++g)
      s += ld_f32(reinterpret_cast<const T*>(p.q) + b * p.q_sb + (int64_t)(h * G + g) * p.q_sh +
                  (int64_t)t * p.q_st + d);
    // mean in fp32, then one rounding to the query dtype (identity for fp32)
    qg[d] = (G == 1) ? s : ld_f32_round<T>(s / (float)G);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pg = blockIdx.x * 4 + warp;
  if (pg >= p.P) return;
  const T* mn = reinterpret_cast<const T*>(p.kmin) + b * p.ob + h * p.oh + (int64_t)pg * p.op;
  const T* mx = reinterpret_cast<const T*>(p.kmax) + b * p.ob + h * p.oh + (int64_t)pg * p.op;
  float acc = 0.f;
  for (int d = lane; d < p.D; d += 32) {
    const float q = qg[d];
    acc += fmaxf(q * ld_f32(mn + d), q * ld_f32(mx + d));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) p.scores[(int64_t)row * p.P + pg] = acc;
}

// grid (ceil(P / 4), B * H_kv * T_q); one warp per page: q_g . K_mean.
template <typename T>
__global__ void __launch_bounds__(128) page_attn_kernel(const ScoreParams p) {
  extern __shared__ float qg[];
  const int row = blockIdx.y;
  const int t = row % p.T_q;
  const int bh = row / p.T_q;
  const int b = bh / p.H_kv, h = bh % p.H_kv;
  const int G = p.H / p.H_kv;
  for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
    float s = 0.f;
    for (int g = 0; g < G; ++g)
      s += ld_f32(reinterpret_cast<const T*>(p.q) + b * p.q_sb + (int64_t)(h * G + g) * p.q_sh +
                  (int64_t)t * p.q_st + d);
    qg[d] = (G == 1) ? s : ld_f32_round<T>(s / (float)G);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pg = blockIdx.x * 4 + warp;
  if (pg >= p.P) return;
  const T* km = reinterpret_cast<const T*>(p.kmin) + b * p.ob + h * p.oh + (int64_t)pg * p.op;
  float acc = 0.f;
  for (int d = lane; d < p.D; d += 32) acc = fmaf(qg[d], ld_f32(km + d), acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) p.scores[(int64_t)row * p.P + pg] = acc;
}

struct TopkParams {
  const float* scores;        // (R, P) rows to max over
  const uint8_t* exclude;     // (P,) nonzero = never select, or NULL
  float* per_page;            // (P,) out, or NULL
  int64_t* topk;              // (k,) out
  int32_t R, P, k;
};

// Order-preserving float -> uint32 key (larger float -> larger key).
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One CTA: per-page max over rows, then a descending bitonic sort of
// (score key, inverted page index) pairs; the first k indices win.
__global__ void __launch_bounds__(1024) page_topk_kernel(const TopkParams p, int n_pow2) {
  extern __shared__ unsigned long long keys[];
  for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
    unsigned long long kv = 0ull;  // padding sorts last
    if (i < p.P) {
      float m = -INFINITY;
      for (int r = 0; r < p.R; ++r) m = fmaxf(m, p.scores[(int64_t)r * p.P + i]);
      if (p.per_page) p.per_page[i] = m;
      if (p.exclude && p.exclude[i]) m = -INFINITY;
      kv = ((unsigned long long)fkey(m) << 32) | (0xFFFFFFFFu - (uint32_t)i);
    }
    keys[i] = kv;
  }
  __syncthreads();
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long a = keys[i], c = keys[j];
          if ((a < c) == desc) {
            keys[i] = c;
            keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < p.k; i += blockDim.x)
    p.topk[i] = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[i] & 0xFFFFFFFFull));
}

struct PressParams {
  const float* scores;        // (R, P) q_g . K_mean
  float* per_page;            // (P,) final score out, or NULL
  int64_t* topk;              // (k,) out
  int32_t R, P, k;
  float alpha, beta, gamma;
  int32_t window;             // recency window (>= 1)
  int32_t n_sink;             // sink pages
};

// CTA-wide reduction of one value per thread through `red` (blockDim / 32
// floats); every thread returns the result.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? fmaxf(v, w) : v + w;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) r = kMax ? fmaxf(r, red[i]) : r + red[i];
  return r;
}

// One CTA: the closed-form HALOPress page score and its top-k.
__global__ void __launch_bounds__(1024) press_topk_kernel(const PressParams p, int n_pow2) {
  extern __shared__ unsigned long long keys[];
  float* vals = reinterpret_cast<float*>(keys + n_pow2);   // (n_pow2,) attention proxy
  __shared__ float red[32];
  // attention proxy per page: max over rows
  float lmin = INFINITY, lmax = -INFINITY;
  for (int i = threadIdx.x; i < p.P; i += blockDim.x) {
    float m = -INFINITY;
    for (int r = 0; r < p.R; ++r) m = fmaxf(m, p.scores[(int64_t)r * p.P + i]);
    vals[i] = m;
    lmin = fminf(lmin, m);
  }
  const float mn = -block_reduce<true>(-lmin, red);
  for (int i = threadIdx.x; i < p.P; i += blockDim.x) {
    vals[i] = __fsub_rn(vals[i], mn);
    lmax = fmaxf(lmax, vals[i]);
  }
  const float mx = block_reduce<true>(lmax, red);
  // recency: exp(-(P - 1 - i) / window), normalised by its sum, then its max
  const float win = (float)p.window;
  float lsum = 0.f;
  for (int i = threadIdx.x; i < p.P; i += blockDim.x)
    lsum += expf(__fdiv_rn(-__fsub_rn((float)(p.P - 1), (float)i), win));
  const float rsum = block_reduce<false>(lsum, red);
  const float rden = __fadd_rn(rsum, 1e-12f);
  // the largest recency term is page P - 1's: exp(0) / rden
  const float rmax = __fadd_rn(__fdiv_rn(1.f, rden), 1e-12f);
  for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
    unsigned long long kv = 0ull;  // padding sorts last
    if (i < p.P) {
      const float attn = (mx > 0.f) ? __fdiv_rn(vals[i], mx) : vals[i];
      float rec = expf(__fdiv_rn(-__fsub_rn((float)(p.P - 1), (float)i), win));
      rec = __fdiv_rn(__fdiv_rn(rec, rden), rmax);
      const float sink = (i < p.n_sink) ? 1.f : 0.f;
      const float sc = __fadd_rn(__fadd_rn(__fmul_rn(p.alpha, attn), __fmul_rn(p.beta, rec)),
                                 __fmul_rn(p.gamma, sink));
      if (p.per_page) p.per_page[i] = sc;
      kv = ((unsigned long long)fkey(sc) << 32) | (0xFFFFFFFFu - (uint32_t)i);
    }
    keys[i] = kv;
  }
  __syncthreads();
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long a = keys[i], c = keys[j];
          if ((a < c) == desc) {
            keys[i] = c;
            keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < p.k; i += blockDim.x)
    p.topk[i] = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[i] & 0xFFFFFFFFull));
}

}  // namespace halo

using namespace halo;

static int scorer_elt(int dtype) {
  return dtype == HALO_DTYPE_F32 ? 4 : (dtype == HALO_DTYPE_BF16 || dtype == HALO_DTYPE_F16) ? 2 : 0;
}

extern "C" int32_t halo_page_summary(const void* k, int64_t k_sb, int64_t k_sh, int64_t k_st,
                                     int32_t B, int32_t H_kv, int32_t D, int32_t dtype,
                                     int32_t page_size, int32_t page_begin, int32_t n_pages,
                                     void* kmin, void* kmax, int64_t o_sb, int64_t o_sh,
                                     int64_t o_sp, halo_stream_t stream) {
  if (B <= 0 || H_kv <= 0 || D <= 0 || page_size <= 0 || page_begin < 0 || n_pages < 0)
    return fail(HALO_ERR_INVALID_ARG, "bad page-summary shape");
  if (!scorer_elt(dtype)) return fail(HALO_ERR_INVALID_ARG, "bad dtype %d", dtype);
  if (n_pages == 0) return HALO_OK;
  if (!k || !kmin || !kmax) return fail(HALO_ERR_INVALID_ARG, "NULL pointer");
  SummaryParams sp{static_cast<const char*>(k), k_sb, k_sh, k_st, static_cast<char*>(kmin),
                   static_cast<char*>(kmax), o_sb, o_sh, o_sp, H_kv, D, page_size, page_begin,
                   n_pages};
  dim3 grid((n_pages + 3) / 4, B * H_kv);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == HALO_DTYPE_BF16) page_summary_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(sp);
  else if (dtype == HALO_DTYPE_F16) page_summary_kernel<__half><<<grid, 128, 0, st>>>(sp);
  else page_summary_kernel<float><<<grid, 128, 0, st>>>(sp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "page_summary_kernel launch");
  count_launches();
  return HALO_OK;
}

extern "C" int32_t halo_page_score_topk(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                                        int32_t B, int32_t H, int32_t T_q, int32_t H_kv,
                                        int32_t D, int32_t dtype, const void* kmin,
                                        const void* kmax, int64_t o_sb, int64_t o_sh,
                                        int64_t o_sp, int32_t P, float* scores,
                                        const uint8_t* exclude, int32_t k, float* per_page,
                                        int64_t* topk, halo_stream_t stream) {
  if (B <= 0 || H <= 0 || T_q <= 0 || H_kv <= 0 || D <= 0 || P < 0 || k < 0 || k > P)
    return fail(HALO_ERR_INVALID_ARG, "bad page-score shape");
  if (H % H_kv) return fail(HALO_ERR_INVALID_ARG, "H=%d not divisible by H_kv=%d", H, H_kv);
  if (!scorer_elt(dtype)) return fail(HALO_ERR_INVALID_ARG, "bad dtype %d", dtype);
  if (P == 0) return HALO_OK;
  if (!q || !kmin || !kmax || !scores || (k > 0 && !topk))
    return fail(HALO_ERR_INVALID_ARG, "NULL pointer");
  int n_pow2 = 1;
  while (n_pow2 < P) n_pow2 <<= 1;
  if (k > 0 && n_pow2 > 16384)
    return fail(HALO_ERR_UNSUPPORTED, "top-k over %d pages (max 16384)", P);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ScoreParams sp{static_cast<const char*>(q), q_sb, q_sh, q_st, static_cast<const char*>(kmin),
                 static_cast<const char*>(kmax), o_sb, o_sh, o_sp, scores, B, H, H_kv, T_q, D, P};
  dim3 grid((P + 3) / 4, B * H_kv * T_q);
  const size_t smem = (size_t)D * sizeof(float);
  if (dtype == HALO_DTYPE_BF16) page_score_kernel<__nv_bfloat16><<<grid, 128, smem, st>>>(sp);
  else if (dtype == HALO_DTYPE_F16) page_score_kernel<__half><<<grid, 128, smem, st>>>(sp);
  else page_score_kernel<float><<<grid, 128, smem, st>>>(sp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "page_score_kernel launch");
  count_launches();
  if (k == 0 && !per_page) return HALO_OK;
  TopkParams tp{scores, exclude, per_page, topk, B * H_kv * T_q, P, k};
  const size_t tsmem = (size_t)n_pow2 * sizeof(unsigned long long);
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [] {
    cudaFuncSetAttribute(page_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 16384 * 8);
  });
  page_topk_kernel<<<1, 1024, tsmem, st>>>(tp, n_pow2);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "page_topk_kernel launch");
  count_launches();
  return HALO_OK;
}

extern "C" int32_t halo_page_mean(const void* k, int64_t k_sb, int64_t k_sh, int64_t k_st,
                                  int32_t B, int32_t H_kv, int32_t D, int32_t dtype,
                                  int32_t page_size, int32_t page_begin, int32_t n_pages,
                                  void* kmean, int64_t o_sb, int64_t o_sh, int64_t o_sp,
                                  halo_stream_t stream) {
  if (B <= 0 || H_kv <= 0 || D <= 0 || page_size <= 0 || page_begin < 0 || n_pages < 0)
    return fail(HALO_ERR_INVALID_ARG, "bad page-mean shape");
  if (!scorer_elt(dtype)) return fail(HALO_ERR_INVALID_ARG, "bad dtype %d", dtype);
  if (n_pages == 0) return HALO_OK;
  if (!k || !kmean) return fail(HALO_ERR_INVALID_ARG, "NULL pointer");
  SummaryParams sp{static_cast<const char*>(k), k_sb, k_sh, k_st, static_cast<char*>(kmean),
                   nullptr, o_sb, o_sh, o_sp, H_kv, D, page_size, page_begin, n_pages};
  dim3 grid((n_pages + 3) / 4, B * H_kv);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == HALO_DTYPE_BF16) page_mean_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(sp);
  else if (dtype == HALO_DTYPE_F16) page_mean_kernel<__half><<<grid, 128, 0, st>>>(sp);
  else page_mean_kernel<float><<<grid, 128, 0, st>>>(sp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "page_mean_kernel launch");
  count_launches();
  return HALO_OK;
}

extern "C" int32_t halo_page_press_topk(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                                        int32_t B, int32_t H, int32_t T_q, int32_t H_kv,
                                        int32_t D, int32_t dtype, const void* kmean,
                                        int64_t o_sb, int64_t o_sh, int64_t o_sp, int32_t P,
                                        float alpha, float beta, float gamma,
                                        int32_t refresh_window, int32_t n_sink_pages,
                                        float* scores, int32_t k, float* per_page,
                                        int64_t* topk, halo_stream_t stream) {
  if (B <= 0 || H <= 0 || T_q <= 0 || H_kv <= 0 || D <= 0 || P < 0 || k < 0 || k > P ||
      n_sink_pages < 0)
    return fail(HALO_ERR_INVALID_ARG, "bad press-score shape");
  if (H % H_kv) return fail(HALO_ERR_INVALID_ARG, "H=%d not divisible by H_kv=%d", H, H_kv);
  if (!scorer_elt(dtype)) return fail(HALO_ERR_INVALID_ARG, "bad dtype %d", dtype);
  if (P == 0) return HALO_OK;
  if (!q || !kmean || !scores || (k > 0 && !topk))
    return fail(HALO_ERR_INVALID_ARG, "NULL pointer");
  int n_pow2 = 1;
  while (n_pow2 < P) n_pow2 <<= 1;
  if (n_pow2 > 8192) return fail(HALO_ERR_UNSUPPORTED, "press score over %d pages (max 8192)", P);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ScoreParams sp{static_cast<const char*>(q), q_sb, q_sh, q_st, static_cast<const char*>(kmean),
                 nullptr, o_sb, o_sh, o_sp, scores, B, H, H_kv, T_q, D, P};
  dim3 grid((P + 3) / 4, B * H_kv * T_q);
  const size_t smem = (size_t)D * sizeof(float);
  if (dtype == HALO_DTYPE_BF16) page_attn_kernel<__nv_bfloat16><<<grid, 128, smem, st>>>(sp);
  else if (dtype == HALO_DTYPE_F16) page_attn_kernel<__half><<<grid, 128, smem, st>>>(sp);
  else page_attn_kernel<float><<<grid, 128, smem, st>>>(sp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "page_attn_kernel launch");
  count_launches();
  PressParams pp{scores, per_page, topk, B * H_kv * T_q, P, k, alpha, beta, gamma,
                 refresh_window < 1 ? 1 : refresh_window, n_sink_pages};
  const size_t psmem = (size_t)n_pow2 * (sizeof(unsigned long long) + sizeof(float));
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [] {
    cudaFuncSetAttribute(press_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         8192 * (sizeof(unsigned long long) + sizeof(float)));
  });
  press_topk_kernel<<<1, 1024, psmem, st>>>(pp, n_pow2);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "press_topk_kernel launch");
  count_launches();
  return HALO_OK;
}
