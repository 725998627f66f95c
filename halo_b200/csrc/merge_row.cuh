// Row-wise log-sum-exp merge of P partial states (m, l, o), shared by the
// single-GPU merge (km_kernel) and the cross-GPU exchange merge (kx_kernel).
// One CTA of WARPS warps owns one output row; lane l owns the DPL
// consecutive columns [l*DPL, l*DPL + DPL).  Partial s of the row has score
// max mr[s*ps], weight lr[s*ps] (lr NULL: 1) and output orow[s*ops + d].
#pragma once

#include "halo_common.cuh"

namespace halo {

// Max of mr[s*ps] over s < P, reduced over the CTA through s_red[WARPS].
template <int WARPS>
__device__ __forceinline__ float row_max(const float* mr, int64_t ps, int P, float* s_red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float M = -INFINITY;
  for (int s = threadIdx.x; s < P; s += WARPS * 32) M = fmaxf(M, mr[(int64_t)s * ps]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  if (lane == 0) s_red[warp] = M;
  __syncthreads();
  M = -INFINITY;
#pragma unroll
  for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_red[w]);
  return M;
}

// This warp's share (s = warp, warp + WARPS, ...) of sum_s l_s e^{m_s - M}
// and sum_s e^{m_s - M} o_s, INFLIGHT partials loaded before any is used so
// the row streams at memory bandwidth rather than latency.
// VEC: the o rows are 16-byte aligned (DPL == 4 loads one float4 per lane).
template <int DPL, int WARPS, int INFLIGHT, bool VEC>
__device__ __forceinline__ void fold_partials(const float* mr, const float* lr,
                                              const float* orow, int64_t ps, int64_t ops, int P,
                                              int Dv, float M, float& L, float (&acc)[DPL]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d0 = lane * DPL;
  const bool active = d0 < Dv;
  L = 0.f;
#pragma unroll
  for (int e = 0; e < DPL; ++e) acc[e] = 0.f;
  if (M == -INFINITY) return;
  int s = warp;
  for (; s + (INFLIGHT - 1) * WARPS < P; s += INFLIGHT * WARPS) {
    float ms[INFLIGHT], ls[INFLIGHT];
    float ov[INFLIGHT][DPL];
#pragma unroll
    for (int j = 0; j < INFLIGHT; ++j) {
      const int64_t sj = s + j * WARPS;
      ms[j] = mr[sj * ps];
      ls[j] = lr ? lr[sj * ps] : 1.f;
      if (active) {
        const float* src = orow + sj * ops + d0;
        if constexpr (VEC && DPL == 4) {
          const float4 v = *reinterpret_cast<const float4*>(src);
          ov[j][0] = v.x; ov[j][1] = v.y; ov[j][2] = v.z; ov[j][3] = v.w;
        } else {
#pragma unroll
          for (int e = 0; e < DPL; ++e) ov[j][e] = src[e];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < INFLIGHT; ++j) {
      const float w = (ms[j] == -INFINITY) ? 0.f : expf(ms[j] - M);
      L = fmaf(ls[j], w, L);
      if (active)
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[e] = fmaf(ov[j][e], w, acc[e]);
    }
  }
  for (; s < P; s += WARPS) {
    const float ms = mr[(int64_t)s * ps];
    if (ms == -INFINITY) continue;
    const float w = expf(ms - M);
    L = fmaf(lr ? lr[(int64_t)s * ps] : 1.f, w, L);
    if (active) {
      const float* src = orow + (int64_t)s * ops + d0;
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc[e] = fmaf(src[e], w, acc[e]);
    }
  }
}

// The row's P partials folded in as few memory round trips as possible:
// warp w takes partials s = w, w + WARPS, ...; a round loads ROUND of them
// (m, l and the lane's DPL columns of o) before using any, folds them into
// a running (max, sum, acc) rescaled when the max grows, and the warps'
// states are then combined through shared memory (s_m, s_l [WARPS],
// s_o [WARPS][DPL * 32]).  Every thread returns the row's M (natural log,
// -inf if no partial has a key), L = sum_s l_s e^{m_s - M} and, for its
// lane's columns d0 = lane * DPL ..., acc = sum_s e^{m_s - M} o_s.
// With P <= WARPS * ROUND the whole row takes one round trip.
template <int DPL, int WARPS, int ROUND, bool VEC>
__device__ __forceinline__ void merge_partials(const float* mr, const float* lr, const float* orow,
                                               int64_t ps, int64_t ops, int P, int Dv,
                                               float* s_m, float* s_l, float (*s_o)[DPL * 32],
                                               float& M, float& L, float (&acc)[DPL]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d0 = lane * DPL;
  const bool active = d0 < Dv;
  M = -INFINITY;
  L = 0.f;
#pragma unroll
  for (int e = 0; e < DPL; ++e) acc[e] = 0.f;
  for (int base = warp; base < P; base += WARPS * ROUND) {
    float ms[ROUND], ls[ROUND], ov[ROUND][DPL];
#pragma unroll
    for (int u = 0; u < ROUND; ++u) {
      const int s = base + u * WARPS;
      if (s < P) {
        ms[u] = mr[(int64_t)s * ps];
        ls[u] = lr ? lr[(int64_t)s * ps] : 1.f;
        const float* src = orow + (int64_t)s * ops + d0;
        if (active) {
          if constexpr (VEC && DPL == 4) {
            const float4 v = *reinterpret_cast<const float4*>(src);
            ov[u][0] = v.x;
            ov[u][1] = v.y;
            ov[u][2] = v.z;
            ov[u][3] = v.w;
          } else {
#pragma unroll
            for (int e = 0; e < DPL; ++e) ov[u][e] = src[e];
          }
        } else {
#pragma unroll
          for (int e = 0; e < DPL; ++e) ov[u][e] = 0.f;
        }
      } else {
        ms[u] = -INFINITY;
        ls[u] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) ov[u][e] = 0.f;
      }
    }
    float Mc = M;
#pragma unroll
    for (int u = 0; u < ROUND; ++u) Mc = fmaxf(Mc, ms[u]);
    if (Mc == -INFINITY) continue;
    const float a = (M == -INFINITY) ? 0.f : expf(M - Mc);
    L *= a;
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[e] *= a;
#pragma unroll
    for (int u = 0; u < ROUND; ++u) {
      const float w = (ms[u] == -INFINITY) ? 0.f : expf(ms[u] - Mc);
      L = fmaf(ls[u], w, L);
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc[e] = fmaf(ov[u][e], w, acc[e]);
    }
    M = Mc;
  }
  if (lane == 0) {
    s_m[warp] = M;
    s_l[warp] = L;
  }
#pragma unroll
  for (int e = 0; e < DPL; ++e) s_o[warp][d0 + e] = acc[e];
  __syncthreads();
  M = -INFINITY;
#pragma unroll
  for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s_m[w]);
  L = 0.f;
#pragma unroll
  for (int e = 0; e < DPL; ++e) acc[e] = 0.f;
  if (M == -INFINITY) return;
#pragma unroll
  for (int w = 0; w < WARPS; ++w) {
    const float wt = (s_m[w] == -INFINITY) ? 0.f : expf(s_m[w] - M);
    L = fmaf(s_l[w], wt, L);
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[e] = fmaf(s_o[w][d0 + e], wt, acc[e]);
  }
}

}  // namespace halo
