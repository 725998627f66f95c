// Row-wise log-sum-exp merge of P partial states (m, l, o), shared by the
// single-GPU merge (km_kernel) and the cross-GPU exchange merge (kx_kernel).
// One CTA of WARPS warps owns one output row; lane l owns the DPL
// consecutive columns [l*DPL, l*DPL + DPL).  Partial s of the row has score
// max mr[s*ps] (natural log), weight lr[s*ps] (lr NULL: 1) and output
// orow[s*ops + d].
#pragma once

#include "halo_common.cuh"

namespace halo {

// The row's P partials folded in as few memory round trips as possible:
// warp w takes partials s = w, w + WARPS, ...; a round loads ROUND of them
// (m, l and the lane's DPL columns of o) before using any, folds them into
// a running (max, sum, acc) rescaled when the max grows, and the warps'
// states are then combined through shared memory (s_m, s_l [WARPS],
// s_o [WARPS][DPL * 32]).  Every thread returns the row's M (natural log,
// -inf if no partial has a key), L = sum_s l_s e^{m_s - M} and, for its
// lane's columns d0 = lane * DPL ..., acc = sum_s e^{m_s - M} o_s.
// With P <= WARPS * ROUND the whole row takes one round trip.  A round
// holds ROUND * (DPL + 2) loaded values per thread: kMergeRound<DPL> keeps
// that within the merge kernels' 88-register budget for every row width.
template <int DPL>
constexpr int kMergeRound = DPL >= 8 ? 4 : 10;

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
