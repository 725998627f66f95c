// Chunked-prefill attention on the Blackwell tensor cores (tcgen05 + TMEM).
//
// T_q > 1 query rows of one (batch, head) slice attend to a list of K/V
// chunks (the accumulated cache of halo/kv_cache_chunked.py:873-942 and the
// slices of halo/chunked_prefill.py:73-135 in lzbaclz/HALO) with an online
// softmax; there is no split over keys, so results leave a CTA merged.  The
// kernel (kp2_kernel below) gives each CTA two 128-row query tiles of one
// q-head; its layout, warp roles and synchronisation are described at the
// kernel.
//
// Numerics: scores and outputs accumulate in fp32 (TMEM).  P = exp2(s*c - m)
// with a running max m that is only moved when it grows by more than 2^8
// (O is then rescaled in TMEM), so P <= 256.  bf16 inputs feed P to the
// tensor core as hi + lo 16-bit parts (two MMAs; ~16 significant bits): a
// single bf16 P puts errors up to ~2^-9 |v| on peaked rows, above the 2e-3
// budget.  fp16 inputs use one fp16 P (11 bits, |err| <~ 2^-12 |v|).
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "halo_common.cuh"
#include "umma.cuh"

namespace halo {

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
int device_sms();

namespace prefill {

constexpr int kBM = 128;            // query rows per CTA (TMEM lanes)
constexpr int kBN = 128;            // keys per tile
constexpr int kMaxSegs = 48;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.f;

struct Seg {
  int64_t start;   // global position of row 0
  int32_t len;
  int16_t causal;
  int16_t bcast;   // batch stride 0: every batch row reads batch 0
};

struct alignas(64) Params {
  CUtensorMap qmap;                 // {D, T_q, H, B}
  CUtensorMap kmap[kMaxSegs];       // {D, len, H_kv, B}
  CUtensorMap vmap[kMaxSegs];
  Seg seg[kMaxSegs];
  int32_t n_seg;
  int32_t B, H, G, T_q, n_qtiles;
  int64_t q_pos0;
  float scale_log2;                 // softmax scale * log2(e)
  int32_t mode;                     // HALO_MERGE_*
  int32_t out_dtype;
  char* out;
  int64_t out_sb, out_sh, out_st;   // elements
  float* lse;
  float* m;
  float* l;
  float* o;
  unsigned int* err;
};

// exp2 on the special-function unit (relative error ~2^-22).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// K/V tiles of segment `sg` visible to query positions <= qmax.
__device__ __forceinline__ int seg_tiles(const Seg& sg, int64_t qmax) {
  int n = (sg.len + kBN - 1) / kBN;
  if (sg.causal) {
    const int64_t lim = qmax - sg.start;   // last visible row
    if (lim < 0) return 0;
    const int64_t nv = lim / kBN + 1;
    if (nv < n) n = (int)nv;
  }
  return n;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  return Elem<T>::pack(a, b);
}

// ======================================================================
// kp2_kernel: two query tiles per CTA, double-buffered 64-key score tiles.
//
// CTA = query tiles A = 2*pair and B = 2*pair + 1 (B may be absent) of one
// q-head; both walk the same K/V tiles (B's causal range; A joins the tiles
// it can see).  K/V arrive as 128-key TMA tiles; scores are computed per
// 64-key sub-tile j (half j%2 of K/V tile j/2).  384 threads:
//   WG0  warp 0 TMA producer; warp 1 TMEM owner and MMA issuer of tile A
//        (lane 0); warp 2 MMA issuer of tile B; warp 3 idle.  Registers
//        lowered to 104 per thread.
//   WG1  softmax of tile A (thread r = TMEM lane r), 200 registers.
//   WG2  softmax of tile B, 200 registers.
// TMEM (512 columns): tile X has two 64-column score buffers S_X[0..1] and a
// D-column output accumulator O_X: S_A[b] = [64b, 64b+64), S_B[b] =
// [128+64b, ...), O_A = [256, 256+D), O_B = [256+D, 256+2D).  P of sub-tile
// j overwrites S_X[j%2] in place as 16-bit pairs (keys 32c..32c+31: hi in
// columns [32c, 32c+16), lo in [32c+16, 32c+32)) and is the A operand of
// O_X += P V (tcgen05.mma with A in TMEM).  With two score buffers the MMA
// issuer computes S_X(j+1) while the softmax of S_X(j) runs; S_X(j+2) waits
// for O_X += P_X(j) V to finish reading P.  A softmax that must rescale O_X
// first waits for the previous PV_X.
// Each tile's issuer runs PV(j), QK(j+2), PV(j+1), QK(j+3), ... on its own
// commit chain; the two chains interleave on the tensor pipe.
// Descriptors are precomputed (one add per MMA) so an issuing thread keeps
// pace with the pipe.
// Barriers: q_full; k_full/v_full/k_empty/v_empty [stages]; per tile X and
// buffer b: s_full (commit after QK), p_full (128 softmax arrivals), pv_done
// (commit after PV); mma_done per issuer.  K/V empty barriers take one
// arrival per issuer (the producer stands in for an issuer whose tile sits
// that K/V tile out).  All waits bounded.
constexpr int kThreads2 = 384;
constexpr int kSub = 64;                 // keys per score sub-tile

template <int D>
struct Geom2 {
  static constexpr int kBlocks = D / 64;
  static constexpr int kBlockBytes = kBM * 128;
  static constexpr int kTileBytes = kBlocks * kBlockBytes;
  static constexpr int kStages = D == 64 ? 4 : 2;
  static constexpr int kOffQ = 0;                         // Q_A, Q_B
  static constexpr int kOffK = 2 * kTileBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffBar = kOffV + kStages * kTileBytes;
  static constexpr int kSmemBytes = kOffBar + 512 + 1024;
  static constexpr uint32_t kColO = 256;
};

struct Bars2 {
  uint64_t q_full;
  uint64_t k_full[4], v_full[4], k_empty[4], v_empty[4];
  uint64_t s_full[2][2], p_full[2][2], pv_done[2][2], mma_done[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ bool wait_bar2(uint64_t* bar, uint32_t parity, Bars2* bs,
                                          unsigned int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile int*>(&bs->abort_flag)) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_device_error(err, static_cast<unsigned int>(-HALO_ERR_TIMEOUT));
      *reinterpret_cast<volatile int*>(&bs->abort_flag) = 1;
      return false;
    }
  }
}

// Sub-tile walk shared by every role: K/V tile index g (within segment s,
// tile t of that segment) and which query tiles take part.
struct Walk {
  int s, t, g;          // segment, tile in segment, global K/V tile
  int ntU, ntA;         // tiles of segment s for the union / tile A
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads2, 1) kp2_kernel(const __grid_constant__ Params p) {
  using Gm = Geom2<D>;
  constexpr int ST = Gm::kStages;
  // bf16 keeps P as hi + lo (two MMAs); fp16's 11-bit P alone keeps the
  // output within the error budget (|err| <~ 2^-12 |v|), so one MMA.
  constexpr bool kSplitP = Elem<T>::kDtype == HALO_DTYPE_BF16;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars2* bs = reinterpret_cast<Bars2*>(smem + Gm::kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int BH = p.B * p.H;
  const int n_pairs = (p.n_qtiles + 1) / 2;
  const int pair = n_pairs - 1 - (int)(blockIdx.x / BH);   // heavy first
  const int bh = (int)(blockIdx.x % BH);
  const int b = bh / p.H, h = bh % p.H, hk = h / p.G;
  const int qA0 = 2 * pair * kBM;
  const bool hasB = 2 * pair + 1 < p.n_qtiles;
  const int validA = min(kBM, p.T_q - qA0);
  const int validB = hasB ? min(kBM, p.T_q - (qA0 + kBM)) : 0;
  const int64_t qminA = p.q_pos0 + qA0, qmaxA = qminA + validA - 1;
  const int64_t qminB = qminA + kBM, qmaxB = qminB + validB - 1;
  const int64_t qmaxU = hasB ? qmaxB : qmaxA;

  if (threadIdx.x == 0) {
    mbar_init(&bs->q_full, 1);
    for (int i = 0; i < ST; ++i) {
      mbar_init(&bs->k_full[i], 1);
      mbar_init(&bs->v_full[i], 1);
      mbar_init(&bs->k_empty[i], 2);
      mbar_init(&bs->v_empty[i], 2);
    }
    for (int x = 0; x < 2; ++x) {
      for (int k = 0; k < 2; ++k) {
        mbar_init(&bs->s_full[x][k], 1);
        mbar_init(&bs->p_full[x][k], kBM);
        mbar_init(&bs->pv_done[x][k], 1);
      }
      mbar_init(&bs->mma_done[x], 1);
    }
    bs->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    umma::tmem_alloc(&bs->tmem_base, kTmemCols);
    umma::tmem_relinquish();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = bs->tmem_base;

  // K/V tiles of the union walk and tile A's share of them
  int nU = 0, nA = 0;
  for (int s = 0; s < p.n_seg; ++s) {
    nU += seg_tiles(p.seg[s], qmaxU);
    nA += seg_tiles(p.seg[s], qmaxA);
  }

  const uint32_t sQ = smem_addr(smem + Gm::kOffQ);
  const uint32_t sK = smem_addr(smem + Gm::kOffK);
  const uint32_t sV = smem_addr(smem + Gm::kOffV);

  // Register split (128 x 104 + 256 x 200 = 384 x 168, the launch budget),
  // made inside each role's branch so the compiler sizes each role's code
  // for its own budget.
  if (warp < 4) {
    umma::regs_dec<104>();
    if (warp == 0) {
      // ---------------------------------------------------------- producer
      if (lane == 0 && nU > 0) {
        mbar_arrive_expect_tx(&bs->q_full, (hasB ? 2 : 1) * Gm::kTileBytes);
        for (int x = 0; x < (hasB ? 2 : 1); ++x)
          for (int blk = 0; blk < Gm::kBlocks; ++blk)
            tma_load_4d(smem + Gm::kOffQ + x * Gm::kTileBytes + blk * Gm::kBlockBytes, &p.qmap,
                        blk * 64, qA0 + x * kBM, h, b, &bs->q_full);
        int nk = 0, nv = 0;
        bool ok = true;
        for (int s = 0; s < p.n_seg && ok; ++s) {
          const int nt = seg_tiles(p.seg[s], qmaxU);
          const int ntA = seg_tiles(p.seg[s], qmaxA);
          const int bb = p.seg[s].bcast ? 0 : b;
          for (int t = 0; t < nt; ++t) {
            // the empty barriers take one arrival per issuer; the issuer of a
            // tile that sits this K/V tile out is arrived for here
            const uint32_t absent = (t < ntA ? 0u : 1u) + (hasB ? 0u : 1u);
            const int st = nk % ST, use = nk / ST;
            if (use > 0 && !(ok = wait_bar2(&bs->k_empty[st], (use - 1) & 1, bs, p.err))) break;
            mbar_arrive_expect_tx(&bs->k_full[st], Gm::kTileBytes);
            for (int blk = 0; blk < Gm::kBlocks; ++blk)
              tma_load_4d(smem + Gm::kOffK + st * Gm::kTileBytes + blk * Gm::kBlockBytes,
                          &p.kmap[s], blk * 64, t * kBN, hk, bb, &bs->k_full[st]);
            if (absent) mbar_arrive_n(&bs->k_empty[st], absent);
            ++nk;
            if (use > 0 && !(ok = wait_bar2(&bs->v_empty[st], (use - 1) & 1, bs, p.err))) break;
            mbar_arrive_expect_tx(&bs->v_full[st], Gm::kTileBytes);
            for (int blk = 0; blk < Gm::kBlocks; ++blk)
              tma_load_4d(smem + Gm::kOffV + st * Gm::kTileBytes + blk * Gm::kBlockBytes,
                          &p.vmap[s], blk * 64, t * kBN, hk, bb, &bs->v_full[st]);
            if (absent) mbar_arrive_n(&bs->v_empty[st], absent);
            ++nv;
          }
        }
        // let every issued copy land before the CTA can exit
        mbar_wait(&bs->q_full, 0, p.err);
        for (int st = 0; st < ST; ++st) {
          const int uk = (nk - st + ST - 1) / ST, uv = (nv - st + ST - 1) / ST;
          if (uk > 0) mbar_wait(&bs->k_full[st], (uk - 1) & 1, p.err);
          if (uv > 0) mbar_wait(&bs->v_full[st], (uv - 1) & 1, p.err);
        }
      }
    } else if ((warp == 1 || (warp == 2 && hasB)) && lane == 0 && nU > 0) {
      // ---------------------------------------------------------- MMA issuers
      // warp 1 issues tile A's MMAs, warp 2 tile B's: two independent
      // commit chains, so one tile's waits never idle the other's work.
      // Both walk every K/V tile: they wait on its full barriers (keeping
      // the phase parity in step) and commit to its empty barriers when
      // they read it; the producer arrives for an issuer that sits it out.
      const int x = warp - 1;
      constexpr bool kBf16 = Elem<T>::kDtype == HALO_DTYPE_BF16;
      constexpr uint32_t kIdQK = umma::instr_desc_f16(kBM, kSub, kBf16, false, false);
      constexpr uint32_t kIdPV = umma::instr_desc_f16(kBM, D, kBf16, false, true);
      const uint64_t qdesc = umma::smem_desc_sw128(sQ + x * Gm::kTileBytes, 16, 1024);
      const uint64_t kdesc0 = umma::smem_desc_sw128(sK, 16, 1024);
      const uint64_t vdesc0 = umma::smem_desc_sw128(sV, Gm::kBlockBytes, 1024);
      const uint32_t scol0 = tmem + x * 128;
      const uint32_t ocol = tmem + Gm::kColO + x * D;
      bool ok = wait_bar2(&bs->q_full, 0, bs, p.err);
      // Two cursors walk the K/V tiles: QK runs two sub-tiles ahead of PV
      // (QK(j+2) is issued right after PV(j), whose completion frees the
      // score buffer it reuses), so the softmax of S(j+1) overlaps PV(j)
      // and QK(j+2).  Tiles this tile sits out are only waited on.
      struct Cursor {
        int s, t, g, ntU, ntA;
      };
      auto load = [&](Cursor& c) {
        while (c.s < p.n_seg) {
          c.ntU = seg_tiles(p.seg[c.s], qmaxU);
          c.ntA = seg_tiles(p.seg[c.s], qmaxA);
          if (c.t < c.ntU) return;
          ++c.s;
          c.t = 0;
        }
      };
      auto next = [&](Cursor& c) {
        ++c.t;
        ++c.g;
        if (c.t >= c.ntU) {
          ++c.s;
          c.t = 0;
          load(c);
        }
      };
      auto takes_part = [&](const Cursor& c) { return x ? hasB : (c.t < c.ntA); };
      Cursor cq{0, 0, 0, 0, 0}, cp{0, 0, 0, 0, 0};
      load(cq);
      load(cp);
      int jq = 0, jp = 0, hq = 0, hp = 0;
      // K side: skip tiles this tile sits out, then QK of the next sub-tile
      auto qk_step = [&]() -> int {   // 1 issued, 0 walk finished, -1 error
        while (cq.s < p.n_seg && !takes_part(cq)) {
          const int st = cq.g % ST;
          if (!wait_bar2(&bs->k_full[st], (cq.g / ST) & 1, bs, p.err)) return -1;
          next(cq);
        }
        if (cq.s >= p.n_seg) return 0;
        const int st = cq.g % ST;
        if (hq == 0 && !wait_bar2(&bs->k_full[st], (cq.g / ST) & 1, bs, p.err)) return -1;
        const int j = jq, bf = j & 1;
        if (j >= 2 && !wait_bar2(&bs->pv_done[x][bf], ((j - 2) >> 1) & 1, bs, p.err)) return -1;
        umma::fence_after_sync();
        const uint64_t kd = kdesc0 + (uint64_t)((st * Gm::kTileBytes + hq * kSub * 128) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * Gm::kBlockBytes + (kk & 3) * 32) >> 4;
          umma::mma_ss(scol0 + bf * kSub, qdesc + off, kd + off, kIdQK, kk > 0);
        }
        umma::commit(&bs->s_full[x][bf]);
        ++jq;
        if (hq == 1) {
          umma::commit(&bs->k_empty[st]);
          next(cq);
          hq = 0;
        } else {
          hq = 1;
        }
        return 1;
      };
      // V side: skip tiles this tile sits out, then PV of the next sub-tile
      auto pv_step = [&]() -> bool {
        while (!takes_part(cp)) {
          const int st = cp.g % ST;
          if (!wait_bar2(&bs->v_full[st], (cp.g / ST) & 1, bs, p.err)) return false;
          next(cp);
        }
        const int st = cp.g % ST;
        if (hp == 0 && !wait_bar2(&bs->v_full[st], (cp.g / ST) & 1, bs, p.err)) return false;
        const int j = jp, bf = j & 1;
        if (!wait_bar2(&bs->p_full[x][bf], (j >> 1) & 1, bs, p.err)) return false;
        umma::fence_after_sync();
        const uint32_t pcol = scol0 + bf * kSub;
        const uint64_t vd = vdesc0 + (uint64_t)((st * Gm::kTileBytes + hp * kSub * 128) >> 4);
#pragma unroll
        for (int part = 0; part < (kSplitP ? 2 : 1); ++part)
#pragma unroll
          for (int kk = 0; kk < kSub / 16; ++kk)
            umma::mma_ts(ocol, pcol + (kk >> 1) * 32 + part * 16 + (kk & 1) * 8,
                         vd + (uint64_t)((kk * 16 * 128) >> 4), kIdPV, (j > 0) || part || kk);
        umma::commit(&bs->pv_done[x][bf]);
        ++jp;
        if (hp == 1) {
          umma::commit(&bs->v_empty[st]);
          next(cp);
          hp = 0;
        } else {
          hp = 1;
        }
        return true;
      };
      // Offset tile B by one softmax: its chain starts once tile A's first P
      // is out, so the two softmax warpgroups alternate with the MMAs
      // instead of competing at the same moments.
      if (x == 1 && ok && p.seg[0].len > 0 && seg_tiles(p.seg[0], qmaxA) > 0)
        ok = wait_bar2(&bs->p_full[0][0], 0, bs, p.err);
      int rq = ok ? qk_step() : -1;
      if (rq > 0) rq = qk_step();
      ok = rq >= 0;
      while (ok && jp < jq) {
        if (!(ok = pv_step())) break;
        if (rq > 0) {
          rq = qk_step();
          ok = rq >= 0;
        }
      }
      // this thread's MMAs complete before the CTA can free TMEM
      umma::commit(&bs->mma_done[x]);
      mbar_wait(&bs->mma_done[x], 0, p.err);
    }
  } else {
    umma::regs_inc<200>();
    // ------------------------------------------------------------ softmax X
    const int x = (warp - 4) >> 2;              // 0: tile A, 1: tile B
    const int sub = warp & 3;
    const int r = sub * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(sub * 32) << 16);
    const uint32_t ocol = Gm::kColO + x * D;
    const bool active = x == 0 || hasB;
    const int64_t qmin = x ? qminB : qminA;
    const int64_t qmaxX = x ? qmaxB : qmaxA;
    const int64_t qpos = qmin + r;
    int nX = 0;                                  // sub-tiles of tile X
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    int j = 0;
    for (int s = 0; s < p.n_seg && ok && active; ++s) {
      const Seg sg = p.seg[s];
      const int nt = seg_tiles(sg, qmaxX);
      for (int t = 0; t < nt * 2; ++t, ++j) {
        const int bf = j & 1;
        const uint32_t scol = x * 128 + bf * kSub;
        ok = __all_sync(0xffffffffu, wait_bar2(&bs->s_full[x][bf], (j >> 1) & 1, bs, p.err));
        if (!ok) break;
        umma::fence_after_sync();
        const int row0 = (t >> 1) * kBN + (t & 1) * kSub;
        const int64_t kpos0 = sg.start + row0;
        const bool full = (row0 + kSub <= sg.len) && (!sg.causal || kpos0 + kSub - 1 <= qmin);
        const int lim_len = sg.len - row0;
        const int64_t lim_pos = sg.causal ? qpos - kpos0 : (int64_t)kSub;
        // the sub-tile's 64 scores: two loads, one wait
        float sv[kSub];
        umma::tmem_ld32(trow + scol, sv);
        umma::tmem_ld32(trow + scol + 32, sv + 32);
        umma::tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int c = 0; c < kSub; ++c)
            if (!(c < lim_len && (int64_t)c <= lim_pos)) sv[c] = -INFINITY;
        }
        float mx8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx8[e] = sv[e];
#pragma unroll
        for (int c = 8; c < kSub; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) *
                         p.scale_log2;
        const bool grow = mx > m + kRescaleLog2 || (m == -INFINITY && mx > -INFINITY);
        float fac = 1.f;
        if (grow) {
          fac = (m == -INFINITY) ? 0.f : ex2(m - mx);
          l *= fac;
          m = mx;
        }
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
          // O_X must be quiescent: wait for O_X += P_X(j-1) V
          ok = __all_sync(0xffffffffu, wait_bar2(&bs->pv_done[x][bf ^ 1], ((j - 1) >> 1) & 1,
                                                  bs, p.err));
          if (!ok) break;
          umma::fence_after_sync();
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float ov[32];
            umma::tmem_ld32(trow + ocol + c * 32, ov);
            umma::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] *= fac;
            umma::tmem_st32(trow + ocol + c * 32, ov);
          }
        }
        // P = exp2(s * scale_log2 - m) as 16-bit pairs into S's columns
        const float nmu = (m == -INFINITY) ? 0.f : -m;
        const float sl2 = p.scale_log2;
        float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < kSub / 32; ++c) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = ex2(fmaf(sv[c * 32 + 2 * e], sl2, nmu));
            const float p1 = ex2(fmaf(sv[c * 32 + 2 * e + 1], sl2, nmu));
            rs4[e & 3] += p0 + p1;
            if constexpr (kSplitP) {
              // hi = p truncated to bf16 (upper halves, one byte permute
              // per pair), lo = rnd(p - hi): ~16 significant bits in all
              const uint32_t b0 = __float_as_uint(p0), b1 = __float_as_uint(p1);
              hi[e] = __byte_perm(b0, b1, 0x7632);
              lo[e] = pack2<T>(p0 - __uint_as_float(b0 & 0xFFFF0000u),
                               p1 - __uint_as_float(b1 & 0xFFFF0000u));
            } else {
              hi[e] = pack2<T>(p0, p1);
            }
          }
          umma::tmem_st16u(trow + scol + c * 32, hi);
          if constexpr (kSplitP) umma::tmem_st16u(trow + scol + c * 32 + 16, lo);
        }
        l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
        umma::tmem_wait_st();
        umma::fence_before_sync();
        mbar_arrive(&bs->p_full[x][bf]);
      }
    }
    nX = j;

    // ---- epilogue of tile X: thread r finalises query row q0 + r
    if (active && ok && nX > 0) {
      ok = __all_sync(0xffffffffu, wait_bar2(&bs->pv_done[x][(nX - 1) & 1], ((nX - 1) >> 1) & 1,
                                              bs, p.err));
      if (ok) umma::fence_after_sync();
    }
    const int validX = x ? validB : validA;
    if (active && ok) {
      const int t = qA0 + x * kBM + r;
      const bool live = r < validX;
      const int64_t row = ((int64_t)b * p.H + h) * p.T_q + t;
      float M = (m == -INFINITY) ? -INFINITY : m * kLn2;
      float L = l, wo = 1.f, wp = 0.f;
      const float* op = nullptr;
      if (live && p.m != nullptr) {
        const float mp = p.m[row], lp = p.l[row];
        const float Mn = fmaxf(M, mp);
        wo = (M == -INFINITY) ? 0.f : expf(M - Mn);
        wp = (mp == -INFINITY) ? 0.f : expf(mp - Mn);
        op = p.o + row * D;
        L = L * wo + lp * wp;
        M = Mn;
      }
      const float inv = (L > 0.f) ? 1.f / L : 0.f;
      if (live && p.mode != HALO_MERGE_ACCUMULATE && p.lse)
        p.lse[row] = (L > 0.f) ? M + logf(L) : -INFINITY;
      if (live && p.mode == HALO_MERGE_ACCUMULATE) {
        p.m[row] = M;
        p.l[row] = L;
      }
      const int64_t off = (int64_t)b * p.out_sb + (int64_t)h * p.out_sh + (int64_t)t * p.out_st;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float ov[32];
        if (nX > 0) {
          umma::tmem_ld32(trow + ocol + c * 32, ov);   // warp-collective: every lane
          umma::tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = 0.f;
        }
        if (!live) continue;
        if (op) {
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = ov[e] * wo + op[c * 32 + e] * wp;
        }
        if (p.mode == HALO_MERGE_ACCUMULATE) {
          float4* od = reinterpret_cast<float4*>(p.o + row * D + c * 32);
#pragma unroll
          for (int e = 0; e < 32; e += 4) od[e / 4] = make_float4(ov[e], ov[e + 1], ov[e + 2], ov[e + 3]);
        } else if (p.out_dtype == HALO_DTYPE_F32) {
          float4* od = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + off + c * 32);
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            od[e / 4] = make_float4(ov[e] * inv, ov[e + 1] * inv, ov[e + 2] * inv, ov[e + 3] * inv);
        } else {
          uint4* od = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + off + c * 32);
#pragma unroll
          for (int e = 0; e < 32; e += 8)
            od[e / 8] = make_uint4(pack2<T>(ov[e] * inv, ov[e + 1] * inv),
                                   pack2<T>(ov[e + 2] * inv, ov[e + 3] * inv),
                                   pack2<T>(ov[e + 4] * inv, ov[e + 5] * inv),
                                   pack2<T>(ov[e + 6] * inv, ov[e + 7] * inv));
        }
      }
    }
  }

  // ---- teardown: every TMEM access and MMA has completed
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace prefill

// ================================================================ host side
typedef CUresult (*PfEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                               const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                               const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                               CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PfEncodeFn pf_encode_fn() {
  static PfEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfEncodeFn>(ptr);
  });
  return fn;
}

struct PfMapKey {
  uintptr_t ptr;
  uint64_t dims[4];
  uint64_t strides[3];
  int dtype;
  bool operator==(const PfMapKey& o) const {
    return ptr == o.ptr && dtype == o.dtype && std::memcmp(dims, o.dims, sizeof(dims)) == 0 &&
           std::memcmp(strides, o.strides, sizeof(strides)) == 0;
  }
};
struct PfMapKeyHash {
  size_t operator()(const PfMapKey& k) const {
    uint64_t h = 1469598103934665603ull ^ k.ptr;
    auto mix = [&](uint64_t v) { h = (h ^ v) * 1099511628211ull; };
    for (int i = 0; i < 4; ++i) mix(k.dims[i]);
    for (int i = 0; i < 3; ++i) mix(k.strides[i]);
    mix(static_cast<uint64_t>(k.dtype));
    return static_cast<size_t>(h);
  }
};

// 4-D 16-bit tensor {D, rows, heads, batch} (byte strides of the outer three
// dims), box {64 elements, 128 rows, 1, 1}, 128-byte swizzle, out-of-bounds
// rows zero-filled.  Encodings are cached per (pointer, shape, strides).
static int pf_encode(const void* base, int dtype, const uint64_t dims[4],
                     const uint64_t strides[3], CUtensorMap* out) {
  PfMapKey key;
  key.ptr = reinterpret_cast<uintptr_t>(base);
  std::memcpy(key.dims, dims, sizeof(key.dims));
  std::memcpy(key.strides, strides, sizeof(key.strides));
  key.dtype = dtype;
  static std::mutex mu;
  static std::unordered_map<PfMapKey, CUtensorMap, PfMapKeyHash> cache;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return HALO_OK;
    }
  }
  PfEncodeFn fn = pf_encode_fn();
  if (!fn) return fail(HALO_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t gdim[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t gstr[3] = {strides[0], strides[1], strides[2]};
  cuuint32_t box[4] = {64, (cuuint32_t)prefill::kBN, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == HALO_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(out, dt, 4, const_cast<void*>(base), gdim, gstr, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(HALO_ERR_INVALID_ARG,
                "prefill tensor map encode failed (%d): dims {%llu,%llu,%llu,%llu} strides "
                "{%llu,%llu,%llu} bytes",
                (int)r, (unsigned long long)dims[0], (unsigned long long)dims[1],
                (unsigned long long)dims[2], (unsigned long long)dims[3],
                (unsigned long long)strides[0], (unsigned long long)strides[1],
                (unsigned long long)strides[2]);
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, *out);
  return HALO_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Chunk c continues segment s in memory and in position (one tensor map).
static bool pf_continues(const halo_kv_chunk_t& a, int64_t a_len, const halo_kv_chunk_t& c) {
  return c.causal == a.causal && c.k_stride_b == a.k_stride_b && c.k_stride_h == a.k_stride_h &&
         c.k_stride_t == a.k_stride_t && c.v_stride_b == a.v_stride_b &&
         c.v_stride_h == a.v_stride_h && c.v_stride_t == a.v_stride_t &&
         c.start == a.start + a_len &&
         static_cast<const char*>(c.k) ==
             static_cast<const char*>(a.k) + a_len * a.k_stride_t * 2 &&
         static_cast<const char*>(c.v) ==
             static_cast<const char*>(a.v) + a_len * a.v_stride_t * 2 &&
         a_len + c.len <= INT32_MAX;
}

template <typename T, int D>
static int launch_kp2(const prefill::Params& prm, int grid, cudaStream_t st) {
  using Gm = prefill::Geom2<D>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(prefill::kp2_kernel<T, D>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, Gm::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "kp2_kernel shared-memory attribute");
  prefill::kp2_kernel<T, D><<<grid, prefill::kThreads2, Gm::kSmemBytes, st>>>(prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kp2_kernel launch");
  count_launches();
  return HALO_OK;
}

// One coalesced run of chunks: the first chunk's pointers, strides, start
// and causal flag, its total length and whether the batch broadcasts.
struct PfSeg {
  halo_kv_chunk_t c;
  int64_t len;
  bool bcast;
};

// K/V tiles of a segment visible to query positions <= qmax (host copy of
// prefill::seg_tiles).
static int pf_seg_tiles(const PfSeg& sg, int64_t qmax) {
  int64_t n = (sg.len + prefill::kBN - 1) / prefill::kBN;
  if (sg.c.causal) {
    const int64_t lim = qmax - sg.c.start;
    if (lim < 0) return 0;
    n = std::min<int64_t>(n, lim / prefill::kBN + 1);
  }
  return (int)n;
}

// Whether every query-tile pair (A, B) of the call sees, along the union
// walk of its K/V tiles, at most one tile in a row that A sits out.  A run
// of two or more can stall A's MMA issuer: it waits for the K tile after the
// run while the producer, one ring stage later, waits for A's pending P V
// to free a V stage.  Within one segment A sits out at most the last tile
// (query tiles are 128 rows, K/V tiles 128 keys apart), so runs only form
// across segments.
static bool pf_order_ok(const PfSeg* segs, int n, int T_q, int64_t q_pos0) {
  const int n_qtiles = (T_q + prefill::kBM - 1) / prefill::kBM;
  for (int pair = 0; 2 * pair + 1 < n_qtiles; ++pair) {
    const int qA0 = 2 * pair * prefill::kBM;
    const int64_t qmaxA = q_pos0 + qA0 + prefill::kBM - 1;   // A is full when B exists
    const int validB = std::min(prefill::kBM, T_q - (qA0 + prefill::kBM));
    const int64_t qmaxB = q_pos0 + qA0 + prefill::kBM + validB - 1;
    int64_t run = 0;
    for (int i = 0; i < n; ++i) {
      const int ntU = pf_seg_tiles(segs[i], qmaxB), ntA = pf_seg_tiles(segs[i], qmaxA);
      run = (ntA > 0 ? 0 : run) + (ntU - ntA);
      if (run > 1) return false;
    }
  }
  return true;
}

}  // namespace halo

using namespace halo;

extern "C" int32_t halo_prefill_attention(const halo_prefill_problem_t* pb,
                                          const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                          const halo_prefill_out_t* po, halo_stream_t stream) {
  if (!pb || !po) return fail(HALO_ERR_INVALID_ARG, "problem/out is NULL");
  if (pb->B <= 0 || pb->H <= 0 || pb->H_kv <= 0 || pb->T_q < 0 || pb->D <= 0)
    return fail(HALO_ERR_INVALID_ARG, "non-positive dimension (B=%d H=%d H_kv=%d T_q=%d D=%d)",
                pb->B, pb->H, pb->H_kv, pb->T_q, pb->D);
  if (pb->H % pb->H_kv) return fail(HALO_ERR_INVALID_ARG, "H=%d not divisible by H_kv=%d", pb->H, pb->H_kv);
  if (pb->dtype != HALO_DTYPE_BF16 && pb->dtype != HALO_DTYPE_F16)
    return fail(HALO_ERR_UNSUPPORTED, "prefill kernel needs bf16 or fp16 (dtype %d)", pb->dtype);
  if (pb->D != 64 && pb->D != 128)
    return fail(HALO_ERR_UNSUPPORTED, "prefill kernel head_dim %d (64 or 128)", pb->D);
  if (!(pb->scale > 0.f) || !std::isfinite(pb->scale))
    return fail(HALO_ERR_UNSUPPORTED, "prefill kernel needs a positive finite scale");
  if (n_chunks < 0 || (n_chunks > 0 && !chunks)) return fail(HALO_ERR_INVALID_ARG, "bad chunk list");
  if (po->mode != HALO_MERGE_FINALIZE && po->mode != HALO_MERGE_ACCUMULATE)
    return fail(HALO_ERR_INVALID_ARG, "bad mode %d", po->mode);
  const bool have_state = po->m || po->l || po->o;
  if (have_state && !(po->m && po->l && po->o))
    return fail(HALO_ERR_INVALID_ARG, "running state needs all of m, l, o");
  if (po->mode == HALO_MERGE_ACCUMULATE && !have_state)
    return fail(HALO_ERR_INVALID_ARG, "accumulate needs m, l, o");
  if (po->o && !aligned16(po->o)) return fail(HALO_ERR_MISALIGNED, "o must be 16-byte aligned");
  const int D = pb->D;
  if (po->mode == HALO_MERGE_FINALIZE) {
    if (!po->out) return fail(HALO_ERR_INVALID_ARG, "out is NULL");
    const int oe = po->out_dtype == HALO_DTYPE_F32 ? 4 : 2;
    if (po->out_dtype != HALO_DTYPE_F32 && po->out_dtype != pb->dtype)
      return fail(HALO_ERR_UNSUPPORTED, "out dtype must be fp32 or the input dtype");
    if (!aligned16(po->out) || (po->out_stride_b * oe) % 16 || (po->out_stride_h * oe) % 16 ||
        (po->out_stride_t * oe) % 16)
      return fail(HALO_ERR_MISALIGNED, "out rows must be 16-byte aligned");
  }
  if (pb->T_q == 0) return HALO_OK;
  if (!pb->q || !aligned16(pb->q) || (pb->q_stride_t * 2) % 16 || (pb->q_stride_h * 2) % 16 ||
      (pb->B > 1 && (pb->q_stride_b * 2) % 16) || pb->q_stride_t <= 0 || pb->q_stride_h <= 0)
    return fail(HALO_ERR_MISALIGNED, "q must be 16-byte aligned with 16-byte row strides");

  // ---- segments: coalesce chunks contiguous in memory and position
  static thread_local prefill::Params prm;
  PfSeg segs[prefill::kMaxSegs];
  int n_seg = 0;
  halo_kv_chunk_t cur{};
  int64_t cur_len = 0;
  auto flush = [&]() -> int {
    if (cur_len == 0) return HALO_OK;
    if (n_seg >= prefill::kMaxSegs)
      return fail(HALO_ERR_UNSUPPORTED, "more than %d non-contiguous chunks in one call",
                  prefill::kMaxSegs);
    const bool bk = cur.k_stride_b == 0, bv = cur.v_stride_b == 0;
    if (bk != bv) return fail(HALO_ERR_INVALID_ARG, "k and v must both broadcast the batch or neither");
    segs[n_seg++] = PfSeg{cur, cur_len, bk};
    cur_len = 0;
    return HALO_OK;
  };
  for (int i = 0; i < n_chunks; ++i) {
    const halo_kv_chunk_t& c = chunks[i];
    if (c.len < 0) return fail(HALO_ERR_INVALID_ARG, "chunk %d: negative length", i);
    if (c.len == 0) continue;
    if (!c.k || !c.v) return fail(HALO_ERR_INVALID_ARG, "chunk %d: NULL k/v", i);
    if (!aligned16(c.k) || !aligned16(c.v) || (c.k_stride_t * 2) % 16 || (c.v_stride_t * 2) % 16 ||
        (c.k_stride_h * 2) % 16 || (c.v_stride_h * 2) % 16 || (c.k_stride_b * 2) % 16 ||
        (c.v_stride_b * 2) % 16 || c.k_stride_t <= 0 || c.v_stride_t <= 0)
      return fail(HALO_ERR_MISALIGNED, "chunk %d: k/v rows must be 16-byte aligned", i);
    if (cur_len > 0 && pf_continues(cur, cur_len, c)) {
      cur_len += c.len;
      continue;
    }
    int rc = flush();
    if (rc != HALO_OK) return rc;
    cur = c;
    cur_len = c.len;
  }
  int rc = flush();
  if (rc != HALO_OK) return rc;
  if (!pf_order_ok(segs, n_seg, pb->T_q, pb->q_pos0))
    return fail(HALO_ERR_SPLIT, "chunk order: a query tile would sit out two or more K/V tiles "
                "in a row; pass the chunks in smaller calls");
  for (int i = 0; i < n_seg; ++i) {
    const halo_kv_chunk_t& c = segs[i].c;
    const bool bk = segs[i].bcast;
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)segs[i].len, (uint64_t)pb->H_kv,
                              (uint64_t)(bk ? 1 : pb->B)};
    const uint64_t ks[3] = {(uint64_t)c.k_stride_t * 2, (uint64_t)c.k_stride_h * 2,
                            (uint64_t)(bk || pb->B == 1 ? c.k_stride_h * 2 * pb->H_kv
                                                        : c.k_stride_b * 2)};
    const uint64_t vs[3] = {(uint64_t)c.v_stride_t * 2, (uint64_t)c.v_stride_h * 2,
                            (uint64_t)(bk || pb->B == 1 ? c.v_stride_h * 2 * pb->H_kv
                                                        : c.v_stride_b * 2)};
    rc = pf_encode(c.k, pb->dtype, dims, ks, &prm.kmap[i]);
    if (rc != HALO_OK) return rc;
    rc = pf_encode(c.v, pb->dtype, dims, vs, &prm.vmap[i]);
    if (rc != HALO_OK) return rc;
    prm.seg[i].start = c.start;
    prm.seg[i].len = (int32_t)segs[i].len;
    prm.seg[i].causal = c.causal ? 1 : 0;
    prm.seg[i].bcast = bk ? 1 : 0;
  }

  // ---- Q map {D, T_q, H, B}
  {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)pb->T_q, (uint64_t)pb->H, (uint64_t)pb->B};
    const uint64_t qs[3] = {(uint64_t)pb->q_stride_t * 2, (uint64_t)pb->q_stride_h * 2,
                            (uint64_t)(pb->B > 1 ? pb->q_stride_b * 2
                                                 : pb->q_stride_h * 2 * pb->H)};
    rc = pf_encode(pb->q, pb->dtype, dims, qs, &prm.qmap);
    if (rc != HALO_OK) return rc;
  }
  prm.n_seg = n_seg;
  prm.B = pb->B;
  prm.H = pb->H;
  prm.G = pb->H / pb->H_kv;
  prm.T_q = pb->T_q;
  prm.n_qtiles = (pb->T_q + prefill::kBM - 1) / prefill::kBM;
  prm.q_pos0 = pb->q_pos0;
  prm.scale_log2 = pb->scale * kLog2e;
  prm.mode = po->mode;
  prm.out_dtype = po->out_dtype;
  prm.out = static_cast<char*>(po->out);
  prm.out_sb = po->out_stride_b;
  prm.out_sh = po->out_stride_h;
  prm.out_st = po->out_stride_t;
  prm.lse = po->lse;
  prm.m = po->m;
  prm.l = po->l;
  prm.o = po->o;
  prm.err = device_error_ptr();
  const int64_t grid = (int64_t)((prm.n_qtiles + 1) / 2) * pb->B * pb->H;
  if (grid > INT32_MAX) return fail(HALO_ERR_UNSUPPORTED, "grid too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pb->event_begin) cudaEventRecord(static_cast<cudaEvent_t>(pb->event_begin), st);
  if (pb->dtype == HALO_DTYPE_BF16)
    rc = D == 128 ? launch_kp2<__nv_bfloat16, 128>(prm, (int)grid, st)
                  : launch_kp2<__nv_bfloat16, 64>(prm, (int)grid, st);
  else
    rc = D == 128 ? launch_kp2<__half, 128>(prm, (int)grid, st)
                  : launch_kp2<__half, 64>(prm, (int)grid, st);
  if (rc == HALO_OK && pb->event_end) cudaEventRecord(static_cast<cudaEvent_t>(pb->event_end), st);
  return rc;
}
