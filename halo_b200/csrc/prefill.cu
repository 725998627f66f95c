// Chunked-prefill attention on the Blackwell tensor cores (tcgen05 + TMEM).
//
// T_q > 1 query rows of one (batch, head) slice attend to a list of K/V
// chunks (the accumulated cache of halo/kv_cache_chunked.py:873-942 and the
// slices of halo/chunked_prefill.py:73-135 in lzbaclz/HALO) with an online
// softmax; there is no split over keys, so results leave a CTA merged.  The
// kernel (kp3_kernel below) gives each CTA two 128-row query tiles of one
// q-head; its layout, warp roles and synchronisation are described at the
// kernel.
//
// Numerics: scores and outputs accumulate in fp32 (TMEM).  P = exp2(s*c - m)
// with a running max m that is only moved when it grows by more than 2^8
// (O is then rescaled in TMEM), so P <= 256.  P enters the P V product as
// one fp16 operand (11 significant bits, |err| <~ 2^-12 |v| per term) with V
// in fp16: fp16 inputs as they are, bf16 inputs through an fp16 copy of V
// that a pre-pass (v16_kernel) writes into the caller's workspace.  That
// copy is exact for 2^-14 <= |v| < 2^16 and loses at most 2^-25 in absolute
// terms below; a call whose V holds a finite |v| >= 2^16 is flagged by the
// pre-pass and runs the bf16 route instead: bf16 V and P as a truncated bf16
// high part plus a bf16 residual (two MMAs, ~16 significant bits).  A single
// bf16 P would put errors up to ~2^-9 |v| on peaked rows, above the 2e-3
// budget.  Calls without a workspace take the bf16 route.
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

constexpr int kBM = 128;            // query rows per tile (TMEM lanes)
constexpr int kBN = 128;            // keys per K/V tile and per score tile
constexpr int kMaxSegs = 48;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.f;
// split-unit partial row: o[D], M, L, 2 floats of padding (16-byte rows)
template <int D>
constexpr int kPartStride = D + 4;
constexpr int64_t kWsHeader = 256;  // workspace: flag word, then the fp16 V copies

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
  CUtensorMap v16map[kMaxSegs];     // fp16 copy of V (workspace), bf16 inputs only
  Seg seg[kMaxSegs];
  const unsigned int* v16_flag;     // non-NULL: fp16 copies exist; *flag != 0: out of range
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
  // Split units (the last partial wave): CTAs blockIdx >= n_full take half
  // of a unit's K/V walk each (2 CTAs per unit, first half then second) and
  // write their rows' fp32 (M, L, o) to part instead of out; pf_merge_kernel
  // folds the two halves.  n_full = all units and part = NULL: no split.
  int32_t n_full;
  float* part;
  unsigned int* err;
};

// Non-blocking probe of an mbarrier phase (true: the phase with this parity
// has completed).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Suspend in hardware (the warp issues nothing) until the phase with this
// parity completes or about `ns` nanoseconds pass; true when it completed.
__device__ __forceinline__ bool mbar_sleep_wait(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// K/V tiles of segment `sg` visible to query positions <= qmax.
__host__ __device__ __forceinline__ int seg_tiles(const Seg& sg, int64_t qmax) {
  int n = (sg.len + kBN - 1) / kBN;
  if (sg.causal) {
    const int64_t lim = qmax - sg.start;   // last visible row
    if (lim < 0) return 0;
    const int64_t nv = lim / kBN + 1;
    if (nv < n) n = (int)nv;
  }
  return n;
}

// The value itself, opaque to the compiler: keeps the issuer from hoisting
// every unrolled MMA's descriptor out of its polling loop into registers.
__device__ __forceinline__ uint64_t opaque(uint64_t v) {
  asm volatile("mov.b64 %0, %0;" : "+l"(v));
  return v;
}

// ---- packed fp32 pairs (sm_100 f32x2 instructions: two lanes per issue)
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two floats as one 32-bit register of two fp16 values (round to nearest).
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// P = exp2(s * scale_log2 - m) of one row's 128 scores into TMEM columns
// [col, col + 64) as fp16 pairs (kSplit = false), or as bf16 high parts
// there and bf16 residuals in [col + 64, col + 128) (kSplit = true); the
// fp32 row sum accumulates into rs2 (two pairs).
template <bool kSplit>
__device__ __forceinline__ void write_p(const float (&sv)[kBN], uint64_t sl2, uint64_t nm2,
                                        uint32_t col, uint64_t (&rs2)[2]) {
#pragma unroll
  for (int c = 0; c < kBN / 32; ++c) {
    uint32_t hv[16], lv[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      float x0, x1, p0, p1;
      f2unpack(ffma2(f2pack(sv[c * 32 + 2 * e], sv[c * 32 + 2 * e + 1]), sl2, nm2), x0, x1);
      p0 = ex2(x0);
      p1 = ex2(x1);
      rs2[e & 1] = fadd2(rs2[e & 1], f2pack(p0, p1));
      if constexpr (!kSplit) {
        hv[e] = pack_h2(p0, p1);
      } else {
        // hi = p truncated to bf16 (upper halves, one byte permute per pair),
        // lo = rnd(p - hi): ~16 significant bits in all
        const uint32_t b0 = __float_as_uint(p0), b1 = __float_as_uint(p1);
        hv[e] = __byte_perm(b0, b1, 0x7632);
        lv[e] = pack_bf2(p0 - __uint_as_float(b0 & 0xFFFF0000u),
                         p1 - __uint_as_float(b1 & 0xFFFF0000u));
      }
    }
    umma::tmem_st16u(col + c * 16, hv);
    if constexpr (kSplit) umma::tmem_st16u(col + 64 + c * 16, lv);
  }
}

// ======================================================================
// kp3_kernel: two query tiles per CTA, 128-key score tiles, one MMA issuer
// that polls.
//
// CTA = query tiles A = 2*pair and B = 2*pair + 1 (B may be absent) of one
// q-head; both walk the same K/V tiles (B's causal range; A takes part in
// the tiles it can see, a prefix of each segment's).  384 threads:
//   WG0  warp 0 lane 0: TMA producer (Q once, then K and V tiles of 128
//        keys through ST-stage rings); warp 1: TMEM owner, lane 0 issues
//        every MMA of both tiles; warps 2-3 idle.  88 registers.
//   WG1  softmax of tile A (thread r = TMEM lane r = query row r), 208 regs.
//   WG2  softmax of tile B.
// TMEM (512 columns): per tile X a 128-column score buffer S_X = [128X,
// 128X + 128) and a D-column output accumulator O_X = [256 + D X, ...).
// QK_X(j): S_X = Q_X K(j)^T, M128 N128, both operands in shared memory.
// The softmax writes P_X(j) back into S_X's columns as 16-bit pairs (fp16
// route: keys 2c, 2c+1 in column c < 64; bf16 route: the high parts there
// and the residuals in column 64 + c) and PV_X(j): O_X += P_X(j) V(j) takes
// P from TMEM as the A operand (M128 N=D), so P never touches shared memory.
// With one score buffer per tile, QK_X(j+1) is issued only once PV_X(j) has
// completed; the issuer keeps the tensor pipe busy with the other tile's
// work meanwhile, so the two softmax groups alternate with the MMAs.
// Issuer: a single thread polls (mbarrier.test_wait) and issues whichever
// of the four next steps (QK/PV of A/B) has its inputs ready; it never waits
// on one step while another could go, so no order of chunks can stall it.
// It observes K and V landings in walk order (landed prefixes), so no ring
// stage is probed before its previous use was seen to land.
// Ring barriers: k_full/v_full (one arrival + the copy's bytes), k_empty /
// v_empty (two arrivals: a tcgen05.commit per query tile that reads the
// tile, the producer arriving for a tile that sits it out).  Per tile X:
// s_full (commit after QK), p_full (one arrival per softmax warp), pv_done
// (commit after PV).  All waits bounded; TMEM freed on every exit path.
constexpr int kThreads = 384;

template <int D>
struct Geom {
  static constexpr int kBlocks = D / 64;                  // 128-byte column blocks
  static constexpr int kBlockBytes = kBN * 128;           // one block of a 128-row tile
  static constexpr int kTileBytes = kBlocks * kBlockBytes;
  static constexpr int kStages = D == 64 ? 4 : 2;
  static constexpr int kOffQ = 0;                         // Q_A, Q_B
  static constexpr int kOffK = 2 * kTileBytes;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffBar = kOffV + kStages * kTileBytes;
  static constexpr int kSmemBytes = kOffBar + 512 + 1024;   // barriers + tile table, alignment
  static constexpr uint32_t kColO = 256;
};

struct Bars {
  uint64_t q_full;
  uint64_t k_full[4], v_full[4], k_empty[4], v_empty[4];
  uint64_t s_full[2], p_full[2], pv_done[2], mma_done;
  uint32_t tmem_base;
  int abort_flag;
  int nU, nA;                        // K/V tiles of the walk, and tile A's share
  int16_t ntU[kMaxSegs], ntA[kMaxSegs];   // per segment: tiles B (the walk) / A see
  int16_t t0[kMaxSegs];              // per segment: first tile of this CTA's window
};
static_assert(sizeof(Bars) <= 512, "barrier block");

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Bars* bs,
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

// Position in the walk over the K/V tiles of a CTA (segment s, tile t of
// that segment, global tile index g counting every tile of the walk).
struct Cursor {
  int s, t, g;
  int end;     // tiles of segment s this query tile takes part in (cached)
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) kp3_kernel(const __grid_constant__ Params p) {
  using Gm = Geom<D>;
  constexpr int ST = Gm::kStages;
  constexpr bool kBf16 = Elem<T>::kDtype == HALO_DTYPE_BF16;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bs = reinterpret_cast<Bars*>(smem + Gm::kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int BH = p.B * p.H;
  const int n_pairs = (p.n_qtiles + 1) / 2;
  // unit = (pair, bh), heaviest pairs first; units from n_full on are split
  // into two CTAs (half 0: the first half of the walk, half 1: the rest)
  int unit = (int)blockIdx.x, half = -1;
  if (unit >= p.n_full) {
    const int k = unit - p.n_full;
    unit = p.n_full + (k >> 1);
    half = k & 1;
  }
  const int pair = n_pairs - 1 - unit / BH;
  const int bh = unit % BH;
  const int b = bh / p.H, h = bh % p.H, hk = h / p.G;
  const int qA0 = 2 * pair * kBM;
  const bool hasB = 2 * pair + 1 < p.n_qtiles;
  const int validA = min(kBM, p.T_q - qA0);
  const int validB = hasB ? min(kBM, p.T_q - (qA0 + kBM)) : 0;
  const int64_t qminA = p.q_pos0 + qA0, qmaxA = qminA + validA - 1;
  const int64_t qminB = qminA + kBM, qmaxB = qminB + validB - 1;
  const int64_t qmaxU = hasB ? qmaxB : qmaxA;
  // P as one fp16 operand with fp16 V (fp16 inputs, or bf16 inputs whose
  // fp16 V copy is in range); otherwise bf16 hi + lo with bf16 V
  const bool p16 = !kBf16 || (p.v16_flag != nullptr && *p.v16_flag == 0u);
  const CUtensorMap* vmaps = (kBf16 && p16) ? p.v16map : p.vmap;

  if (threadIdx.x == 0) {
    mbar_init(&bs->q_full, 1);
    for (int i = 0; i < ST; ++i) {
      mbar_init(&bs->k_full[i], 1);
      mbar_init(&bs->v_full[i], 1);
      mbar_init(&bs->k_empty[i], 2);
      mbar_init(&bs->v_empty[i], 2);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bs->s_full[x], 1);
      mbar_init(&bs->p_full[x], kBM / 32);
      mbar_init(&bs->pv_done[x], 1);
    }
    mbar_init(&bs->mma_done, 1);
    bs->abort_flag = 0;
    // this CTA's window [glo, ghi) of the union walk: all of it, or one
    // half of a split unit's
    int nfull = 0;
    for (int s = 0; s < p.n_seg; ++s) nfull += seg_tiles(p.seg[s], qmaxU);
    const int glo = half == 1 ? nfull / 2 : 0;
    const int ghi = half == 0 ? nfull / 2 : nfull;
    int nu = 0, na = 0, gb = 0;
    for (int s = 0; s < p.n_seg; ++s) {
      const int tu = seg_tiles(p.seg[s], qmaxU), ta = seg_tiles(p.seg[s], qmaxA);
      const int lo = min(max(glo - gb, 0), tu), hi = min(max(ghi - gb, 0), tu);
      // tile A's tiles are a prefix of the segment's, so of the window too
      const int wa = max(0, min(hi, ta) - lo);
      bs->t0[s] = (int16_t)lo;
      bs->ntU[s] = (int16_t)(hi - lo);
      bs->ntA[s] = (int16_t)wa;
      nu += hi - lo;
      na += wa;
      gb += tu;
    }
    bs->nU = nu;
    bs->nA = na;
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
  const int nU = bs->nU, nA = bs->nA;

  const uint32_t sQ = smem_addr(smem + Gm::kOffQ);
  const uint32_t sK = smem_addr(smem + Gm::kOffK);
  const uint32_t sV = smem_addr(smem + Gm::kOffV);

  // Register split (128 x 88 + 256 x 208 = 384 x 168, the launch budget),
  // made inside each role's branch so the compiler sizes each role's code
  // for its own budget.
  if (warp < 4) {
    umma::regs_dec<88>();
    if (warp == 0) {
      // ---------------------------------------------------------- producer
      if (lane == 0 && nU > 0) {
        mbar_arrive_expect_tx(&bs->q_full, (hasB ? 2 : 1) * Gm::kTileBytes);
        for (int x = 0; x < (hasB ? 2 : 1); ++x)
          for (int blk = 0; blk < Gm::kBlocks; ++blk)
            tma_load_4d(smem + Gm::kOffQ + x * Gm::kTileBytes + blk * Gm::kBlockBytes, &p.qmap,
                        blk * 64, qA0 + x * kBM, h, b, &bs->q_full);
        int nk = 0, nv = 0;   // K and V tile loads issued
        bool ok = true;
        for (int s = 0; s < p.n_seg && ok; ++s) {
          const int nt = bs->ntU[s];
          const int ntA = bs->ntA[s];
          const int bb = p.seg[s].bcast ? 0 : b;
          for (int t = 0; t < nt; ++t) {
            // the empty barriers take one arrival per query tile; a tile
            // that sits this K/V tile out is arrived for here
            const uint32_t absent = (t < ntA ? 0u : 1u) + (hasB ? 0u : 1u);
            const int st = nk % ST, use = nk / ST;
            if (use > 0 && !(ok = wait_bar(&bs->k_empty[st], (use - 1) & 1, bs, p.err))) break;
            mbar_arrive_expect_tx(&bs->k_full[st], Gm::kTileBytes);
            for (int blk = 0; blk < Gm::kBlocks; ++blk)
              tma_load_4d(smem + Gm::kOffK + st * Gm::kTileBytes + blk * Gm::kBlockBytes,
                          &p.kmap[s], blk * 64, (bs->t0[s] + t) * kBN, hk, bb, &bs->k_full[st]);
            if (absent) mbar_arrive_n(&bs->k_empty[st], absent);
            ++nk;
            if (use > 0 && !(ok = wait_bar(&bs->v_empty[st], (use - 1) & 1, bs, p.err))) break;
            mbar_arrive_expect_tx(&bs->v_full[st], Gm::kTileBytes);
            for (int blk = 0; blk < Gm::kBlocks; ++blk)
              tma_load_4d(smem + Gm::kOffV + st * Gm::kTileBytes + blk * Gm::kBlockBytes,
                          &vmaps[s], blk * 64, (bs->t0[s] + t) * kBN, hk, bb, &bs->v_full[st]);
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
    } else if (warp == 1 && lane == 0 && nU > 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t kIdQK = umma::instr_desc_f16(kBM, kBN, kBf16, false, false);
      const uint32_t kIdPV = umma::instr_desc_f16(kBM, D, !p16, false, true);
      const uint64_t kdesc0 = umma::smem_desc_sw128(sK, 16, 1024);
      const uint64_t vdesc0 = umma::smem_desc_sw128(sV, Gm::kBlockBytes, 1024);
      const int nX[2] = {nA, hasB ? nU : 0};
      // cursors: next K/V tile each query tile takes part in, for QK and PV
      const int n_seg = p.n_seg;
      // (re)enter a segment: skip the tiles and segments tile x sits out
      auto seek = [&](Cursor& c, int x) {
        while (c.s < n_seg) {
          const int ntU = bs->ntU[c.s];
          const int ntX = x ? ntU : bs->ntA[c.s];
          if (c.t < ntX) {
            c.end = ntX;
            return;
          }
          c.g += ntU - c.t;   // the rest of this segment is sat out
          ++c.s;
          c.t = 0;
        }
      };
      // next tile: stays in the segment without touching shared memory
      auto step = [&](Cursor& c, int x) {
        ++c.t;
        ++c.g;
        if (c.t >= c.end) seek(c, x);
      };
      // qc: next K/V tile each query tile's QK takes; pg: the tile of its
      // pending P V (one at most: QK(j+1) waits for PV(j))
      Cursor qc[2] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
      int pg[2] = {0, 0};
      for (int x = 0; x < 2; ++x) seek(qc[x], x);
      int jq[2] = {0, 0}, jp[2] = {0, 0};
      // (The two softmax groups settle half a step apart by themselves:
      // with one tensor pipe and one score buffer per tile, their tiles'
      // softmaxes overlap < 1 % of the time, measured; no gate is needed.)
      // Landed prefixes: K (V) tiles below kpre (vpre) are known to have
      // landed.  The next tile's full barrier is probed in walk order, so a
      // stage is only probed after its previous use was seen to land: a
      // parity probe of phase n while phase n-1 is still open would read
      // as complete (a query tile that sits tiles out would otherwise
      // probe ahead of the ring).
      int kpre = 0, vpre = 0;
      int qseq[2] = {0, 0}, seq = 0;       // issue order of each tile's latest QK
      bool ok = wait_bar(&bs->q_full, 0, bs, p.err);
      uint64_t t_idle = 0;
      int idle = 0;
      // advance a landed prefix up to tile g, probing only as far as needed
      // (each probe is a shared-memory access that queues behind the MMAs'
      // operand reads)
      auto landed = [&](int& pre, uint64_t* full, int g) {
        while (pre <= g && mbar_test(&full[pre % ST], (pre / ST) & 1)) ++pre;
        return g < pre;
      };
      while (ok) {
        bool did = false;
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          // O_X += P_X(j) V(j): P written and V landed
          if (jp[x] < jq[x]) {
            const int g = pg[x], st = g % ST;
            if (mbar_test(&bs->p_full[x], jp[x] & 1) && landed(vpre, bs->v_full, g)) {
              umma::fence_after_sync();
              const uint32_t pcol = tmem + x * 128;
              const uint32_t ocol = tmem + Gm::kColO + x * D;
              const uint64_t vd = opaque(vdesc0 + (uint64_t)((st * Gm::kTileBytes) >> 4));
              const bool acc0 = jp[x] > 0;
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk)
                umma::mma_ts(ocol, pcol + kk * 8, vd + (uint64_t)((kk * 16 * 128) >> 4), kIdPV,
                             acc0 || kk > 0);
              if (!p16) {
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk)
                  umma::mma_ts(ocol, pcol + 64 + kk * 8, vd + (uint64_t)((kk * 16 * 128) >> 4),
                               kIdPV, true);
              }
              umma::commit(&bs->pv_done[x]);
              umma::commit(&bs->v_empty[st]);
              ++jp[x];
              did = true;
            }
          }
          // S_X = Q_X K(j)^T: S_X free (previous PV_X completed) and K landed
          if (jq[x] < nX[x] && jq[x] == jp[x]) {
            const int g = qc[x].g, st = g % ST;
            if ((jq[x] == 0 || mbar_test(&bs->pv_done[x], (jq[x] - 1) & 1)) &&
                landed(kpre, bs->k_full, g)) {
              umma::fence_after_sync();
              const uint64_t qd = opaque(umma::smem_desc_sw128(sQ + x * Gm::kTileBytes, 16, 1024));
              const uint64_t kd = opaque(kdesc0 + (uint64_t)((st * Gm::kTileBytes) >> 4));
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t off = ((kk >> 2) * Gm::kBlockBytes + (kk & 3) * 32) >> 4;
                umma::mma_ss(tmem + x * 128, qd + off, kd + off, kIdQK, kk > 0);
              }
              umma::commit(&bs->s_full[x]);
              umma::commit(&bs->k_empty[st]);
              qseq[x] = ++seq;
              pg[x] = g;
              ++jq[x];
              step(qc[x], x);
              did = true;
            }
          }
        }
        if (jp[0] >= nX[0] && jp[1] >= nX[1]) break;
        if (did) {
          idle = 0;
          continue;
        }
        // Nothing ready.  Sleep in hardware on the event expected first, so
        // the issuer takes no issue slots from the softmax warps that share
        // its scheduler: a P V completing (it frees a score buffer for the
        // next QK), else the oldest pending P (its softmax started first),
        // else the next K or V tile to land (probed in walk order); every
        // probe stays within one phase of its barrier, as above.
        {
          bool slept = false;
#pragma unroll
          for (int x = 0; x < 2 && !slept; ++x) {
            if (jq[x] < nX[x] && jq[x] == jp[x] && jq[x] > 0 &&
                !mbar_test(&bs->pv_done[x], (jq[x] - 1) & 1)) {
              mbar_sleep_wait(&bs->pv_done[x], (jq[x] - 1) & 1, 1000);
              slept = true;
            }
          }
          if (!slept) {
            int xo = -1;
            if (jp[0] < jq[0]) xo = 0;
            if (jp[1] < jq[1] && (xo < 0 || qseq[1] < qseq[0])) xo = 1;
            if (xo >= 0 && !mbar_test(&bs->p_full[xo], jp[xo] & 1)) {
              mbar_sleep_wait(&bs->p_full[xo], jp[xo] & 1, 1000);
              slept = true;
            } else if (xo >= 0 && vpre < nU) {
              mbar_sleep_wait(&bs->v_full[vpre % ST], (vpre / ST) & 1, 1000);
              slept = true;
            } else if (kpre < nU) {
              mbar_sleep_wait(&bs->k_full[kpre % ST], (kpre / ST) & 1, 1000);
              slept = true;
            }
          }
          if (!slept) __nanosleep(64);
        }
        // bounded idle time; stop if another role aborted
        if (++idle == 64) t_idle = globaltimer_ns();
        if (idle > 64 && (idle & 63) == 0) {
          if (*reinterpret_cast<volatile int*>(&bs->abort_flag)) {
            ok = false;
          } else if (globaltimer_ns() - t_idle > kWaitLimitNs) {
            set_device_error(p.err, static_cast<unsigned int>(-HALO_ERR_TIMEOUT));
            *reinterpret_cast<volatile int*>(&bs->abort_flag) = 1;
            ok = false;
          }
        }
      }
      // this thread's MMAs complete before the CTA can free TMEM
      umma::commit(&bs->mma_done);
      mbar_wait(&bs->mma_done, 0, p.err);
    }
  } else {
    umma::regs_inc<208>();
    // ------------------------------------------------------------ softmax X
    const int x = (warp - 4) >> 2;              // 0: tile A, 1: tile B
    const int sub = warp & 3;
    const int r = sub * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(sub * 32) << 16);
    const uint32_t scol = x * 128;
    const uint32_t ocol = Gm::kColO + x * D;
    const bool active = x == 0 || hasB;
    const int64_t qmin = x ? qminB : qminA;
    const int64_t qpos = qmin + r;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    int j = 0;
    for (int s = 0; s < p.n_seg && ok && active; ++s) {
      const Seg sg = p.seg[s];
      const int nt = x ? bs->ntU[s] : bs->ntA[s];
      for (int t = 0; t < nt; ++t, ++j) {
        ok = __all_sync(0xffffffffu, wait_bar(&bs->s_full[x], j & 1, bs, p.err));
        if (!ok) break;
        umma::fence_after_sync();
        const int row0 = (bs->t0[s] + t) * kBN;
        const int64_t kpos0 = sg.start + row0;
        const bool full = (row0 + kBN <= sg.len) && (!sg.causal || kpos0 + kBN - 1 <= qmin);
        const int lim_len = sg.len - row0;
        const int64_t lim_pos = sg.causal ? qpos - kpos0 : (int64_t)kBN;
        float sv[kBN];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) umma::tmem_ld32(trow + scol + c * 32, sv + c * 32);
        umma::tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int c = 0; c < kBN; ++c)
            if (!(c < lim_len && (int64_t)c <= lim_pos)) sv[c] = -INFINITY;
        }
        float mx8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx8[e] = sv[e];
#pragma unroll
        for (int c = 8; c < kBN; c += 16) {
#pragma unroll
          for (int e = 0; e < 8; ++e) mx8[e] = fmax3(mx8[e], sv[c + e], sv[c + 8 + e]);
        }
        const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                               fmaxf(mx8[6], mx8[7])) *
                         p.scale_log2;
        const bool grow = mx > m + kRescaleLog2 || (m == -INFINITY && mx > -INFINITY);
        float fac = 1.f;
        if (grow) {
          fac = (m == -INFINITY) ? 0.f : ex2(m - mx);
          l *= fac;
          m = mx;
        }
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
          // O_X is quiescent: QK_X(j) was issued after PV_X(j-1) completed,
          // and PV_X(j) waits for this P
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
        const uint64_t sl2 = f2pack(p.scale_log2, p.scale_log2), nm2 = f2pack(nmu, nmu);
        uint64_t rs2[2] = {0ull, 0ull};   // row-sum pairs (+0.f bits)
        if (p16)
          write_p<false>(sv, sl2, nm2, trow + scol, rs2);
        else
          write_p<true>(sv, sl2, nm2, trow + scol, rs2);
        float rs4[4];
        f2unpack(rs2[0], rs4[0], rs4[1]);
        f2unpack(rs2[1], rs4[2], rs4[3]);
        l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
        umma::tmem_wait_st();
        umma::fence_before_sync();
        __syncwarp();                    // the warp's P is in TMEM: one arrival
        if (lane == 0) mbar_arrive(&bs->p_full[x]);
      }
    }
    const int nX = j;

    // ---- epilogue of tile X: thread r finalises query row q0 + r
    if (active && ok && nX > 0) {
      ok = __all_sync(0xffffffffu, wait_bar(&bs->pv_done[x], (nX - 1) & 1, bs, p.err));
      if (ok) umma::fence_after_sync();
    }
    const int validX = x ? validB : validA;
    if (active && ok && half >= 0) {
      // one half of a split unit: unnormalised o, M (natural log), L of the
      // row, for pf_merge_kernel
      float* pr = p.part + ((int64_t)((int)blockIdx.x - p.n_full) * 2 * kBM + x * kBM + r) *
                               kPartStride<D>;
      const bool live = r < validX;
      if (live) {
        pr[D] = (m == -INFINITY) ? -INFINITY : m * kLn2;
        pr[D + 1] = l;
      }
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
        float4* od = reinterpret_cast<float4*>(pr + c * 32);
#pragma unroll
        for (int e = 0; e < 32; e += 4) od[e / 4] = make_float4(ov[e], ov[e + 1], ov[e + 2], ov[e + 3]);
      }
    } else if (active && ok) {
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
            od[e / 8] = make_uint4(Elem<T>::pack(ov[e] * inv, ov[e + 1] * inv),
                                   Elem<T>::pack(ov[e + 2] * inv, ov[e + 3] * inv),
                                   Elem<T>::pack(ov[e + 4] * inv, ov[e + 5] * inv),
                                   Elem<T>::pack(ov[e + 6] * inv, ov[e + 7] * inv));
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

// ======================================================================
// v16_kernel: fp16 copy of each segment's bf16 V rows into the workspace
// (layout [batch'][H_kv][len][D] per segment, batch' = 1 for a segment that
// broadcasts the batch) and a flag raised when a finite |v| >= 2^16 would
// overflow fp16.  Memory-bound: 16-byte loads and stores, grid (row blocks,
// segment, batch' x H_kv).
struct V16Seg {
  const uint16_t* src;    // bf16 bits
  int64_t sb, sh, st;     // element strides
  uint16_t* dst;          // fp16 bits
  int32_t len;
  int32_t nb;             // batch rows stored (1 when broadcast)
};

struct V16Params {
  V16Seg seg[kMaxSegs];
  int32_t H_kv, D;
  unsigned int* flag;
};

constexpr int kV16Rows = 64;     // rows per CTA
constexpr int kV16Threads = 128;

__global__ void __launch_bounds__(kV16Threads) v16_kernel(const __grid_constant__ V16Params p) {
  const V16Seg& sg = p.seg[blockIdx.y];
  const int bh = blockIdx.z;
  if (bh >= sg.nb * p.H_kv) return;
  const int b = bh / p.H_kv, hk = bh % p.H_kv;
  const int r0 = blockIdx.x * kV16Rows;
  if (r0 >= sg.len) return;
  const int rows = min(kV16Rows, sg.len - r0);
  const int vpr = p.D / 8;                      // 16-byte vectors per row
  const uint16_t* src = sg.src + (int64_t)b * sg.sb + (int64_t)hk * sg.sh;
  uint16_t* dst = sg.dst + ((int64_t)bh * sg.len) * p.D;
  unsigned int bad = 0;
  for (int i = threadIdx.x; i < rows * vpr; i += kV16Threads) {
    const int r = r0 + i / vpr, c = i % vpr;
    const uint4 w = *reinterpret_cast<const uint4*>(src + (int64_t)r * sg.st + c * 8);
    const uint32_t in[4] = {w.x, w.y, w.z, w.w};
    uint32_t out[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t lo = in[k] & 0xFFFFu, hi = in[k] >> 16;
      // finite magnitude at or above 2^16 (bf16 0x4780) overflows fp16
      bad |= (((lo & 0x7FFFu) >= 0x4780u) & ((lo & 0x7FFFu) < 0x7F80u)) |
             (((hi & 0x7FFFu) >= 0x4780u) & ((hi & 0x7FFFu) < 0x7F80u));
      out[k] = pack_h2(__uint_as_float(lo << 16), __uint_as_float(hi << 16));
    }
    *reinterpret_cast<uint4*>(dst + (int64_t)r * p.D + c * 8) =
        make_uint4(out[0], out[1], out[2], out[3]);
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(p.flag, 1u);
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

namespace prefill {
// Folds the two halves of each split unit: block (u, x) = query tile x of
// split unit u, thread r = row; the same output contract as kp3_kernel's
// finalising epilogue (out in out_dtype, lse in natural log).
template <typename T, int D>
__global__ void __launch_bounds__(kBM) pf_merge_kernel(const __grid_constant__ Params p) {
  const int BH = p.B * p.H;
  const int n_pairs = (p.n_qtiles + 1) / 2;
  const int unit = p.n_full + (int)blockIdx.x;
  const int pair = n_pairs - 1 - unit / BH, bh = unit % BH;
  const int b = bh / p.H, h = bh % p.H;
  const int x = (int)blockIdx.y, r = (int)threadIdx.x;
  const int t = 2 * pair * kBM + x * kBM + r;
  if (t >= p.T_q) return;
  constexpr int kS = kPartStride<D>;
  const float* p0 = p.part + ((int64_t)(2 * (int)blockIdx.x) * 2 * kBM + x * kBM + r) * kS;
  const float* p1 = p0 + (int64_t)2 * kBM * kS;
  const float M0 = p0[D], L0 = p0[D + 1], M1 = p1[D], L1 = p1[D + 1];
  const float Mn = fmaxf(M0, M1);
  const float w0 = (M0 == -INFINITY) ? 0.f : expf(M0 - Mn);
  const float w1 = (M1 == -INFINITY) ? 0.f : expf(M1 - Mn);
  const float L = L0 * w0 + L1 * w1;
  const float inv = (L > 0.f) ? 1.f / L : 0.f;
  const int64_t row = ((int64_t)b * p.H + h) * p.T_q + t;
  if (p.lse) p.lse[row] = (L > 0.f) ? Mn + logf(L) : -INFINITY;
  const int64_t off = (int64_t)b * p.out_sb + (int64_t)h * p.out_sh + (int64_t)t * p.out_st;
  const float4* a4 = reinterpret_cast<const float4*>(p0);
  const float4* c4 = reinterpret_cast<const float4*>(p1);
#pragma unroll 4
  for (int c = 0; c < D / 8; ++c) {
    const float4 a0 = a4[2 * c], a1 = a4[2 * c + 1], c0 = c4[2 * c], c1 = c4[2 * c + 1];
    const float v[8] = {(a0.x * w0 + c0.x * w1) * inv, (a0.y * w0 + c0.y * w1) * inv,
                        (a0.z * w0 + c0.z * w1) * inv, (a0.w * w0 + c0.w * w1) * inv,
                        (a1.x * w0 + c1.x * w1) * inv, (a1.y * w0 + c1.y * w1) * inv,
                        (a1.z * w0 + c1.z * w1) * inv, (a1.w * w0 + c1.w * w1) * inv};
    if (p.out_dtype == HALO_DTYPE_F32) {
      float4* od = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + off + c * 8);
      od[0] = make_float4(v[0], v[1], v[2], v[3]);
      od[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      uint4* od = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + off + c * 8);
      *od = make_uint4(Elem<T>::pack(v[0], v[1]), Elem<T>::pack(v[2], v[3]),
                       Elem<T>::pack(v[4], v[5]), Elem<T>::pack(v[6], v[7]));
    }
  }
}
}  // namespace prefill

template <typename T, int D>
static int launch_kp3(const prefill::Params& prm, int grid, int n_split, cudaStream_t st) {
  using Gm = prefill::Geom<D>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(prefill::kp3_kernel<T, D>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, Gm::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "kp3_kernel shared-memory attribute");
  prefill::kp3_kernel<T, D><<<grid, prefill::kThreads, Gm::kSmemBytes, st>>>(prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kp3_kernel launch");
  count_launches();
  if (n_split > 0) {
    prefill::pf_merge_kernel<T, D><<<dim3((unsigned)n_split, 2), prefill::kBM, 0, st>>>(prm);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "pf_merge_kernel launch");
    count_launches();
  }
  return HALO_OK;
}

// One coalesced run of chunks: the first chunk's pointers, strides, start
// and causal flag, its total length and whether the batch broadcasts.
struct PfSeg {
  halo_kv_chunk_t c;
  int64_t len;
  bool bcast;
};

// Validate the problem and the output description (everything but the
// chunks).
static int pf_check(const halo_prefill_problem_t* pb, const halo_prefill_out_t* po, bool need_out) {
  if (!pb || (need_out && !po)) return fail(HALO_ERR_INVALID_ARG, "problem/out is NULL");
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
  if (!need_out) return HALO_OK;
  if (po->mode != HALO_MERGE_FINALIZE && po->mode != HALO_MERGE_ACCUMULATE)
    return fail(HALO_ERR_INVALID_ARG, "bad mode %d", po->mode);
  const bool have_state = po->m || po->l || po->o;
  if (have_state && !(po->m && po->l && po->o))
    return fail(HALO_ERR_INVALID_ARG, "running state needs all of m, l, o");
  if (po->mode == HALO_MERGE_ACCUMULATE && !have_state)
    return fail(HALO_ERR_INVALID_ARG, "accumulate needs m, l, o");
  if (po->o && !aligned16(po->o)) return fail(HALO_ERR_MISALIGNED, "o must be 16-byte aligned");
  if (po->mode == HALO_MERGE_FINALIZE) {
    if (!po->out) return fail(HALO_ERR_INVALID_ARG, "out is NULL");
    const int oe = po->out_dtype == HALO_DTYPE_F32 ? 4 : 2;
    if (po->out_dtype != HALO_DTYPE_F32 && po->out_dtype != pb->dtype)
      return fail(HALO_ERR_UNSUPPORTED, "out dtype must be fp32 or the input dtype");
    if (!aligned16(po->out) || (po->out_stride_b * oe) % 16 || (po->out_stride_h * oe) % 16 ||
        (po->out_stride_t * oe) % 16)
      return fail(HALO_ERR_MISALIGNED, "out rows must be 16-byte aligned");
  }
  return HALO_OK;
}

// Coalesce chunks contiguous in memory and position into segments (at most
// kMaxSegs), validating each chunk.
static int pf_segments(const halo_kv_chunk_t* chunks, int32_t n_chunks, PfSeg* segs, int* n_out) {
  if (n_chunks < 0 || (n_chunks > 0 && !chunks)) return fail(HALO_ERR_INVALID_ARG, "bad chunk list");
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
  *n_out = n_seg;
  return HALO_OK;
}

static int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// Bytes of segment i's fp16 V copy in the workspace.
static int64_t pf_v16_bytes(const PfSeg& sg, const halo_prefill_problem_t* pb) {
  return align256((int64_t)(sg.bcast ? 1 : pb->B) * pb->H_kv * sg.len * pb->D * 2);
}

// Units of the last partial wave that run as two half-walk CTAs each (0:
// none): the grid has more units than SMs (one CTA per SM), a remainder, and
// the lightest unit (pair 0, the last in heavy-first order) walks at least
// 8 K/V tiles.  Splitting those units fills the last wave with half-length
// work instead of leaving SMs idle for a whole unit's time.
static int pf_split_units(const PfSeg* segs, int n_seg, const halo_prefill_problem_t* pb) {
  const int64_t n_qtiles = (pb->T_q + prefill::kBM - 1) / prefill::kBM;
  const int64_t units = (n_qtiles + 1) / 2 * pb->B * pb->H;
  const int W = device_sms();
  if (n_seg == 0 || W <= 0 || units <= W || units % W == 0) return 0;
  const int64_t qmax0 = pb->q_pos0 + std::min<int64_t>(2 * prefill::kBM, pb->T_q) - 1;
  int tiles = 0;
  for (int i = 0; i < n_seg; ++i) {
    prefill::Seg sg;
    sg.start = segs[i].c.start;
    sg.len = (int32_t)segs[i].len;
    sg.causal = segs[i].c.causal ? 1 : 0;
    sg.bcast = segs[i].bcast ? 1 : 0;
    tiles += prefill::seg_tiles(sg, qmax0);
  }
  return tiles >= 8 ? (int)(units % W) : 0;
}

// Workspace layout: [flag word, 256 B][fp16 V copies (bf16 inputs)][split
// partials: per half-walk CTA 2 x 128 rows of kPartStride floats].
static int64_t pf_part_offset(const PfSeg* segs, int n_seg, const halo_prefill_problem_t* pb) {
  int64_t n = prefill::kWsHeader;
  if (pb->dtype == HALO_DTYPE_BF16)
    for (int i = 0; i < n_seg; ++i) n += pf_v16_bytes(segs[i], pb);
  return align256(n);
}

static int64_t pf_part_bytes(int n_split, int D) {
  return (int64_t)n_split * 2 * 2 * prefill::kBM * (D + 4) * 4;
}

static int64_t pf_workspace_bytes(const PfSeg* segs, int n_seg, const halo_prefill_problem_t* pb) {
  if (n_seg == 0) return 0;
  const int n_split = pf_split_units(segs, n_seg, pb);
  if (n_split > 0) return pf_part_offset(segs, n_seg, pb) + pf_part_bytes(n_split, pb->D);
  if (pb->dtype != HALO_DTYPE_BF16) return 0;
  int64_t n = prefill::kWsHeader;
  for (int i = 0; i < n_seg; ++i) n += pf_v16_bytes(segs[i], pb);
  return n;
}

static int pf_run(const halo_prefill_problem_t* pb, const halo_kv_chunk_t* chunks,
                  int32_t n_chunks, const halo_prefill_out_t* po, void* workspace,
                  int64_t workspace_bytes, halo_stream_t stream) {
  int rc = pf_check(pb, po, true);
  if (rc != HALO_OK) return rc;
  PfSeg segs[prefill::kMaxSegs];
  int n_seg = 0;
  rc = pf_segments(chunks, n_chunks, segs, &n_seg);
  if (rc != HALO_OK) return rc;
  if (pb->T_q == 0) return HALO_OK;
  if (!pb->q || !aligned16(pb->q) || (pb->q_stride_t * 2) % 16 || (pb->q_stride_h * 2) % 16 ||
      (pb->B > 1 && (pb->q_stride_b * 2) % 16) || pb->q_stride_t <= 0 || pb->q_stride_h <= 0)
    return fail(HALO_ERR_MISALIGNED, "q must be 16-byte aligned with 16-byte row strides");
  const int D = pb->D;
  const bool v16 = workspace != nullptr && pb->dtype == HALO_DTYPE_BF16 && n_seg > 0;
  // split the last wave's units only for a finalising call without a
  // caller running state (the halves' partials are merged into out here)
  const int n_split = (workspace != nullptr && po->mode != HALO_MERGE_ACCUMULATE &&
                       po->m == nullptr)
                          ? pf_split_units(segs, n_seg, pb)
                          : 0;
  if (workspace != nullptr) {
    const int64_t need = pf_workspace_bytes(segs, n_seg, pb);
    if (workspace_bytes < need)
      return fail(HALO_ERR_WORKSPACE, "prefill workspace has %lld bytes, needs %lld",
                  (long long)workspace_bytes, (long long)need);
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
      return fail(HALO_ERR_MISALIGNED, "prefill workspace must be 256-byte aligned");
  }

  static thread_local prefill::Params prm;
  static thread_local prefill::V16Params vp;
  char* ws = static_cast<char*>(workspace);
  int64_t ws_off = prefill::kWsHeader;
  for (int i = 0; i < n_seg; ++i) {
    const halo_kv_chunk_t& c = segs[i].c;
    const bool bk = segs[i].bcast;
    const uint64_t nb = bk ? 1 : pb->B;
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)segs[i].len, (uint64_t)pb->H_kv, nb};
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
    if (v16) {
      // contiguous fp16 copy [nb][H_kv][len][D]
      void* dst = ws + ws_off;
      const uint64_t s16[3] = {(uint64_t)D * 2, (uint64_t)segs[i].len * D * 2,
                               (uint64_t)pb->H_kv * segs[i].len * D * 2};
      rc = pf_encode(dst, HALO_DTYPE_F16, dims, s16, &prm.v16map[i]);
      if (rc != HALO_OK) return rc;
      prefill::V16Seg& vsg = vp.seg[i];
      vsg.src = static_cast<const uint16_t*>(c.v);
      vsg.sb = bk ? 0 : c.v_stride_b;
      vsg.sh = c.v_stride_h;
      vsg.st = c.v_stride_t;
      vsg.dst = static_cast<uint16_t*>(dst);
      vsg.len = (int32_t)segs[i].len;
      vsg.nb = (int32_t)nb;
      ws_off += pf_v16_bytes(segs[i], pb);
    }
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
  prm.v16_flag = v16 ? reinterpret_cast<const unsigned int*>(ws) : nullptr;
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
  const int64_t units = (int64_t)((prm.n_qtiles + 1) / 2) * pb->B * pb->H;
  prm.n_full = (int32_t)(units - n_split);
  prm.part = n_split > 0 ? reinterpret_cast<float*>(ws + pf_part_offset(segs, n_seg, pb))
                         : nullptr;
  const int64_t grid = units + n_split;
  if (grid > INT32_MAX) return fail(HALO_ERR_UNSUPPORTED, "grid too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pb->event_begin) cudaEventRecord(static_cast<cudaEvent_t>(pb->event_begin), st);
  if (v16) {
    // the fp16 V copies and the range flag, on the same stream
    cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return cuda_fail(e, "clear prefill range flag");
    int64_t max_len = 0, max_bh = 0;
    for (int i = 0; i < n_seg; ++i) {
      max_len = std::max<int64_t>(max_len, segs[i].len);
      max_bh = std::max<int64_t>(max_bh, (int64_t)vp.seg[i].nb * pb->H_kv);
    }
    if (max_bh > 65535) return fail(HALO_ERR_UNSUPPORTED, "batch x H_kv too large");
    vp.H_kv = pb->H_kv;
    vp.D = D;
    vp.flag = reinterpret_cast<unsigned int*>(ws);
    const dim3 vgrid((unsigned)((max_len + prefill::kV16Rows - 1) / prefill::kV16Rows),
                     (unsigned)n_seg, (unsigned)max_bh);
    prefill::v16_kernel<<<vgrid, prefill::kV16Threads, 0, st>>>(vp);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "v16_kernel launch");
    count_launches();
  }
  if (pb->dtype == HALO_DTYPE_BF16)
    rc = D == 128 ? launch_kp3<__nv_bfloat16, 128>(prm, (int)grid, n_split, st)
                  : launch_kp3<__nv_bfloat16, 64>(prm, (int)grid, n_split, st);
  else
    rc = D == 128 ? launch_kp3<__half, 128>(prm, (int)grid, n_split, st)
                  : launch_kp3<__half, 64>(prm, (int)grid, n_split, st);
  if (rc == HALO_OK && pb->event_end) cudaEventRecord(static_cast<cudaEvent_t>(pb->event_end), st);
  return rc;
}

}  // namespace halo

using namespace halo;

extern "C" int32_t halo_prefill_attention(const halo_prefill_problem_t* pb,
                                          const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                          const halo_prefill_out_t* po, halo_stream_t stream) {
  return pf_run(pb, chunks, n_chunks, po, nullptr, 0, stream);
}

extern "C" int64_t halo_prefill_workspace_bytes(const halo_prefill_problem_t* pb,
                                                const halo_kv_chunk_t* chunks, int32_t n_chunks) {
  int rc = pf_check(pb, nullptr, false);
  if (rc != HALO_OK) return rc;
  PfSeg segs[prefill::kMaxSegs];
  int n_seg = 0;
  rc = pf_segments(chunks, n_chunks, segs, &n_seg);
  if (rc != HALO_OK) return rc;
  return pf_workspace_bytes(segs, n_seg, pb);
}

extern "C" int32_t halo_prefill_attention_ws(const halo_prefill_problem_t* pb,
                                             const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                             const halo_prefill_out_t* po, void* workspace,
                                             int64_t workspace_bytes, halo_stream_t stream) {
  return pf_run(pb, chunks, n_chunks, po, workspace, workspace_bytes, stream);
}
