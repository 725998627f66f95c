// Split-KV chunked decode attention + log-sum-exp merge for B200 (sm_100a).
//
// Replaces the reference's per-chunk Triton kernel (halo/triton_chunked.py:47-138,
// one program per (b, q-head), one launch per chunk, K/V re-read by every
// q-head of a GQA group) with:
//   * kd: a producer lane streams 64-row K/V tiles into a 3-stage
//     shared-memory ring with tensor TMA (cp.async.bulk.tensor + mbarrier
//     transaction counts); four consumer warps each own 16 rows of every
//     tile and attend ALL q-heads of the GQA group at once, so every K/V
//     byte is read from HBM exactly once.
//       - bf16/fp16: S = Q K^T and O += P V on tensor cores (mma.m16n8k16,
//         fp32 accumulate).  P is split into a 16-bit high part and a 16-bit
//         residual, so P V keeps ~16 mantissa bits (the reference's P is fp32).
//       - fp32: CUDA-core FMA (exact fp32 products and sums).
//     Online softmax in the exp2 domain with warp-shuffle row reductions.
//     kd_dyn_kernel (16-bit inputs, long contexts) hands the rows out at run
//     time from per-pair counters and writes one combined partial per CTA;
//     kd_kernel splits them statically (fp32, short contexts, or a fixed
//     max_split_rows, which is bit-reproducible).
//   * kk: the same pipeline over KIVI-packed K/V, dequantised per tile; GQA
//     groups of at most 8 q-heads use transposed tile math (keys as the MMA
//     rows), where 2-bit K goes straight into MMA registers (a permuted k
//     order gives each thread one quantisation group) and only V is staged
//     as a 16-bit tile in shared memory.
//   * km: one CTA per (b, q-head) row folds all partial states (and
//     optionally a prior running state) into the final output + LSE, or
//     into the running (m, l, o) accumulators of update_chunk.
// Every split-KV kernel is a programmatic dependent launch of its
// predecessor, and the merge one of the split-KV kernel, so consecutive
// kernels overlap launch and prologue with the previous kernel's tail.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <unordered_map>
#include <vector>

#include "halo_common.cuh"
#include "merge_row.cuh"

namespace halo {

__device__ unsigned int g_device_error = 0;

std::atomic<uint64_t> g_launch_count{0};

void count_launches(int n) { g_launch_count.fetch_add((uint64_t)n, std::memory_order_relaxed); }

unsigned int* device_error_ptr() {
  static std::mutex mu;
  static unsigned int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_device_error) == cudaSuccess)
      cache[dev] = static_cast<unsigned int*>(ptr);
  }
  return cache[dev];
}

// ---------------------------------------------------------------- config
constexpr int kBlockN = 64;          // K/V rows per pipeline stage (one TMA box high)
constexpr int kConsumerWarps = 4;    // each owns 16 rows of every stage
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxSegs = 48;         // tensor-map pairs per launch
constexpr float kLazyMax = 8.f;      // KIVI decode: log2 headroom before the running max moves
constexpr uint32_t kKiviWaitHintNs = 2000;  // KIVI decode: suspend-time hint of its ring waits
constexpr int kMaxItems = 512;       // work items per launch
// kCtrlBytes (halo_common.cuh): the control block at the start of every
// decode workspace.
constexpr int kMaxDynPairs = (int)(kCtrlBytes / 4) - 1;
constexpr int kPieceTiles = 2;       // 64-row tiles per piece of the dynamic schedule

// A work item: `rows` consecutive rows of one segment (a K/V view with its
// own pair of tensor maps), starting at segment row `row0`, whose first row
// sits at global position `start`.
struct Item {
  int64_t start;
  int32_t seg;
  int32_t row0;
  int32_t rows;
  int32_t slot;     // first partial slot; warp w writes slot + w
  int32_t causal;
  int32_t b_bcast;  // batch stride 0: every batch row reads batch 0
};

struct alignas(64) DecodeParams {
  CUtensorMap maps[2 * kMaxSegs];  // K, V tensor map per segment
  CUtensorMap qmap;                // q as {D, H, B}
  Item items[kMaxItems];
  const int64_t* q_pos;
  float* m_part;
  float* l_part;
  float* o_part;
  unsigned int* err;  // device error word
  unsigned int* ctrl; // dynamic schedule: counters[n_pairs], exit counter
  int32_t B, H, H_kv, G, gblocks;
  int32_t S;          // partial slots per (b, h) row
  int32_t n_items, n_units;
  int32_t n_pairs, n_dyn_tiles;  // dynamic schedule: pairs, 64-row tiles per pair
  float scale_log2;   // softmax scale * log2(e)
};
static_assert(sizeof(DecodeParams) <= 32764, "kernel parameter block limit");

// Parameter block of the dynamically scheduled decode for launches of at
// most kDynSegs segments: DecodeParams' fields with short tables, ~1.6 KB
// instead of ~29 KB.  A launch's parameter block travels through the GPU's
// command path; on B200 28 KB more of it costs ~2 us per launch.
constexpr int kDynSegs = 4;
struct alignas(64) DynParams {
  CUtensorMap maps[2 * kDynSegs];
  CUtensorMap qmap;
  Item items[kDynSegs];
  const int64_t* q_pos;
  float* m_part;
  float* l_part;
  float* o_part;
  unsigned int* err;
  unsigned int* ctrl;
  int32_t B, H, H_kv, G, gblocks;
  int32_t S;
  int32_t n_items, n_units;
  int32_t n_pairs, n_dyn_tiles;
  float scale_log2;
};


template <typename T, int D, int STAGES>
struct Geom {
  static constexpr int kElt = sizeof(T);
  static constexpr int kRowBytes = D * kElt;
  // TMA inner box: the largest of 128/64/32 bytes dividing a row; swizzle
  // mode of the same width.
  static constexpr int kInner = kRowBytes % 128 == 0 ? 128 : (kRowBytes % 64 == 0 ? 64 : 32);
  static constexpr int kBoxElems = kInner / kElt;
  static constexpr int kNBox = kRowBytes / kInner;     // boxes per row
  static constexpr int kBoxBytes = kBlockN * kInner;
  static constexpr int kTileBytes = kNBox * kBoxBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kGpb = (kElt == 4 ? 8 : 16);   // q-heads per unit
  static constexpr int kQSlotBytes = ((kNBox * kGpb * kInner) + 1023) / 1024 * 1024;
  static constexpr int kPBytes = (kElt == 4 ? kConsumerWarps * 16 * 8 * 4 : 0);
  static constexpr int kBarBytes = 128;
  // ring | q ring (2 slots) | P | barriers ; +1024 for manual alignment
  static constexpr int kSmemBytes =
      STAGES * kStageBytes + 2 * kQSlotBytes + kPBytes + kBarBytes + 1024;
  static_assert(kRowBytes % 32 == 0, "row must be a whole number of 32-byte TMA boxes");
  static_assert(kTileBytes % 1024 == 0, "tiles must keep 1024-byte alignment");
};

struct Unit {
  int item, b, h_kv, gbase, gcount;
};

template <class P>
__device__ __forceinline__ Unit decode_unit(const P& p, int u, int gpb) {
  Unit r;
  r.item = u % p.n_items;
  int pair = u / p.n_items;
  const int gb = pair % p.gblocks;
  pair /= p.gblocks;
  r.h_kv = pair % p.H_kv;
  r.b = pair / p.H_kv;
  r.gbase = gb * gpb;
  r.gcount = min(gpb, p.G - r.gbase);
  return r;
}

// Write one warp's partial state for q-head rows [gbase, gbase+gcount).
template <class P>
__device__ __forceinline__ void write_partial_meta(const P& p, const Unit& un,
                                                   const Item& it, int warp, int g, float m_log2,
                                                   float l) {
  const int h = un.h_kv * p.G + un.gbase + g;
  const int64_t row = ((int64_t)un.b * p.H + h) * p.S + it.slot + warp;
  p.m_part[row] = (m_log2 == -INFINITY) ? -INFINITY : m_log2 * kLn2;
  p.l_part[row] = l;
}

// ---------------------------------------------------------------- consumers
// 16-bit inputs: tensor-core path.  Warp `w` handles rows [16w, 16w+16) of
// every stage; the 16 query rows of the MMA are the unit's q-heads.
// K/V tiles from the TMA ring: wait for stage `gt % STAGES`, hand out its
// K and V tile addresses, release the stage after the tile is consumed.
template <int STAGES, int STAGE_BYTES, int TILE_BYTES>
struct RingTiles {
  char* ring;
  uint64_t* full;
  uint64_t* empty;
  unsigned int* err;
  __device__ __forceinline__ bool acquire(int t, int gt, uint32_t& kbase, uint32_t& vbase) {
    const int s = gt % STAGES;
    if (!mbar_wait(&full[s], (gt / STAGES) & 1, err)) return false;
    kbase = smem_addr(ring + s * STAGE_BYTES);
    vbase = kbase + TILE_BYTES;
    return true;
  }
  __device__ __forceinline__ void release(int gt) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[gt % STAGES]);
  }
};

// Q fragments (A operand) of all k-steps from a swizzled q tile.
template <typename T, int D, int STAGES>
__device__ __forceinline__ void load_q_frags(const char* qslot, uint32_t (&qf)[D / 16][4]) {
  using Gm = Geom<T, D, STAGES>;
  const int lane = threadIdx.x & 31;
  const uint32_t qb = smem_addr(qslot);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int row = lane & 15;
    const int c16 = kk * 2 + (lane >> 4);
    ldsm_x4(qb + swz<Gm::kInner, Gm::kGpb>(row, c16), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }
}

// One 64-row K/V tile on the tensor cores for this warp's 16 rows of it:
// S = Q K^T (16 q-heads x 16 keys), scale + mask, online softmax (rows
// g0 = lane/4 and g1 = lane/4 + 8 of the q-head block), O += P V with
// P = hi + lo (two 16-bit MMAs).  Row r of the tile (0..63) is a key if
// r < valid and, for a causal tile, pos0 + r <= qpos.
template <typename T, int D, int STAGES>
__device__ __forceinline__ void mma_tile(float scale_log2, uint32_t kbase, uint32_t vbase,
                                         const uint32_t (&qf)[D / 16][4], float (&o)[D / 8][4],
                                         float& m0, float& m1, float& l0, float& l1, int valid,
                                         int64_t pos0, bool causal, int64_t qpos) {
  using Gm = Geom<T, D, STAGES>;
  const int lane = threadIdx.x & 31;
  const int wrow = (threadIdx.x >> 5) * 16;
  const int c = lane & 3;

  // ---- S = Q K^T
  float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  {
    const int key = wrow + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int c16 = kk * 2 + ((lane >> 3) & 1);
      uint32_t b00, b01, b10, b11;
      ldsm_x4(kbase + swz<Gm::kInner>(key, c16), b00, b01, b10, b11);
      mma_16816(sacc[0], qf[kk], b00, b01, (T*)nullptr);
      mma_16816(sacc[1], qf[kk], b10, b11, (T*)nullptr);
    }
  }

  // ---- scale + mask (rows beyond the valid range, or causally hidden)
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int r = wrow + nt * 8 + 2 * c + e;
      const bool ok = r < valid && (!causal || pos0 + r <= qpos);
      sacc[nt][e] = ok ? sacc[nt][e] * scale_log2 : -INFINITY;
      sacc[nt][e + 2] = ok ? sacc[nt][e + 2] * scale_log2 : -INFINITY;
    }

  // ---- online softmax
  float r0 = fmaxf(fmaxf(sacc[0][0], sacc[0][1]), fmaxf(sacc[1][0], sacc[1][1]));
  float r1 = fmaxf(fmaxf(sacc[0][2], sacc[0][3]), fmaxf(sacc[1][2], sacc[1][3]));
  r0 = fmaxf(r0, __shfl_xor_sync(0xffffffffu, r0, 1));
  r0 = fmaxf(r0, __shfl_xor_sync(0xffffffffu, r0, 2));
  r1 = fmaxf(r1, __shfl_xor_sync(0xffffffffu, r1, 1));
  r1 = fmaxf(r1, __shfl_xor_sync(0xffffffffu, r1, 2));
  const float mn0 = fmaxf(m0, r0), mn1 = fmaxf(m1, r1);
  const float mu0 = (mn0 == -INFINITY) ? 0.f : mn0;
  const float mu1 = (mn1 == -INFINITY) ? 0.f : mn1;
  const float a0 = exp2f(m0 - mu0), a1 = exp2f(m1 - mu1);
  m0 = mn0;
  m1 = mn1;
  float pr[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    pr[nt][0] = exp2f(sacc[nt][0] - mu0);
    pr[nt][1] = exp2f(sacc[nt][1] - mu0);
    pr[nt][2] = exp2f(sacc[nt][2] - mu1);
    pr[nt][3] = exp2f(sacc[nt][3] - mu1);
  }
  l0 = l0 * a0 + (pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1]);
  l1 = l1 * a1 + (pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3]);
  if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= a0;
      o[i][1] *= a0;
      o[i][2] *= a1;
      o[i][3] *= a1;
    }
  }

  // ---- O += P V with P = hi + lo (two 16-bit MMAs)
  uint32_t ph[4], pl[4];
  {
    const float v[4][2] = {{pr[0][0], pr[0][1]}, {pr[0][2], pr[0][3]},
                           {pr[1][0], pr[1][1]}, {pr[1][2], pr[1][3]}};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      ph[r] = Elem<T>::pack(v[r][0], v[r][1]);
      float h0, h1;
      Elem<T>::unpack(ph[r], h0, h1);
      pl[r] = Elem<T>::pack(v[r][0] - h0, v[r][1] - h1);
    }
  }
  {
    const int key = wrow + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
      const int c16 = j * 2 + (lane >> 4);
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(vbase + swz<Gm::kInner>(key, c16), v0, v1, v2, v3);
      mma_16816(o[2 * j], ph, v0, v1, (T*)nullptr);
      mma_16816(o[2 * j], pl, v0, v1, (T*)nullptr);
      mma_16816(o[2 * j + 1], ph, v2, v3, (T*)nullptr);
      mma_16816(o[2 * j + 1], pl, v2, v3, (T*)nullptr);
    }
  }
}

// This warp's partial state (m, l, o) of the unit's q-heads -> partial slot
// `slot` of each (b, h) row (rows < gcount only).
template <int D, class P>
__device__ __forceinline__ void store_partial_mma(const P& p, const Unit& un, int slot,
                                                  const float (&o)[D / 8][4], float m0, float m1,
                                                  float l0, float l1) {
  const int lane = threadIdx.x & 31;
  const int c = lane & 3;
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const int g0 = lane >> 2;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int g = g0 + 8 * half;
    if (g < un.gcount) {
      const int h = un.h_kv * p.G + un.gbase + g;
      const int64_t row = ((int64_t)un.b * p.H + h) * p.S + slot;
      if (c == 0) {
        const float m = half ? m1 : m0;
        p.m_part[row] = (m == -INFINITY) ? -INFINITY : m * kLn2;
        p.l_part[row] = half ? l1 : l0;
      }
      float* op = p.o_part + row * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<float2*>(op + i * 8 + 2 * c) =
            make_float2(o[i][2 * half], o[i][2 * half + 1]);
    }
  }
}

template <typename T, int D, int STAGES, class P, class Tiles>
__device__ __forceinline__ bool consume_mma(const P& p, const Unit& un, const Item& it,
                                            Tiles& tiles, const char* qslot,
                                            uint64_t* qempty, int n_tiles,
                                            int& gt, int64_t qpos) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint32_t qf[D / 16][4];
  load_q_frags<T, D, STAGES>(qslot, qf);
  __syncwarp();
  if (lane == 0) mbar_arrive(qempty);

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  bool ok = true;
  for (int t = 0; t < n_tiles; ++t, ++gt) {
    uint32_t kbase, vbase;
    if (!tiles.acquire(t, gt, kbase, vbase)) { ok = false; ++gt; break; }
    mma_tile<T, D, STAGES>(p.scale_log2, kbase, vbase, qf, o, m0, m1, l0, l1,
                           it.rows - t * kBlockN, it.start + (int64_t)t * kBlockN,
                           it.causal != 0, qpos);
    tiles.release(gt);
  }
  store_partial_mma<D>(p, un, it.slot + warp, o, m0, m1, l0, l1);
  return ok;
}

// ---- transposed tile math for GQA groups of at most 8 q-heads
// S^T = K Q^T with the 16 keys of the warp as the MMA's M rows and the
// q-heads as its 8 columns, and O^T = V^T P^T: half the MMAs of the
// q-heads-as-rows form (whose 16 rows are mostly empty for G <= 8) and half
// the accumulator registers (O^T is D x 8), so more CTAs fit on an SM.
// Thread t holds heads 2(t%4), 2(t%4)+1 and keys t/4, t/4 + 8 of the warp's
// 16; the per-head max over keys is a reduction across the eight lanes that
// share t%4.  P^T goes from the S^T accumulator layout to the B operand of
// the P V product with one movmatrix transpose per 8x8 block.

// Q^T fragments (B operand) of all k-steps: q-heads as columns.
template <typename T, int D, int STAGES>
__device__ __forceinline__ void load_qT_frags(const char* qslot, uint32_t (&qb)[D / 16][2]) {
  using Gm = Geom<T, D, STAGES>;
  static_assert(D % 32 == 0, "two k-steps per ldmatrix.x4");
  const int lane = threadIdx.x & 31;
  const uint32_t base = smem_addr(qslot);
#pragma unroll
  for (int kk = 0; kk < D / 16; kk += 2)
    ldsm_x4(base + swz<Gm::kInner, Gm::kGpb>(lane & 7, kk * 2 + (lane >> 3)), qb[kk][0],
            qb[kk][1], qb[kk + 1][0], qb[kk + 1][1]);
}

// ---- K-direct (2-bit codes, transposed tile math).  Thread (g, c) of a
// warp (g = lane / 4, c = lane % 4) owns the K elements of its rows g and
// g + 8 in head-dim columns [c*D/4, (c+1)*D/4): one quantisation group
// (half of one for D = 64), so one scale and zero per row.  The S^T
// MMAs take K in a permuted k order: logical column 2c + e + 8h of k-step kk
// is head-dim column c*D/4 + 4kk + 2h + e.  A permutation of k leaves
// sum_k K Q^T unchanged when Q^T is loaded in the same order, and in this
// one a thread's A-fragment pairs are consecutive elements of its own
// group: K is dequantised straight into A-operand registers, with no
// shared-memory round trip.

// Q^T fragments (B operand) in the permuted k order: qb[kk] holds head g's
// columns c*D/4 + 4kk .. + 4, i.e. 16 consecutive bytes per two k-steps.
template <typename T, int D, int STAGES>
__device__ __forceinline__ void load_qT_frags_perm(const char* qslot, uint32_t (&qb)[D / 16][2]) {
  using Gm = Geom<T, D, STAGES>;
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const uint32_t base = smem_addr(qslot);
#pragma unroll
  for (int m = 0; m < D / 32; ++m)
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(qb[2 * m][0]), "=r"(qb[2 * m][1]), "=r"(qb[2 * m + 1][0]),
                   "=r"(qb[2 * m + 1][1])
                 : "r"(base + swz<Gm::kInner, Gm::kGpb>(g, c * (D / 32) + m)));
}

// ---- 2-bit codes to 16-bit values without the integer pipe
// Packed 2-bit layout: code e (0..15) of each 16-code block at bit
// 16*(e & 1) + 2*(e >> 1) of the block's little-endian 32-bit word, so the
// two codes of pair q = (2q, 2q+1) sit at the same bit 2q of the word's two
// 16-bit halves.  One LOP3 ((w & (0x00030003 << 2q)) | M_q) puts them into
// the mantissas of two 16-bit floats whose exponent makes bit 2q worth 1:
// each half reads E_q + c exactly, and a packed subtract of E_q leaves the
// codes as exact small floats; one packed FMA then gives c*s + z rounded once
// to the 16-bit type (the reference rounds c*s + z to fp32 first; with
// c <= 3 and s, z 16-bit that only differs when the exact sum lies within
// 2^-23 of a 16-bit rounding midpoint).  Pairs whose bits would reach the
// exponent field are taken from the word shifted right first.  Two 16-bit
// values per LOP3 and two per FMA-pipe instruction, instead of byte permutes
// on the integer pipe.
template <typename T>
struct Code2;
template <>
struct Code2<__half> {
  static constexpr int kPairsPerShift = 5;         // bits 0..9 of the mantissa
  static constexpr int kShiftBits = 10;
  // 2^(10 - 2q) in both halves: exponent 25 - 2q
  __host__ __device__ static constexpr uint32_t magic(int q) {
    return ((uint32_t)(25 - 2 * q) << 10) | ((uint32_t)(25 - 2 * q) << 26);
  }
};
template <>
struct Code2<__nv_bfloat16> {
  static constexpr int kPairsPerShift = 3;         // bits 0..5 of the mantissa
  static constexpr int kShiftBits = 6;
  // 2^(7 - 2q) in both halves: exponent 134 - 2q
  __host__ __device__ static constexpr uint32_t magic(int q) {
    return ((uint32_t)(134 - 2 * q) << 7) | ((uint32_t)(134 - 2 * q) << 23);
  }
};

// (w & mask) | magic, minus magic as two 16-bit floats, times s plus z: one
// LOP3 and two packed 16-bit instructions, with the magic constant as the
// operand of both the LOP3 and the subtract.
template <typename T>
__device__ __forceinline__ uint32_t code2_decode(uint32_t w, uint32_t mask, uint32_t magic,
                                                 uint32_t s2, uint32_t z2) {
  uint32_t r;
  if constexpr (std::is_same<T, __half>::value)
    asm("{\n\t.reg .b32 t;\n\t"
        "lop3.b32 t, %1, %2, %3, 0xEA;\n\t"
        "sub.f16x2 t, t, %3;\n\t"
        "fma.rn.f16x2 %0, t, %4, %5;\n\t}"
        : "=r"(r) : "r"(w), "r"(mask), "r"(magic), "r"(s2), "r"(z2));
  else
    asm("{\n\t.reg .b32 t;\n\t"
        "lop3.b32 t, %1, %2, %3, 0xEA;\n\t"
        "sub.bf16x2 t, t, %3;\n\t"
        "fma.rn.bf16x2 %0, t, %4, %5;\n\t}"
        : "=r"(r) : "r"(w), "r"(mask), "r"(magic), "r"(s2), "r"(z2));
  return r;
}

// Values of pair p (0..7) of a 16-code word: codes 2p and 2p+1 as one
// register of two 16-bit values c*s + z.
template <typename T>
__device__ __forceinline__ uint32_t code2_pair(uint32_t word, int p, uint32_t s2, uint32_t z2) {
  using C = Code2<T>;
  const int seg = p / C::kPairsPerShift, q = p % C::kPairsPerShift;
  const uint32_t w = seg ? (word >> (seg * C::kShiftBits)) : word;
  return code2_decode<T>(w, 0x00030003u << (2 * q), C::magic(q), s2, z2);
}

// This thread's packed K codes (rows g, g + 8; D/4 codes each, the span of
// one quantisation group, as the packed format stores them) and the group's
// scale and zero of each row, duplicated into both 16-bit halves.
template <int D>
struct KRegs {
  uint32_t words[2][D / 64];
  uint32_t s2[2], z2[2];
};

template <typename T, int D>
__device__ __forceinline__ void load_k_regs(const char* pack, int code_tile, int sz_tile,
                                            KRegs<D>& kr) {
  constexpr int kSpan = D / 4;          // head-dim columns of one thread
  constexpr int kCB = D / 4;            // 2-bit code bytes per row
  constexpr int kGS = D / 32;           // groups per row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int gi = (c * kSpan) / 32;      // the thread's quantisation group
  const uint32_t s_codes = smem_addr(pack) + c * (kSpan / 4);
  const uint32_t s_sc = smem_addr(pack + code_tile) + 2 * gi;
  const uint32_t s_ze = smem_addr(pack + code_tile + sz_tile) + 2 * gi;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = warp * 16 + g + 8 * r;
    if constexpr (D == 128)
      asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];"
                   : "=r"(kr.words[r][0]), "=r"(kr.words[r][1])
                   : "r"(s_codes + row * kCB));
    else
      asm volatile("ld.shared.u32 %0, [%1];" : "=r"(kr.words[r][0]) : "r"(s_codes + row * kCB));
    uint16_t sb, zb;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sb) : "r"(s_sc + row * kGS * 2));
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(zb) : "r"(s_ze + row * kGS * 2));
    kr.s2[r] = (uint32_t)sb | ((uint32_t)sb << 16);
    kr.z2[r] = (uint32_t)zb | ((uint32_t)zb << 16);
  }
}

// A fragments of k-step kk: span elements 4kk + 2h + {0, 1} (pair 2kk + h of
// the span) of rows g (a0, a2) and g + 8 (a1, a3).
template <typename T, int D>
__device__ __forceinline__ void k_frag(const KRegs<D>& kr, int kk, uint32_t (&a)[4]) {
  const int w = kk >> 2, p = 2 * (kk & 3);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    a[r] = code2_pair<T>(kr.words[r][w], p, kr.s2[r], kr.z2[r]);
    a[2 + r] = code2_pair<T>(kr.words[r][w], p + 1, kr.s2[r], kr.z2[r]);
  }
}

template <typename T, int D, int STAGES, class KFrag>
__device__ __forceinline__ void mma_tile_t(float scale_log2, const KFrag& kfrag, uint32_t vbase,
                                           const uint32_t (&qb)[D / 16][2],
                                           float (&o)[D / 16][4], float& m0, float& m1, float& l0,
                                           float& l1, int valid, int64_t pos0, bool causal,
                                           int64_t qpos) {
  using Gm = Geom<T, D, STAGES>;
  const int lane = threadIdx.x & 31;
  const int wrow = (threadIdx.x >> 5) * 16;
  const int g = lane >> 2;

  // ---- S^T = K Q^T (16 keys x 8 heads); kfrag(kk, a) gives k-step kk's
  // A fragments (the warp's 16 keys)
  float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t a[4];
    kfrag(kk, a);
    mma_16816(s, a, qb[kk][0], qb[kk][1], (T*)nullptr);
  }

  // ---- mask, only on a tile that ends early or crosses the causal limit
  // (warp-uniform test): s[0], s[1] are key g, s[2], s[3] key g + 8
  if (valid < kBlockN || (causal && pos0 + (kBlockN - 1) > qpos)) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = wrow + g + ((e >> 1) << 3);
      if (!(r < valid && (!causal || pos0 + r <= qpos))) s[e] = -INFINITY;
    }
  }

  // ---- online softmax per head (columns 2c, 2c+1) in log2 units.  The
  // running max moves only when a key exceeds it by more than kLazyMax:
  // P = exp2(s - m) then stays <= 2^kLazyMax (exact to 16-bit rounding, far
  // from fp16 overflow) and most tiles skip the cross-lane max and the
  // rescale of O.
  float t0 = fmaxf(s[0], s[2]) * scale_log2, t1 = fmaxf(s[1], s[3]) * scale_log2;
  if (__any_sync(0xffffffffu, t0 > m0 + kLazyMax || t1 > m1 + kLazyMax)) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, off));
      t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, off));
    }
    const float mn0 = fmaxf(m0, t0), mn1 = fmaxf(m1, t1);
    const float a0 = (m0 == -INFINITY) ? 0.f : ex2(m0 - mn0);
    const float a1 = (m1 == -INFINITY) ? 0.f : ex2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    l0 *= a0;
    l1 *= a1;
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
      o[i][0] *= a0;
      o[i][1] *= a1;
      o[i][2] *= a0;
      o[i][3] *= a1;
    }
  }
  // -m (0 while a head has seen no key, so masked scores give exp2(-inf) = 0)
  const float nm0 = (m0 == -INFINITY) ? 0.f : -m0;
  const float nm1 = (m1 == -INFINITY) ? 0.f : -m1;
  const float p0 = ex2(fmaf(s[0], scale_log2, nm0)), p1 = ex2(fmaf(s[1], scale_log2, nm1));
  const float p2 = ex2(fmaf(s[2], scale_log2, nm0)), p3 = ex2(fmaf(s[3], scale_log2, nm1));
  l0 += p0 + p2;      // this thread's keys; reduced over lanes at the end
  l1 += p1 + p3;

  // ---- P^T transposed into the B operand (keys x heads).  fp16 keeps 11
  // significant bits of P (relative error <= 2^-11) in one MMA; bf16 keeps
  // 8, so its P is split into hi + lo (two MMAs, ~16 bits).
  constexpr bool kSplitP = !std::is_same<T, __half>::value;
  uint32_t bh[2], bl[2] = {0u, 0u};
  {
    const uint32_t h0 = Elem<T>::pack(p0, p1), h1 = Elem<T>::pack(p2, p3);
    bh[0] = movmatrix_t(h0);
    bh[1] = movmatrix_t(h1);
    if constexpr (kSplitP) {
      float x0, x1, x2, x3;
      Elem<T>::unpack(h0, x0, x1);
      Elem<T>::unpack(h1, x2, x3);
      const uint32_t r0 = Elem<T>::pack(p0 - x0, p1 - x1), r1 = Elem<T>::pack(p2 - x2, p3 - x3);
      bl[0] = movmatrix_t(r0);
      bl[1] = movmatrix_t(r1);
    }
  }

  // ---- O^T += V^T P^T, 16 rows of d at a time
  {
    const int key = wrow + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
      uint32_t a[4];
      ldsm_x4_t(vbase + swz<Gm::kInner>(key, i * 2 + ((lane >> 3) & 1)), a[0], a[1], a[2], a[3]);
      mma_16816(o[i], a, bh[0], bh[1], (T*)nullptr);
      if constexpr (kSplitP) mma_16816(o[i], a, bl[0], bl[1], (T*)nullptr);
    }
  }
}

// This warp's transposed partial state -> partial slot `slot` of its heads.
template <int D, class P>
__device__ __forceinline__ void store_partial_t(const P& p, const Unit& un, int slot,
                                                const float (&o)[D / 16][4], float m0, float m1,
                                                float l0, float l1) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int hl = 2 * c + e;
    if (hl < un.gcount) {
      const int h = un.h_kv * p.G + un.gbase + hl;
      const int64_t row = ((int64_t)un.b * p.H + h) * p.S + slot;
      if (g == 0) {
        const float m = e ? m1 : m0;
        p.m_part[row] = (m == -INFINITY) ? -INFINITY : m * kLn2;
        p.l_part[row] = e ? l1 : l0;
      }
      float* op = p.o_part + row * D;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        op[i * 16 + g] = o[i][e];
        op[i * 16 + g + 8] = o[i][e + 2];
      }
    }
  }
}

template <typename T, int D, int STAGES, class P, class Tiles>
__device__ __forceinline__ bool consume_mma_t(const P& p, const Unit& un, const Item& it,
                                              Tiles& tiles, const char* qslot, uint64_t* qempty,
                                              int n_tiles, int& gt, int64_t qpos) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint32_t qb[D / 16][2];
  if constexpr (Tiles::kKDirect)
    load_qT_frags_perm<T, D, STAGES>(qslot, qb);
  else
    load_qT_frags<T, D, STAGES>(qslot, qb);
  __syncwarp();
  if (lane == 0) mbar_arrive(qempty);

  float o[D / 16][4];
#pragma unroll
  for (int i = 0; i < D / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  bool ok = true;
  for (int t = 0; t < n_tiles; ++t, ++gt) {
    uint32_t kbase, vbase;
    if (!tiles.acquire(t, gt, kbase, vbase)) { ok = false; ++gt; break; }
    const int valid = it.rows - t * kBlockN;
    const int64_t pos0 = it.start + (int64_t)t * kBlockN;
    if constexpr (Tiles::kKDirect) {
      auto kf = [&](int kk, uint32_t (&a)[4]) { k_frag<T, D>(tiles.kr, kk, a); };
      mma_tile_t<T, D, STAGES>(p.scale_log2, kf, vbase, qb, o, m0, m1, l0, l1, valid, pos0,
                               it.causal != 0, qpos);
    } else {
      using Gm = Geom<T, D, STAGES>;
      const int key = warp * 16 + (lane & 15);
      auto kf = [&](int kk, uint32_t (&a)[4]) {
        ldsm_x4(kbase + swz<Gm::kInner>(key, kk * 2 + (lane >> 4)), a[0], a[1], a[2], a[3]);
      };
      mma_tile_t<T, D, STAGES>(p.scale_log2, kf, vbase, qb, o, m0, m1, l0, l1, valid, pos0,
                               it.causal != 0, qpos);
    }
    tiles.release(gt);
  }
  store_partial_t<D>(p, un, it.slot + warp, o, m0, m1, l0, l1);
  return ok;
}

// fp32 inputs: CUDA-core FMA path, up to 8 q-heads per unit.  For S, lane
// pair (2k, 2k+1) owns key k of the warp's 16 rows, each lane one half of
// the row's 16-byte chunks; for P V lane l owns output columns l, l+32, ...
template <int D, int STAGES>
__device__ __forceinline__ bool consume_fma(const DecodeParams& p, const Unit& un, const Item& it,
                                            char* ring, const char* qslot, float* ps_all,
                                            uint64_t* full, uint64_t* empty, uint64_t* qempty,
                                            int n_tiles, int& gt, int64_t qpos) {
  using Gm = Geom<float, D, STAGES>;
  constexpr int GP = 8;
  constexpr int DPL = (D + 31) / 32;   // output columns per lane (strided by 32)
  constexpr int NCH = D / 4;           // 16-byte chunks per row
  constexpr int HALF = (NCH + 1) / 2;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float* ps = ps_all + warp * 16 * GP;
  const int gcount = un.gcount;

  float o[GP][DPL];
  float m[GP], l[GP];
#pragma unroll
  for (int g = 0; g < GP; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[g][e] = 0.f;
  }
  const int key = lane >> 1, half = lane & 1;
  const int item_end = it.row0 + it.rows;
  const int wrow = warp * 16;
  bool ok = true;

  for (int t = 0; t < n_tiles; ++t, ++gt) {
    const int s = gt % STAGES;
    if (!mbar_wait(&full[s], (gt / STAGES) & 1, p.err)) { ok = false; ++gt; break; }
    const char* kt = ring + s * Gm::kStageBytes;
    const char* vt = kt + Gm::kTileBytes;

    float acc[GP];
#pragma unroll
    for (int g = 0; g < GP; ++g) acc[g] = 0.f;
#pragma unroll 4
    for (int i = 0; i < HALF; ++i) {
      const int j = half * HALF + i;
      if (j < NCH) {
        const float4 kv = *reinterpret_cast<const float4*>(kt + swz<Gm::kInner>(wrow + key, j));
#pragma unroll
        for (int g = 0; g < GP; ++g) {
          if (g < gcount) {
            const float4 qv =
                *reinterpret_cast<const float4*>(qslot + swz<Gm::kInner, GP>(g, j));
            acc[g] = fmaf(qv.x, kv.x, acc[g]);
            acc[g] = fmaf(qv.y, kv.y, acc[g]);
            acc[g] = fmaf(qv.z, kv.z, acc[g]);
            acc[g] = fmaf(qv.w, kv.w, acc[g]);
          }
        }
      }
    }
    const int row = it.row0 + t * kBlockN + wrow + key;
    const bool valid = row < item_end && (!it.causal || it.start + (row - it.row0) <= qpos);
    float pk[GP];
#pragma unroll
    for (int g = 0; g < GP; ++g) {
      float sv = acc[g] + __shfl_xor_sync(0xffffffffu, acc[g], 1);
      sv = valid ? sv * p.scale_log2 : -INFINITY;
      float mt = sv;
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float mn = fmaxf(m[g], mt);
      const float mu = (mn == -INFINITY) ? 0.f : mn;
      const float a = exp2f(m[g] - mu);
      m[g] = mn;
      pk[g] = exp2f(sv - mu);
      l[g] = l[g] * a + (half == 0 ? pk[g] : 0.f);
#pragma unroll
      for (int e = 0; e < DPL; ++e) o[g][e] *= a;
    }
    if (half == 0) {
#pragma unroll
      for (int g = 0; g < GP; ++g) ps[key * GP + g] = pk[g];
    }
    __syncwarp();
#pragma unroll 4
    for (int kr = 0; kr < 16; ++kr) {
      float vv[DPL];
#pragma unroll
      for (int e = 0; e < DPL; ++e) {
        const int d = lane + 32 * e;
        vv[e] = d < D ? *reinterpret_cast<const float*>(vt + swz<Gm::kInner>(wrow + kr, d >> 2) +
                                                       ((d & 3) << 2))
                      : 0.f;
      }
      const float4 p03 = *reinterpret_cast<const float4*>(ps + kr * GP);
      const float4 p47 = *reinterpret_cast<const float4*>(ps + kr * GP + 4);
      const float pp[8] = {p03.x, p03.y, p03.z, p03.w, p47.x, p47.y, p47.z, p47.w};
#pragma unroll
      for (int g = 0; g < GP; ++g)
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(pp[g], vv[e], o[g][e]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // Q stays in shared memory for the whole unit on this path.
  __syncwarp();
  if (lane == 0) mbar_arrive(qempty);

#pragma unroll
  for (int g = 0; g < GP; ++g) {
    float v = l[g];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    l[g] = v;
  }
#pragma unroll
  for (int g = 0; g < GP; ++g) {
    if (g < gcount) {
      if (lane == 0) write_partial_meta(p, un, it, warp, g, m[g], l[g]);
      const int h = un.h_kv * p.G + un.gbase + g;
      float* op = p.o_part + (((int64_t)un.b * p.H + h) * p.S + it.slot + warp) * D;
#pragma unroll
      for (int e = 0; e < DPL; ++e)
        if (lane + 32 * e < D) op[lane + 32 * e] = o[g][e];
    }
  }
  return ok;
}

// ---------------------------------------------------------------- kd kernel
// Persistent: CTA c processes units c, c + gridDim.x, ...  The producer lane
// streams every tile of every unit through one STAGES-deep ring (and each
// unit's q tile through a 2-slot ring) without pausing at unit boundaries.
template <typename T, int D, int STAGES, int MINB>
__global__ void __launch_bounds__(kThreads, MINB) kd_kernel(const __grid_constant__ DecodeParams p) {
  using Gm = Geom<T, D, STAGES>;
  extern __shared__ char smem_raw[];
  char* ring = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  char* qring = ring + STAGES * Gm::kStageBytes;
  float* ps = reinterpret_cast<float*>(qring + 2 * Gm::kQSlotBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(qring + 2 * Gm::kQSlotBytes + Gm::kPBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* qfull = empty + STAGES;
  uint64_t* qempty = qfull + 2;

  // the merge launched after this kernel may be scheduled from now on; it
  // waits for this grid to finish before reading the partials
  grid_dep_trigger();
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qempty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // launched as a dependent of the previous kernel on the stream: the
  // prologue above overlapped its tail; nothing it may have written (q,
  // K/V, positions, the workspace) is touched before it has completed
  grid_dep_wait();
  const int warp = tid >> 5, lane = tid & 31;

  if (warp == kConsumerWarps) {
    // ---------------- producer warp: lane 0 issues every TMA load
    if (lane == 0) {
      int gt = 0, ut = 0;
      for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++ut) {
        const Unit un = decode_unit(p, u, Gm::kGpb);
        const Item& it = p.items[un.item];
        const int qs = ut & 1;
        if (ut >= 2 && !mbar_wait(&qempty[qs], ((ut >> 1) & 1) ^ 1, p.err)) return;
        mbar_arrive_expect_tx(&qfull[qs], Gm::kNBox * Gm::kGpb * Gm::kInner);
#pragma unroll
        for (int bx = 0; bx < Gm::kNBox; ++bx)
          tma_load_3d(qring + qs * Gm::kQSlotBytes + bx * Gm::kGpb * Gm::kInner, &p.qmap,
                      bx * Gm::kBoxElems, un.h_kv * p.G + un.gbase, un.b, &qfull[qs]);
        const CUtensorMap* kmap = &p.maps[2 * it.seg];
        const CUtensorMap* vmap = &p.maps[2 * it.seg + 1];
        const int bc = it.b_bcast ? 0 : un.b;
        const int n_tiles = (it.rows + kBlockN - 1) / kBlockN;
        for (int t = 0; t < n_tiles; ++t, ++gt) {
          const int s = gt % STAGES;
          if (gt >= STAGES && !mbar_wait(&empty[s], ((gt / STAGES) & 1) ^ 1, p.err)) return;
          const int r0 = it.row0 + t * kBlockN;
          char* kd = ring + s * Gm::kStageBytes;
          char* vd = kd + Gm::kTileBytes;
          mbar_arrive_expect_tx(&full[s], 2u * Gm::kTileBytes);
#pragma unroll
          for (int bx = 0; bx < Gm::kNBox; ++bx) {
            tma_load_4d(kd + bx * Gm::kBoxBytes, kmap, bx * Gm::kBoxElems, r0, un.h_kv, bc, &full[s]);
            tma_load_4d(vd + bx * Gm::kBoxBytes, vmap, bx * Gm::kBoxElems, r0, un.h_kv, bc, &full[s]);
          }
        }
      }
    }
    return;
  }

  // ---------------- consumer warps
  int gt = 0, ut = 0;
  for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++ut) {
    const Unit un = decode_unit(p, u, Gm::kGpb);
    const Item& it = p.items[un.item];
    const int qs = ut & 1;
    if (!mbar_wait(&qfull[qs], (ut >> 1) & 1, p.err)) return;
    const int64_t qpos = (it.causal && p.q_pos != nullptr) ? p.q_pos[un.b] : INT64_MAX;
    const int n_tiles = (it.rows + kBlockN - 1) / kBlockN;
    bool ok;
    if constexpr (sizeof(T) == 4)
      ok = consume_fma<D, STAGES>(p, un, it, ring, qring + qs * Gm::kQSlotBytes, ps, full, empty,
                                  &qempty[qs], n_tiles, gt, qpos);
    else {
      RingTiles<STAGES, Gm::kStageBytes, Gm::kTileBytes> tiles{ring, full, empty, p.err};
      ok = consume_mma<T, D, STAGES>(p, un, it, tiles, qring + qs * Gm::kQSlotBytes, &qempty[qs],
                                     n_tiles, gt, qpos);
    }
    if (!ok) return;  // the error word is set; remaining units are abandoned
  }
}

// ---------------------------------------------------------------- kd, dynamic schedule
// Same tile math as kd_kernel, but the rows are handed out at run time.
// Each (batch, kv-head, q-head block) pair gets a group of CTAs: CTA c
// serves pair c % n_pairs and is member c / n_pairs of its group.  The
// pair's rows (every segment of the launch, in order) are numbered in 64-row
// tiles, and the group's producer lanes take them from the pair's counter
// in the workspace control block, kPieceTiles at a time and one at a time
// near the end.  CTAs on SMs that stream faster take more tiles and the
// group finishes within about one tile of each other (a static split leaves
// the CTAs of slower SMs finishing ~15 % after the median).  Each consumer
// warp folds every tile its CTA takes into one running state; at the end
// the four warps' states
// are combined through shared memory into the CTA's partial, slot `member`
// (so a row has one partial per CTA of its group).  The
// producer tells the consumers what each stage holds through a per-stage
// descriptor written before the stage's barrier arrival; a descriptor with
// no rows ends the work.  Every CTA's producer lane counts itself out on the
// control block's exit counter after its last take and once its consumers
// are done; the last one zeroes the counters for the next call.
struct TileDesc {
  int64_t pos0;    // global position of the tile's first row
  int32_t valid;   // rows of the tile inside its segment; 0 = no more work
  int32_t causal;
};

template <typename T, int D, int STAGES>
struct DynGeom {
  using Gm = Geom<T, D, STAGES>;
  static constexpr int kDescOff = Gm::kSmemBytes - 1024;   // after the barrier block
  static constexpr int kSmemBytes = Gm::kSmemBytes + 128;
  static_assert(STAGES * (int)sizeof(TileDesc) + 8 <= 128, "descriptor area");
};

template <typename T, int D, int STAGES, int MINB, class P>
__global__ void __launch_bounds__(kThreads, MINB)
    kd_dyn_kernel(const __grid_constant__ P p) {
  using Gm = Geom<T, D, STAGES>;
  using DG = DynGeom<T, D, STAGES>;
  extern __shared__ char smem_raw[];
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  char* ring = base;
  char* qslot = ring + STAGES * Gm::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(qslot + 2 * Gm::kQSlotBytes + Gm::kPBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* qfull = empty + STAGES;
  TileDesc* desc = reinterpret_cast<TileDesc*>(base + DG::kDescOff);
  uint64_t* cons_done = reinterpret_cast<uint64_t*>(desc + STAGES);

  grid_dep_trigger();
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_init(qfull, 1);
    mbar_init(cons_done, kConsumerWarps);
    fence_mbar_init();
  }
  __syncthreads();
  // launched as a dependent of the previous kernel on the stream: the
  // prologue above overlapped its tail; nothing it may have written (q,
  // K/V, positions, the workspace and its counters) is touched before it
  // has completed
  grid_dep_wait();
  const int warp = tid >> 5, lane = tid & 31;
  const int pair = (int)(blockIdx.x % (unsigned)p.n_pairs);
  const int member = (int)(blockIdx.x / (unsigned)p.n_pairs);
  Unit un;
  un.item = 0;
  un.gbase = (pair % p.gblocks) * Gm::kGpb;
  un.gcount = min(Gm::kGpb, p.G - un.gbase);
  un.h_kv = (pair / p.gblocks) % p.H_kv;
  un.b = pair / p.gblocks / p.H_kv;

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      mbar_arrive_expect_tx(qfull, Gm::kNBox * Gm::kGpb * Gm::kInner);
#pragma unroll
      for (int bx = 0; bx < Gm::kNBox; ++bx)
        tma_load_3d(qslot + bx * Gm::kGpb * Gm::kInner, &p.qmap, bx * Gm::kBoxElems,
                    un.h_kv * p.G + un.gbase, un.b, qfull);
      // Takes are ranges of the pair's tiles (numbered across its
      // segments): member m's first take is tiles [2m, 2m + 2); later
      // takes come from the pair's counter (offset by the 2 * cpg
      // pre-assigned tiles), two tiles at a time, then one at a time over
      // the last ~4 tiles per CTA so the group finishes closer together.
      // The next take is in flight while the current one loads.
      unsigned int* ctr = p.ctrl + pair;
      const unsigned int cpg = gridDim.x / (unsigned)p.n_pairs;
      const unsigned int n_tiles = (unsigned)p.n_dyn_tiles;
      const unsigned int single = n_tiles > 4u * cpg ? n_tiles - 4u * cpg : 0u;
      int gt = 0;
      bool ok = true;
      unsigned int cur = 2u * member, len = kPieceTiles;
      unsigned int nxt = 0, nlen = 0;
      auto take = [&]() {
        nlen = (cur + len >= single) ? 1u : (unsigned)kPieceTiles;
        nxt = 2u * cpg + atomicAdd(ctr, nlen);
      };
      if (cur < n_tiles) take();
      while (ok && cur < n_tiles) {
        const unsigned int end = min(cur + len, n_tiles);
        for (unsigned int tt = cur; tt < end && ok; ++tt, ++gt) {
          int si = 0;                  // items[i].slot = first tile of segment i
          while (si + 1 < p.n_items && p.items[si + 1].slot <= (int)tt) ++si;
          const Item& it = p.items[si];
          const int t = (int)tt - it.slot;
          const CUtensorMap* kmap = &p.maps[2 * si];
          const CUtensorMap* vmap = &p.maps[2 * si + 1];
          const int bc = it.b_bcast ? 0 : un.b;
          const int s = gt % STAGES;
          if (gt >= STAGES && !(ok = mbar_wait(&empty[s], ((gt / STAGES) & 1) ^ 1, p.err))) break;
          const int r0 = t * kBlockN;
          desc[s].pos0 = it.start + r0;
          desc[s].valid = min(kBlockN, it.rows - r0);
          desc[s].causal = it.causal;
          char* kd = ring + s * Gm::kStageBytes;
          char* vd = kd + Gm::kTileBytes;
          mbar_arrive_expect_tx(&full[s], 2u * Gm::kTileBytes);
#pragma unroll
          for (int bx = 0; bx < Gm::kNBox; ++bx) {
            tma_load_4d(kd + bx * Gm::kBoxBytes, kmap, bx * Gm::kBoxElems, it.row0 + r0, un.h_kv,
                        bc, &full[s]);
            tma_load_4d(vd + bx * Gm::kBoxBytes, vmap, bx * Gm::kBoxElems, it.row0 + r0, un.h_kv,
                        bc, &full[s]);
          }
        }
        cur = nxt;
        len = nlen;
        if (ok && cur < n_tiles) take();
      }
      if (ok) {   // end of work: a stage descriptor with no rows
        const int s = gt % STAGES;
        if (gt < STAGES || (ok = mbar_wait(&empty[s], ((gt / STAGES) & 1) ^ 1, p.err))) {
          desc[s].valid = 0;
          mbar_arrive(&full[s]);
        }
      }
      // the consumers are done with every stage (bounded), then count out
      mbar_wait(cons_done, 0, p.err);
      __threadfence();
      if (atomicAdd(p.ctrl + p.n_pairs, 1u) == gridDim.x - 1) {
        for (int i = 0; i < p.n_pairs; ++i) p.ctrl[i] = 0;
        p.ctrl[p.n_pairs] = 0;
      }
    }
    return;
  }

  // ---------------- consumer warps
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  if (mbar_wait(qfull, 0, p.err)) {
    uint32_t qf[D / 16][4];
    load_q_frags<T, D, STAGES>(qslot, qf);
    const int64_t qpos = (p.q_pos != nullptr) ? p.q_pos[un.b] : INT64_MAX;
    for (int gt = 0;; ++gt) {
      const int s = gt % STAGES;
      if (!mbar_wait(&full[s], (gt / STAGES) & 1, p.err)) break;
      const TileDesc d = desc[s];
      if (d.valid == 0) break;
      const uint32_t kbase = smem_addr(ring + s * Gm::kStageBytes);
      mma_tile<T, D, STAGES>(p.scale_log2, kbase, kbase + Gm::kTileBytes, qf, o, m0, m1, l0, l1,
                             d.valid, d.pos0, d.causal != 0, qpos);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  // ---- combine the four warps' states into the CTA's partial (slot
  // `member`): every warp is past its last tile, so the ring is free scratch
  named_bar_sync(1, kConsumerWarps * 32);
  constexpr int kStride = D + 8;
  static_assert(kConsumerWarps * 16 * (kStride + 2) * 4 <= STAGES * Gm::kStageBytes,
                "combine scratch must fit in the ring");
  float* sc = reinterpret_cast<float*>(ring);
  float* sm = sc + kConsumerWarps * 16 * kStride;
  float* sl = sm + kConsumerWarps * 16;
  {
    const int c = lane & 3, g0 = lane >> 2;
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    float* r0 = sc + (warp * 16 + g0) * kStride;
    float* r1 = r0 + 8 * kStride;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<float2*>(r0 + i * 8 + 2 * c) = make_float2(o[i][0], o[i][1]);
      *reinterpret_cast<float2*>(r1 + i * 8 + 2 * c) = make_float2(o[i][2], o[i][3]);
    }
    if (c == 0) {
      sm[warp * 16 + g0] = m0;
      sm[warp * 16 + g0 + 8] = m1;
      sl[warp * 16 + g0] = l0;
      sl[warp * 16 + g0 + 8] = l1;
    }
  }
  named_bar_sync(1, kConsumerWarps * 32);
  {
    constexpr int kCols = D / 8;          // columns per thread: 8 threads per row
    const int r = tid >> 3, c0 = (tid & 7) * kCols;
    if (r < un.gcount) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm[w * 16 + r]);
      float wt[kConsumerWarps], L = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float mw = sm[w * 16 + r];
        wt[w] = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
        L = fmaf(sl[w * 16 + r], wt[w], L);
      }
      const int h = un.h_kv * p.G + un.gbase + r;
      const int64_t prow = ((int64_t)un.b * p.H + h) * p.S + member;
      float* op = p.o_part + prow * D + c0;
#pragma unroll
      for (int j = 0; j < kCols; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) acc = fmaf(sc[(w * 16 + r) * kStride + c0 + j], wt[w], acc);
        op[j] = acc;
      }
      if ((tid & 7) == 0) {
        p.m_part[prow] = (M == -INFINITY) ? -INFINITY : M * kLn2;
        p.l_part[prow] = L;
      }
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(cons_done);
}

// ---------------------------------------------------------------- KIVI decode
// Fused dequantise-and-attend over a KIVI-packed prefix.  Same persistent
// producer / consumer structure and the same tensor-core attention math as
// kd_kernel; the tiles are different: the producer streams each 64-row tile's
// packed codes, scales and zero points (cp.async.bulk, ~0.375 B/element at
// 2 bits) and each consumer warp dequantises its own 16 rows into a swizzled
// 16-bit tile in shared memory, bit-identical to the reference's
// `q.float() * scale.float() + zero.float()` rounded to the cache dtype
// (baselines/kivi_cache.py:72-78 in lzbaclz/HALO), before attending.
struct KiviView {
  const uint8_t* codes;
  const char* scale;
  const char* zero;
  int64_t c_sb, c_sh;  // bytes
  int64_t s_sb, s_sh;  // bytes
};

struct alignas(64) KiviParams {
  CUtensorMap qmap;
  Item items[kMaxItems];
  KiviView kv[2];
  const int64_t* q_pos;
  float* m_part;
  float* l_part;
  float* o_part;
  unsigned int* err;
  int32_t B, H, H_kv, G, gblocks;
  int32_t S;
  int32_t n_items, n_units;
  float scale_log2;
};

// Packed-tile geometry of kk_kernel.  TR is the transposed tile math; it
// runs 3 CTAs per SM at 128 registers, no spill (measured faster than 4
// CTAs at 96 registers with spills by 11 % at 2 bits, 7 % at 4 bits and
// 3 % at 8 bits, and than 2 CTAs by 7 % at 2 bits).  With 2-bit codes it
// dequantises K straight into MMA registers (kKDirect) and keeps only the
// V tile in shared memory, which leaves room for a 4-stage packed ring;
// with 4/8-bit codes both tiles are staged and the ring has 2 stages.  The
// row-layout variant runs 2 CTAs per SM with 4 stages.
template <typename T, int D, int BITS, bool TR = false>
struct KGeom {
  using Gm = Geom<T, D, 1>;
  static constexpr int kCB = D * BITS / 8;        // code bytes per row
  static constexpr int kGS = D / 32;              // groups per row
  static constexpr int kCodeTile = 64 * kCB;
  static constexpr int kSZTile = 64 * kGS * 2;
  static constexpr int kPackBytes = kCodeTile + 2 * kSZTile;
  static constexpr bool kKDirect = TR && BITS == 2;
  static constexpr int kStages = (TR && !kKDirect) ? 2 : 4;
  static constexpr int kMinCtas = TR ? 3 : 2;   // per SM
  static constexpr int kStageBytes = 2 * kPackBytes;
  static constexpr int kDqBytes = (kKDirect ? 1 : 2) * Gm::kTileBytes;
  static constexpr int kSmemBytes =
      kDqBytes + 2 * Gm::kQSlotBytes + kStages * kStageBytes + 128 + 1024;
  static_assert(kPackBytes % 16 == 0, "bulk copies need 16-byte multiples");
  static_assert((2 * kStages + 4) * 8 <= 128, "full/empty/qfull/qempty barriers fit their 128 bytes");
};

// Warp w dequantises rows [16w, 16w+16) of one packed K or V tile into the
// swizzled 64-row 16-bit tile `dq`.  Lane: row 16w + lane/2, half of the
// row's columns by lane parity; one group (32 columns) at a time.  All
// accesses are explicit shared-memory loads and stores, free of bank
// conflicts: with two groups per half-row the odd half stores its groups in
// reverse order, so the 8 lanes of each 128-byte store phase (4 rows x 2
// halves) hit 8 different 16-byte bank groups of the swizzled tile, and
// 2-bit codes are read as one 16-byte load per lane (a quarter-warp reads
// 128 contiguous bytes).
template <typename T, int D, int BITS>
__device__ __forceinline__ void dequant_rows(const char* pack, char* dq) {
  using KG = KGeom<T, D, BITS>;
  using Gm = typename KG::Gm;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = warp * 16 + (lane >> 1);
  const int half = lane & 1;
  constexpr int kCols = D / 2;
  constexpr int kGroups = kCols / 32;
  static_assert(kGroups == 1 || kGroups == 2, "64 or 128 columns");
  const uint32_t s_codes = smem_addr(pack) + row * KG::kCB;
  const uint32_t s_sc = smem_addr(pack + KG::kCodeTile) + row * KG::kGS * 2;
  const uint32_t s_ze = smem_addr(pack + KG::kCodeTile + KG::kSZTile) + row * KG::kGS * 2;
  const uint32_t s_dq = smem_addr(dq);
  // 2-bit: this half-row's code words (two per group), in store order
  uint32_t words[2 * kGroups];
  if constexpr (BITS == 2) {
    const uint32_t a = s_codes + half * (kCols / 4);
    if constexpr (kGroups == 2) {
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(words[0]), "=r"(words[1]), "=r"(words[2]), "=r"(words[3]) : "r"(a));
      if (half) {
        const uint32_t t0 = words[0], t1 = words[1];
        words[0] = words[2];
        words[1] = words[3];
        words[2] = t0;
        words[3] = t1;
      }
    } else {
      asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(words[0]), "=r"(words[1]) : "r"(a));
    }
  }
#pragma unroll
  for (int j = 0; j < kGroups; ++j) {
    const int jj = kGroups == 2 ? (j ^ half) : j;
    const int col0 = half * kCols + jj * 32;
    const int g = col0 / 32;
    uint16_t sb, zb;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sb) : "r"(s_sc + 2 * g));
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(zb) : "r"(s_ze + 2 * g));
    uint32_t out[16];
    if constexpr (BITS == 2) {
      // pair p of word w is columns 16w + 2p, 16w + 2p + 1 of the group
      const uint32_t s2 = (uint32_t)sb | ((uint32_t)sb << 16);
      const uint32_t z2 = (uint32_t)zb | ((uint32_t)zb << 16);
#pragma unroll
      for (int w = 0; w < 2; ++w)
#pragma unroll
        for (int q = 0; q < 8; ++q) out[w * 8 + q] = code2_pair<T>(words[2 * j + w], q, s2, z2);
    } else {
      const float s = Elem<T>::to_f32(*reinterpret_cast<const T*>(&sb));
      const float z = Elem<T>::to_f32(*reinterpret_cast<const T*>(&zb));
      constexpr uint32_t kMask = (1u << BITS) - 1u;
      constexpr int kPer = 8 / BITS;
      uint32_t cw[32 * BITS / 32];
#pragma unroll
      for (int i = 0; i < BITS; ++i)
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(cw[i]) : "r"(s_codes + col0 * BITS / 8 + 4 * i));
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const int i0 = e, i1 = e + 1;
        const uint32_t c0 = (cw[(i0 / kPer) / 4] >> (8 * ((i0 / kPer) % 4) + (i0 % kPer) * BITS)) & kMask;
        const uint32_t c1 = (cw[(i1 / kPer) / 4] >> (8 * ((i1 / kPer) % 4) + (i1 % kPer) * BITS)) & kMask;
        out[e / 2] = Elem<T>::pack(__fadd_rn(__fmul_rn((float)c0, s), z),
                                   __fadd_rn(__fmul_rn((float)c1, s), z));
      }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};"
                   ::"r"(s_dq + swz<Gm::kInner>(row, col0 / 8 + c)), "r"(out[4 * c]),
                     "r"(out[4 * c + 1]), "r"(out[4 * c + 2]), "r"(out[4 * c + 3])
                   : "memory");
  }
}

// Tile provider: wait for a packed stage, dequantise this warp's rows of K
// and V into the 16-bit tiles, free the packed stage at once.
template <typename T, int D, int BITS, bool TR>
struct DequantTiles {
  using KG = KGeom<T, D, BITS, TR>;
  static constexpr bool kKDirect = false;
  char* stages;
  char* kdq;
  char* vdq;
  uint64_t* full;
  uint64_t* empty;
  unsigned int* err;
  __device__ __forceinline__ bool acquire(int t, int gt, uint32_t& kbase, uint32_t& vbase) {
    const int s = gt % KG::kStages;
    if (!mbar_wait(&full[s], (gt / KG::kStages) & 1, err)) return false;
    const char* st = stages + s * KG::kStageBytes;
    dequant_rows<T, D, BITS>(st, kdq);
    dequant_rows<T, D, BITS>(st + KG::kPackBytes, vdq);
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[s]);
    kbase = smem_addr(kdq);
    vbase = smem_addr(vdq);
    return true;
  }
  __device__ __forceinline__ void release(int) { __syncwarp(); }
};

// K-direct tile provider (2-bit, transposed): K's codes, scales and zeros go
// to registers (KRegs), V is dequantised into the 16-bit tile; the packed
// stage is freed once both are done.
template <typename T, int D>
struct DequantTilesKD {
  using KG = KGeom<T, D, 2, true>;
  static constexpr bool kKDirect = true;
  char* stages;
  char* vdq;
  uint64_t* full;
  uint64_t* empty;
  unsigned int* err;
  KRegs<D> kr;
  __device__ __forceinline__ bool acquire(int t, int gt, uint32_t& kbase, uint32_t& vbase) {
    const int s = gt % KG::kStages;
    if (!mbar_wait_hint(&full[s], (gt / KG::kStages) & 1, err, kKiviWaitHintNs)) return false;
    const char* st = stages + s * KG::kStageBytes;
    load_k_regs<T, D>(st, KG::kCodeTile, KG::kSZTile, kr);
    dequant_rows<T, D, 2>(st + KG::kPackBytes, vdq);
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[s]);
    kbase = 0;
    vbase = smem_addr(vdq);
    return true;
  }
  __device__ __forceinline__ void release(int) { __syncwarp(); }
};

// TR: transposed tile math (GQA groups of at most 8 q-heads); CTAs per SM
// as KGeom states.
template <typename T, int D, int BITS, bool TR>
__global__ void __launch_bounds__(kThreads, KGeom<T, D, BITS, TR>::kMinCtas)
    kk_kernel(const __grid_constant__ KiviParams p) {
  using KG = KGeom<T, D, BITS, TR>;
  using Gm = typename KG::Gm;
  constexpr int STAGES = KG::kStages;
  extern __shared__ char smem_raw[];
  // 16-bit tiles (K then V; V only with K-direct) | q ring | packed ring
  char* kdq = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                      ~uintptr_t(1023));
  char* vdq = KG::kKDirect ? kdq : kdq + Gm::kTileBytes;
  char* qring = kdq + KG::kDqBytes;
  char* stages = qring + 2 * Gm::kQSlotBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + STAGES * KG::kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* qfull = empty + STAGES;
  uint64_t* qempty = qfull + 2;

  // the merge launched after this kernel may be scheduled from now on; it
  // waits for this grid to finish before reading the partials
  grid_dep_trigger();
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qempty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // launched as a dependent of the previous kernel on the stream: the
  // prologue above overlapped its tail; nothing it may have written (q,
  // K/V, positions, the workspace) is touched before it has completed
  grid_dep_wait();
  const int warp = tid >> 5, lane = tid & 31;

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      int gt = 0, ut = 0;
      for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++ut) {
        const Unit un = decode_unit(p, u, Gm::kGpb);
        const Item& it = p.items[un.item];
        const int qs = ut & 1;
        if (ut >= 2 && !mbar_wait(&qempty[qs], ((ut >> 1) & 1) ^ 1, p.err)) return;
        mbar_arrive_expect_tx(&qfull[qs], Gm::kNBox * Gm::kGpb * Gm::kInner);
#pragma unroll
        for (int bx = 0; bx < Gm::kNBox; ++bx)
          tma_load_3d(qring + qs * Gm::kQSlotBytes + bx * Gm::kGpb * Gm::kInner, &p.qmap,
                      bx * Gm::kBoxElems, un.h_kv * p.G + un.gbase, un.b, &qfull[qs]);
        const int n_tiles = (it.rows + kBlockN - 1) / kBlockN;
        for (int t = 0; t < n_tiles; ++t, ++gt) {
          const int s = gt % STAGES;
          if (gt >= STAGES && !mbar_wait_hint(&empty[s], ((gt / STAGES) & 1) ^ 1, p.err, kKiviWaitHintNs)) return;
          const int64_t r0 = it.row0 + t * kBlockN;
          char* dst = stages + s * KG::kStageBytes;
          mbar_arrive_expect_tx(&full[s], KG::kStageBytes);
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const KiviView& kv = p.kv[w];
            char* d = dst + w * KG::kPackBytes;
            bulk_g2s(d, kv.codes + un.b * kv.c_sb + un.h_kv * kv.c_sh + r0 * KG::kCB,
                     KG::kCodeTile, &full[s]);
            bulk_g2s(d + KG::kCodeTile, kv.scale + un.b * kv.s_sb + un.h_kv * kv.s_sh + r0 * KG::kGS * 2,
                     KG::kSZTile, &full[s]);
            bulk_g2s(d + KG::kCodeTile + KG::kSZTile,
                     kv.zero + un.b * kv.s_sb + un.h_kv * kv.s_sh + r0 * KG::kGS * 2,
                     KG::kSZTile, &full[s]);
          }
        }
      }
    }
    return;
  }

  int gt = 0, ut = 0;
  for (int u = blockIdx.x; u < p.n_units; u += gridDim.x, ++ut) {
    const Unit un = decode_unit(p, u, Gm::kGpb);
    const Item& it = p.items[un.item];
    const int qs = ut & 1;
    if (!mbar_wait(&qfull[qs], (ut >> 1) & 1, p.err)) return;
    const int64_t qpos = (it.causal && p.q_pos != nullptr) ? p.q_pos[un.b] : INT64_MAX;
    const int n_tiles = (it.rows + kBlockN - 1) / kBlockN;
    bool ok;
    if constexpr (KG::kKDirect) {
      DequantTilesKD<T, D> tiles{stages, vdq, full, empty, p.err, {}};
      ok = consume_mma_t<T, D, STAGES>(p, un, it, tiles, qring + qs * Gm::kQSlotBytes, &qempty[qs],
                                       n_tiles, gt, qpos);
    } else if constexpr (TR) {
      DequantTiles<T, D, BITS, TR> tiles{stages, kdq, vdq, full, empty, p.err};
      ok = consume_mma_t<T, D, STAGES>(p, un, it, tiles, qring + qs * Gm::kQSlotBytes, &qempty[qs],
                                       n_tiles, gt, qpos);
    } else {
      DequantTiles<T, D, BITS, TR> tiles{stages, kdq, vdq, full, empty, p.err};
      ok = consume_mma<T, D, STAGES>(p, un, it, tiles, qring + qs * Gm::kQSlotBytes, &qempty[qs],
                                     n_tiles, gt, qpos);
    }
    if (!ok) return;
  }
}

// ---------------------------------------------------------------- km kernel
struct MergeParams {
  const float* m_parts;
  const float* l_parts;   // NULL: every part has l = 1
  const float* o_parts;
  int64_t ps, rs;         // m/l: part stride, row stride (elements)
  int64_t ops, ors;       // o: part stride, row stride (elements)
  int32_t R, H, P, Dv;
  int32_t mode, out_dtype;
  char* out;
  int64_t out_sb, out_sh;  // element strides
  float* lse;
  float* m;
  float* l;
  float* o;
};

// One CTA of kMergeWarps warps per (b, h) row: merge_partials folds the
// row's partials (warp w takes s = w, w + kMergeWarps, ...; up to 40 of them,
// 16 for rows wider than 128, in one memory round trip) with a running max,
// and the warps' states are combined through shared memory; the prior state
// is folded in last.  Four warps and at most 88 registers a thread, so a CTA
// fits beside two split-KV CTAs on an SM: launched as a dependent, the
// merge's CTAs are resident (waiting) while the split-KV kernel drains.
constexpr int kMergeWarps = 4;

template <int DPL, bool VEC>
__global__ void __maxnreg__(88) km_kernel(const MergeParams mp) {
  __shared__ float s_m[kMergeWarps];
  __shared__ float s_l[kMergeWarps];
  __shared__ __align__(16) float s_o[kMergeWarps][DPL * 32];
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x;
  grid_dep_trigger();   // the next split-KV launch may start its prologue
  grid_dep_wait();      // the partials' writer has finished (dependent launch)
  const float* mr = mp.m_parts + (int64_t)row * mp.rs;
  const float* lr = mp.l_parts ? mp.l_parts + (int64_t)row * mp.rs : nullptr;
  const float* orow = mp.o_parts + (int64_t)row * mp.ors;
  const int d0 = lane * DPL;
  const bool active = d0 < mp.Dv;
  float M, L;
  float acc[DPL];
  merge_partials<DPL, kMergeWarps, kMergeRound<DPL>, VEC>(mr, lr, orow, mp.ps, mp.ops, mp.P,
                                                          mp.Dv, s_m, s_l, s_o, M, L, acc);
  if (threadIdx.x >= 32) return;

  // ---- warp 0: fold the prior state in and write
  if (mp.m != nullptr) {
    const float mw = mp.m[row];
    const float Mn = fmaxf(M, mw);
    if (Mn != -INFINITY) {
      const float a = (M == -INFINITY) ? 0.f : expf(M - Mn);
      const float w = (mw == -INFINITY) ? 0.f : expf(mw - Mn);
      L = fmaf(mp.l[row], w, L * a);
#pragma unroll
      for (int e = 0; e < DPL; ++e)
        acc[e] = active ? fmaf(mp.o[(int64_t)row * mp.Dv + d0 + e], w, acc[e] * a) : 0.f;
      M = Mn;
    }
  }

  if (mp.mode == HALO_MERGE_ACCUMULATE) {
    if (lane == 0) {
      mp.m[row] = M;
      mp.l[row] = L;
    }
    if (active)
#pragma unroll
      for (int e = 0; e < DPL; ++e) mp.o[(int64_t)row * mp.Dv + d0 + e] = acc[e];
    return;
  }
  const int b = row / mp.H, h = row % mp.H;
  if (lane == 0 && mp.lse != nullptr) mp.lse[row] = (L > 0.f) ? M + logf(L) : -INFINITY;
  if (!active) return;
  const float inv = (L > 0.f) ? 1.f / L : 0.f;
  const int64_t off = (int64_t)b * mp.out_sb + (int64_t)h * mp.out_sh + d0;
#pragma unroll
  for (int e = 0; e < DPL; ++e) {
    const float v = (L > 0.f) ? acc[e] * inv : 0.f;
    if (mp.out_dtype == HALO_DTYPE_F32)
      reinterpret_cast<float*>(mp.out)[off + e] = v;
    else if (mp.out_dtype == HALO_DTYPE_BF16)
      reinterpret_cast<__nv_bfloat16*>(mp.out)[off + e] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<__half*>(mp.out)[off + e] = __float2half_rn(v);
  }
}

// ================================================================ host side
thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(HALO_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int device_sms() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

static int elt_size(int dtype) {
  return dtype == HALO_DTYPE_F32 ? 4 : (dtype == HALO_DTYPE_BF16 || dtype == HALO_DTYPE_F16) ? 2 : 0;
}

// ---------------------------------------------------------------- tensor maps
// TMA inner box width (bytes) for rows of D elements: the largest of
// 128/64/32 dividing the row, with the swizzle mode of the same width.
static int inner_bytes(int D, int elt) {
  const int rb = D * elt;
  return rb % 128 == 0 ? 128 : (rb % 64 == 0 ? 64 : 32);
}
static CUtensorMapSwizzle swizzle_for(int inner) {
  return inner == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                      : (inner == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

struct MapKey {
  uintptr_t ptr;
  int64_t dims[4];
  int64_t strides[3];
  int dtype;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && dtype == o.dtype && std::memcmp(dims, o.dims, sizeof(dims)) == 0 &&
           std::memcmp(strides, o.strides, sizeof(strides)) == 0;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = 1469598103934665603ull ^ k.ptr;
    auto mix = [&](uint64_t v) { h = (h ^ v) * 1099511628211ull; };
    for (int i = 0; i < 4; ++i) mix(static_cast<uint64_t>(k.dims[i]));
    for (int i = 0; i < 3; ++i) mix(static_cast<uint64_t>(k.strides[i]));
    mix(static_cast<uint64_t>(k.dtype));
    return static_cast<size_t>(h);
  }
};

// Encode (or fetch from a small host cache) the 4-D tiled tensor map of one
// K or V view: dims {D, rows, H_kv, B}, 128-byte inner box x 64 rows, 128B
// swizzle, out-of-bounds rows zero-filled.
static int encode_view(const void* base, int64_t rows, int H_kv, int B, int D, int dtype,
                       int64_t sb_el, int64_t sh_el, int64_t st_el, CUtensorMap* out) {
  const int elt = elt_size(dtype);
  MapKey key;
  key.ptr = reinterpret_cast<uintptr_t>(base);
  const bool bcast = sb_el == 0;
  key.dims[0] = D;
  key.dims[1] = rows;
  key.dims[2] = H_kv;
  key.dims[3] = bcast ? 1 : B;
  key.strides[0] = st_el * elt;
  key.strides[1] = sh_el * elt;
  key.strides[2] = bcast ? sh_el * elt * H_kv : sb_el * elt;
  key.dtype = dtype;
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto itc = cache.find(key);
    if (itc != cache.end()) {
      *out = itc->second;
      return HALO_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(HALO_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (key.strides[2] == 0) key.strides[2] = key.strides[1] > 0 ? key.strides[1] : 16;
  cuuint64_t gdim[4] = {(cuuint64_t)key.dims[0], (cuuint64_t)key.dims[1], (cuuint64_t)key.dims[2],
                        (cuuint64_t)key.dims[3]};
  cuuint64_t gstr[3] = {(cuuint64_t)key.strides[0], (cuuint64_t)key.strides[1],
                        (cuuint64_t)key.strides[2]};
  const int inner = inner_bytes(D, elt);
  cuuint32_t box[4] = {(cuuint32_t)(inner / elt), (cuuint32_t)kBlockN, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == HALO_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == HALO_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(out, dt, 4, const_cast<void*>(base), gdim, gstr, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(inner),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(HALO_ERR_INVALID_ARG,
                "cuTensorMapEncodeTiled failed (%d): dims {%lld,%lld,%lld,%lld} strides "
                "{%lld,%lld,%lld} bytes",
                (int)r, (long long)key.dims[0], (long long)key.dims[1], (long long)key.dims[2],
                (long long)key.dims[3], (long long)key.strides[0], (long long)key.strides[1],
                (long long)key.strides[2]);
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, *out);
  return HALO_OK;
}


static int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// Head dims with a compiled kernel (rows must be whole 32-byte TMA boxes).
static bool supported_head_dim(int dtype, int D) {
  if (dtype == HALO_DTYPE_F32) return D == 16 || D == 32 || D == 64 || D == 80 || D == 96 || D == 128;
  return D == 16 || D == 32 || D == 64 || D == 80 || D == 96 || D == 128;
}

static int validate_problem(const halo_decode_problem_t* p, const halo_kv_chunk_t* chunks,
                            int n_chunks) {
  if (!p) return fail(HALO_ERR_INVALID_ARG, "problem is NULL");
  if (p->B <= 0 || p->H <= 0 || p->H_kv <= 0 || p->D <= 0 || p->Dv <= 0)
    return fail(HALO_ERR_INVALID_ARG, "non-positive dimension (B=%d H=%d H_kv=%d D=%d Dv=%d)",
                p->B, p->H, p->H_kv, p->D, p->Dv);
  if (p->H % p->H_kv != 0)
    return fail(HALO_ERR_INVALID_ARG, "H=%d not divisible by H_kv=%d", p->H, p->H_kv);
  if (elt_size(p->dtype) == 0) return fail(HALO_ERR_INVALID_ARG, "bad dtype %d", p->dtype);
  if (p->Dv != p->D) return fail(HALO_ERR_UNSUPPORTED, "Dv (%d) != D (%d)", p->Dv, p->D);
  const bool d_ok = supported_head_dim(p->dtype, p->D);
  if (!d_ok) return fail(HALO_ERR_UNSUPPORTED, "head_dim %d unsupported for dtype %d", p->D, p->dtype);
  if (n_chunks < 0 || (n_chunks > 0 && !chunks))
    return fail(HALO_ERR_INVALID_ARG, "bad chunk list");
  if (n_chunks > 0 && !p->q) return fail(HALO_ERR_INVALID_ARG, "q is NULL");
  const int elt = elt_size(p->dtype);
  for (int i = 0; i < n_chunks; ++i) {
    const halo_kv_chunk_t& c = chunks[i];
    if (c.len < 0) return fail(HALO_ERR_INVALID_ARG, "chunk %d: negative length", i);
    if (c.len == 0) continue;
    if (!c.k || !c.v) return fail(HALO_ERR_INVALID_ARG, "chunk %d: NULL k/v", i);
    if (c.causal && !p->q_pos) return fail(HALO_ERR_INVALID_ARG, "chunk %d causal but q_pos NULL", i);
    const int64_t s[6] = {c.k_stride_b, c.k_stride_h, c.k_stride_t,
                          c.v_stride_b, c.v_stride_h, c.v_stride_t};
    for (int j = 0; j < 6; ++j)
      if ((s[j] * elt) % 16 != 0)
        return fail(HALO_ERR_MISALIGNED, "chunk %d: stride %lld elements is not 16-byte aligned", i,
                    (long long)s[j]);
    if ((reinterpret_cast<uintptr_t>(c.k) | reinterpret_cast<uintptr_t>(c.v)) & 15)
      return fail(HALO_ERR_MISALIGNED, "chunk %d: k/v pointer not 16-byte aligned", i);
  }
  return HALO_OK;
}

int launch_merge(const MergeParams& mp, cudaStream_t st) {
  if (mp.R == 0) return HALO_OK;
  const int threads = kMergeWarps * 32;
  const bool vec = (reinterpret_cast<uintptr_t>(mp.o_parts) & 15) == 0 && mp.ops % 4 == 0 &&
                   mp.ors % 4 == 0;
  // launched as a dependent of the kernel that wrote the partials, so its
  // launch overlaps that kernel's last CTAs (km_kernel waits for it first)
  cudaError_t e;
  if (mp.Dv <= 32) e = launch_dependent(km_kernel<1, false>, mp.R, threads, 0, st, mp);
  else if (mp.Dv <= 64 && mp.Dv % 2 == 0)
    e = launch_dependent(km_kernel<2, false>, mp.R, threads, 0, st, mp);
  else if (mp.Dv <= 128 && mp.Dv % 4 == 0 && vec)
    e = launch_dependent(km_kernel<4, true>, mp.R, threads, 0, st, mp);
  else if (mp.Dv <= 128 && mp.Dv % 4 == 0)
    e = launch_dependent(km_kernel<4, false>, mp.R, threads, 0, st, mp);
  else if (mp.Dv <= 256 && mp.Dv % 8 == 0)
    e = launch_dependent(km_kernel<8, false>, mp.R, threads, 0, st, mp);
  else return fail(HALO_ERR_UNSUPPORTED, "Dv %d unsupported by the merge", mp.Dv);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "km_kernel launch");
  count_launches();
  return HALO_OK;
}

int validate_merge(const halo_merge_args_t* mg, int Dv) {
  if (!mg) return fail(HALO_ERR_INVALID_ARG, "merge args NULL");
  if (mg->mode == HALO_MERGE_ACCUMULATE) {
    if (!mg->m || !mg->l || !mg->o) return fail(HALO_ERR_INVALID_ARG, "accumulate needs m, l, o");
  } else if (mg->mode == HALO_MERGE_FINALIZE) {
    if (!mg->out) return fail(HALO_ERR_INVALID_ARG, "finalize needs out");
    if (elt_size(mg->out_dtype) == 0) return fail(HALO_ERR_INVALID_ARG, "bad out dtype");
    if ((mg->m != nullptr) != (mg->l != nullptr) || (mg->m != nullptr) != (mg->o != nullptr))
      return fail(HALO_ERR_INVALID_ARG, "prior state needs all of m, l, o");
  } else {
    return fail(HALO_ERR_INVALID_ARG, "bad merge mode %d", mg->mode);
  }
  (void)Dv;
  return HALO_OK;
}

MergeParams merge_params(const halo_merge_args_t* mg, int B, int H, int Dv, int P,
                         const float* m_parts, const float* l_parts, const float* o_parts,
                         int64_t ps, int64_t rs, int64_t ops, int64_t ors) {
  MergeParams mp;
  mp.m_parts = m_parts;
  mp.l_parts = l_parts;
  mp.o_parts = o_parts;
  mp.ps = ps;
  mp.rs = rs;
  mp.ops = ops;
  mp.ors = ors;
  mp.R = B * H;
  mp.H = H;
  mp.P = P;
  mp.Dv = Dv;
  mp.mode = mg->mode;
  mp.out_dtype = mg->out_dtype;
  mp.out = static_cast<char*>(mg->out);
  mp.out_sb = mg->out_stride_b;
  mp.out_sh = mg->out_stride_h;
  mp.lse = mg->lse;
  mp.m = mg->m;
  mp.l = mg->l;
  mp.o = mg->o;
  return mp;
}

// ---------------------------------------------------------------- planning
// A segment is a run of chunks that are contiguous in memory AND in global
// position with one causal flag: it gets one K and one V tensor map and is
// split into equal work items.
struct Seg {
  halo_kv_chunk_t view;  // k/v base, strides, start, total len, causal
  int32_t first_chunk;
};

struct Plan {
  std::vector<Seg> segs;
  std::vector<Item> items;  // static: items[i].slot = i * kConsumerWarps
  int32_t split_tiles = 0;
  int32_t S = 0;            // partial slots per (b, h) row
  // dynamic schedule (kd_dyn_kernel): one item per segment whose slot is
  // its first tile (tiles numbered across the segments); `grid` CTAs =
  // n_pairs groups of S CTAs
  bool dyn = false;
  int32_t n_pairs = 0, n_tiles = 0, grid = 0;
};

static int dyn_ctas_per_sm(int dtype, int D);

static int gpb_for(int dtype) { return dtype == HALO_DTYPE_F32 ? 8 : 16; }

static int ctas_per_sm(int dtype, int D);

static bool continues(const halo_kv_chunk_t& a, const halo_kv_chunk_t& c, int elt) {
  return c.causal == a.causal && c.start == a.start + a.len &&
         c.k_stride_b == a.k_stride_b && c.k_stride_h == a.k_stride_h &&
         c.k_stride_t == a.k_stride_t && c.v_stride_b == a.v_stride_b &&
         c.v_stride_h == a.v_stride_h && c.v_stride_t == a.v_stride_t &&
         static_cast<const char*>(c.k) ==
             static_cast<const char*>(a.k) + (int64_t)a.len * a.k_stride_t * elt &&
         static_cast<const char*>(c.v) ==
             static_cast<const char*>(a.v) + (int64_t)a.len * a.v_stride_t * elt;
}

static Plan make_plan(const halo_decode_problem_t* p, const halo_kv_chunk_t* chunks, int n) {
  Plan plan;
  const int elt = elt_size(p->dtype);
  for (int i = 0; i < n; ++i) {
    const halo_kv_chunk_t& c = chunks[i];
    if (c.len <= 0) continue;
    if (!plan.segs.empty() && continues(plan.segs.back().view, c, elt)) {
      plan.segs.back().view.len += c.len;
    } else {
      Seg sg;
      sg.view = c;
      sg.first_chunk = i;
      plan.segs.push_back(sg);
    }
  }
  if (plan.segs.empty()) return plan;

  const int G = p->H / p->H_kv;
  const int gpb = gpb_for(p->dtype);
  const int64_t pairs = (int64_t)p->B * p->H_kv * ((G + gpb - 1) / gpb);
  const int64_t grid = (int64_t)device_sms() * ctas_per_sm(p->dtype, p->D);
  std::vector<int64_t> seg_tiles;
  int64_t total_tiles = 0;
  for (const Seg& sg : plan.segs) {
    seg_tiles.push_back(ceil_div64(sg.view.len, kBlockN));
    total_tiles += seg_tiles.back();
  }

  // Dynamic schedule: 16-bit inputs, one launch's worth of segments, and
  // enough pieces for every CTA of a pair's group to take several; the
  // groups must fill at least 90 % of the resident CTA slots.
  if (p->dtype != HALO_DTYPE_F32 && p->max_split_rows <= 0 &&
      (int64_t)plan.segs.size() <= kMaxSegs && pairs <= kMaxDynPairs) {
    const int64_t cap = (int64_t)device_sms() * dyn_ctas_per_sm(p->dtype, p->D);
    const int64_t cpg = cap / pairs;
    int64_t pieces = 0;   // in tiles: the kernel takes them two or one at a time
    for (int64_t t : seg_tiles) pieces += t;
    if (cpg >= 1 && pairs * cpg * 10 >= cap * 9 && pieces >= 8 * cpg) {
      plan.dyn = true;
      plan.n_pairs = (int32_t)pairs;
      plan.n_tiles = (int32_t)pieces;
      plan.grid = (int32_t)(pairs * cpg);
      plan.S = (int32_t)cpg;     // one combined partial per CTA of a group
      int32_t first = 0;
      for (size_t si = 0; si < plan.segs.size(); ++si) {
        const Seg& sg = plan.segs[si];
        Item it;
        it.seg = (int32_t)si;
        it.row0 = 0;
        it.rows = (int32_t)sg.view.len;
        it.start = sg.view.start;
        it.causal = sg.view.causal;
        it.b_bcast = (sg.view.k_stride_b == 0 || sg.view.v_stride_b == 0) ? 1 : 0;
        it.slot = first;
        first += (int32_t)seg_tiles[si];
        plan.items.push_back(it);
      }
      return plan;
    }
  }
  int64_t split = 0;
  // Memoise the choice per layout signature: decode steps repeat layouts.
  uint64_t sig = 1469598103934665603ull;
  auto mix = [&](uint64_t v) { sig = (sig ^ v) * 1099511628211ull; };
  mix((uint64_t)pairs); mix((uint64_t)grid); mix((uint64_t)p->D); mix((uint64_t)elt);
  mix((uint64_t)p->B * p->H);
  for (int64_t t : seg_tiles) mix((uint64_t)t);
  static std::mutex plan_mu;
  static std::unordered_map<uint64_t, int64_t> plan_cache;
  if (p->max_split_rows <= 0) {
    std::lock_guard<std::mutex> lk(plan_mu);
    auto f = plan_cache.find(sig);
    if (f != plan_cache.end()) split = f->second;
  }
  if (split > 0) {
    // cached
  } else if (p->max_split_rows > 0) {
    split = std::max<int64_t>(1, p->max_split_rows / kBlockN);
  } else {
    // Choose the item size (in tiles) minimising the estimated time in
    // tile-equivalents: the persistent grid's makespan
    //   ceil(units / grid) * (tiles per item + per-unit cost)
    // plus the merge traffic of kConsumerWarps partials per item and row,
    // spread over the grid.  Ties go to larger items (fewer partials).
    constexpr double kUnitCostTiles = 1.5;
    const double tile_bytes = 2.0 * kBlockN * p->D * elt;
    const double rows = (double)p->B * p->H;
    double best = 1e300;
    for (int64_t cand = std::max<int64_t>(1, total_tiles); cand >= 1; ) {
      int64_t items = 0, longest = 0;
      for (int64_t t : seg_tiles) {
        items += ceil_div64(t, cand);
        longest = std::max<int64_t>(longest, std::min<int64_t>(t, cand));
      }
      const int64_t units = items * pairs;
      const double span = (double)ceil_div64(units, grid) * ((double)longest + kUnitCostTiles);
      const double merge = rows * items * kConsumerWarps * (p->Dv + 2) * 4.0 * 2.0 /
                           (tile_bytes * (double)grid);
      const double cost = span + merge;
      if (items <= 4 * kMaxItems && cost < best * (1.0 - 1e-3)) {
        best = cost;
        split = cand;
      }
      if (cand == 1) break;
      cand = cand > 32 ? cand - std::max<int64_t>(1, cand / 32) : cand - 1;
    }
    if (split == 0) split = std::max<int64_t>(1, ceil_div64(total_tiles, 4 * kMaxItems));
    std::lock_guard<std::mutex> lk(plan_mu);
    if (plan_cache.size() > 4096) plan_cache.clear();
    plan_cache.emplace(sig, split);
  }
  plan.split_tiles = (int32_t)split;
  for (size_t si = 0; si < plan.segs.size(); ++si) {
    const Seg& sg = plan.segs[si];
    const int64_t split_rows = split * kBlockN;
    for (int64_t r = 0; r < sg.view.len; r += split_rows) {
      Item it;
      it.seg = (int32_t)si;
      it.row0 = (int32_t)r;
      it.rows = (int32_t)std::min<int64_t>(split_rows, sg.view.len - r);
      it.start = sg.view.start + r;
      it.causal = sg.view.causal;
      it.b_bcast = (sg.view.k_stride_b == 0 || sg.view.v_stride_b == 0) ? 1 : 0;
      it.slot = (int32_t)plan.items.size() * kConsumerWarps;
      plan.items.push_back(it);
    }
  }
  plan.S = (int32_t)plan.items.size() * kConsumerWarps;
  return plan;
}

static int64_t workspace_for(const halo_decode_problem_t* p, int S) {
  const int64_t R = (int64_t)p->B * p->H;
  return kCtrlBytes + align256(R * S * 4) * 2 + align256(R * S * (int64_t)p->Dv * 4);
}

template <typename T, int D>
struct KdConfig {
  // 3 stages; 2 CTAs per SM unless a stage is larger than 32 KB (fp32 with
  // D > 64), then one.
  static constexpr int kStages = 3;
  static constexpr int kMinBlocks = (2 * 64 * D * (int)sizeof(T)) > 32768 ? 1 : 2;
};

template <typename T, int D>
static int kd_ctas_per_sm() {
  using C = KdConfig<T, D>;
  using Gm = Geom<T, D, C::kStages>;
  static std::once_flag once[64];
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    cudaFuncSetAttribute(kd_kernel<T, D, C::kStages, C::kMinBlocks>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, Gm::kSmemBytes);
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &n, kd_kernel<T, D, C::kStages, C::kMinBlocks>, kThreads, Gm::kSmemBytes) !=
            cudaSuccess || n <= 0)
      n = 1;
    cache[dev & 63] = n;
  });
  return cache[dev & 63];
}

static int ctas_per_sm(int dtype, int D) {
  if (dtype == HALO_DTYPE_BF16) {
    if (D == 16) return kd_ctas_per_sm<__nv_bfloat16, 16>();
    if (D == 32) return kd_ctas_per_sm<__nv_bfloat16, 32>();
    if (D == 64) return kd_ctas_per_sm<__nv_bfloat16, 64>();
    if (D == 80) return kd_ctas_per_sm<__nv_bfloat16, 80>();
    if (D == 96) return kd_ctas_per_sm<__nv_bfloat16, 96>();
    if (D == 128) return kd_ctas_per_sm<__nv_bfloat16, 128>();
  } else if (dtype == HALO_DTYPE_F16) {
    if (D == 16) return kd_ctas_per_sm<__half, 16>();
    if (D == 32) return kd_ctas_per_sm<__half, 32>();
    if (D == 64) return kd_ctas_per_sm<__half, 64>();
    if (D == 80) return kd_ctas_per_sm<__half, 80>();
    if (D == 96) return kd_ctas_per_sm<__half, 96>();
    if (D == 128) return kd_ctas_per_sm<__half, 128>();
  } else {
    if (D == 16) return kd_ctas_per_sm<float, 16>();
    if (D == 32) return kd_ctas_per_sm<float, 32>();
    if (D == 64) return kd_ctas_per_sm<float, 64>();
    if (D == 80) return kd_ctas_per_sm<float, 80>();
    if (D == 96) return kd_ctas_per_sm<float, 96>();
    if (D == 128) return kd_ctas_per_sm<float, 128>();
  }
  return 1;
}

template <typename T, int D>
static int launch_kd(const DecodeParams& prm, cudaStream_t st) {
  using C = KdConfig<T, D>;
  using Gm = Geom<T, D, C::kStages>;
  const int64_t grid_max = (int64_t)device_sms() * kd_ctas_per_sm<T, D>();
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(prm.n_units, grid_max));
  cudaError_t e = launch_dependent(kd_kernel<T, D, C::kStages, C::kMinBlocks>, grid, kThreads,
                                   Gm::kSmemBytes, st, prm);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kd_kernel launch");
  count_launches();
  return HALO_OK;
}

// Shared-memory attribute of one dynamic-schedule instantiation, set once
// per device.
template <typename T, int D, class P>
static void kd_dyn_prepare() {
  using C = KdConfig<T, D>;
  using DG = DynGeom<T, D, C::kStages>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [] {
    cudaFuncSetAttribute(kd_dyn_kernel<T, D, C::kStages, C::kMinBlocks, P>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, DG::kSmemBytes);
  });
}

template <typename T, int D>
static int kd_dyn_ctas_per_sm() {
  using C = KdConfig<T, D>;
  using DG = DynGeom<T, D, C::kStages>;
  static std::once_flag once[64];
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    kd_dyn_prepare<T, D, DynParams>();
    kd_dyn_prepare<T, D, DecodeParams>();
    int n = 0, n2 = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &n, kd_dyn_kernel<T, D, C::kStages, C::kMinBlocks, DynParams>, kThreads,
            DG::kSmemBytes) != cudaSuccess || n <= 0)
      n = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &n2, kd_dyn_kernel<T, D, C::kStages, C::kMinBlocks, DecodeParams>, kThreads,
            DG::kSmemBytes) != cudaSuccess || n2 <= 0)
      n2 = 1;
    cache[dev & 63] = std::min(n, n2);
  });
  return cache[dev & 63];
}

template <typename T>
static int dyn_ctas_for(int D) {
  if (D == 16) return kd_dyn_ctas_per_sm<T, 16>();
  if (D == 32) return kd_dyn_ctas_per_sm<T, 32>();
  if (D == 64) return kd_dyn_ctas_per_sm<T, 64>();
  if (D == 80) return kd_dyn_ctas_per_sm<T, 80>();
  if (D == 96) return kd_dyn_ctas_per_sm<T, 96>();
  if (D == 128) return kd_dyn_ctas_per_sm<T, 128>();
  return 1;
}

static int dyn_ctas_per_sm(int dtype, int D) {
  if (dtype == HALO_DTYPE_BF16) return dyn_ctas_for<__nv_bfloat16>(D);
  if (dtype == HALO_DTYPE_F16) return dyn_ctas_for<__half>(D);
  return 1;
}

template <typename T, int D, class P>
static int launch_kd_dyn(const P& prm, int grid, cudaStream_t st) {
  using C = KdConfig<T, D>;
  using DG = DynGeom<T, D, C::kStages>;
  kd_dyn_ctas_per_sm<T, D>();   // sets the shared-memory attributes once
  cudaError_t e = launch_dependent(kd_dyn_kernel<T, D, C::kStages, C::kMinBlocks, P>, grid,
                                   kThreads, DG::kSmemBytes, st, prm);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kd_dyn_kernel launch");
  count_launches();
  return HALO_OK;
}

template <typename T, class P>
static int dispatch_kd_dyn_t(int D, const P& prm, int grid, cudaStream_t st) {
  if (D == 16) return launch_kd_dyn<T, 16>(prm, grid, st);
  if (D == 32) return launch_kd_dyn<T, 32>(prm, grid, st);
  if (D == 64) return launch_kd_dyn<T, 64>(prm, grid, st);
  if (D == 80) return launch_kd_dyn<T, 80>(prm, grid, st);
  if (D == 96) return launch_kd_dyn<T, 96>(prm, grid, st);
  if (D == 128) return launch_kd_dyn<T, 128>(prm, grid, st);
  return fail(HALO_ERR_UNSUPPORTED, "head_dim %d unsupported", D);
}

// Launch the dynamic schedule from a filled DecodeParams: through the
// compact parameter block when the segments fit in it.
static int dispatch_kd_dyn(int dtype, int D, const DecodeParams& prm, int grid, cudaStream_t st) {
  if (dtype != HALO_DTYPE_BF16 && dtype != HALO_DTYPE_F16)
    return fail(HALO_ERR_UNSUPPORTED, "dynamic schedule needs 16-bit inputs");
  if (prm.n_items <= kDynSegs) {
    DynParams dp;
    for (int i = 0; i < 2 * prm.n_items; ++i) dp.maps[i] = prm.maps[i];
    dp.qmap = prm.qmap;
    for (int i = 0; i < prm.n_items; ++i) dp.items[i] = prm.items[i];
    dp.q_pos = prm.q_pos;
    dp.m_part = prm.m_part;
    dp.l_part = prm.l_part;
    dp.o_part = prm.o_part;
    dp.err = prm.err;
    dp.ctrl = prm.ctrl;
    dp.B = prm.B;
    dp.H = prm.H;
    dp.H_kv = prm.H_kv;
    dp.G = prm.G;
    dp.gblocks = prm.gblocks;
    dp.S = prm.S;
    dp.n_items = prm.n_items;
    dp.n_units = prm.n_units;
    dp.n_pairs = prm.n_pairs;
    dp.n_dyn_tiles = prm.n_dyn_tiles;
    dp.scale_log2 = prm.scale_log2;
    if (dtype == HALO_DTYPE_BF16) return dispatch_kd_dyn_t<__nv_bfloat16>(D, dp, grid, st);
    return dispatch_kd_dyn_t<__half>(D, dp, grid, st);
  }
  if (dtype == HALO_DTYPE_BF16) return dispatch_kd_dyn_t<__nv_bfloat16>(D, prm, grid, st);
  return dispatch_kd_dyn_t<__half>(D, prm, grid, st);
}

static int dispatch_kd(int dtype, int D, const DecodeParams& prm, cudaStream_t st) {
  if (dtype == HALO_DTYPE_BF16) {
    if (D == 16) return launch_kd<__nv_bfloat16, 16>(prm, st);
    if (D == 32) return launch_kd<__nv_bfloat16, 32>(prm, st);
    if (D == 64) return launch_kd<__nv_bfloat16, 64>(prm, st);
    if (D == 80) return launch_kd<__nv_bfloat16, 80>(prm, st);
    if (D == 96) return launch_kd<__nv_bfloat16, 96>(prm, st);
    if (D == 128) return launch_kd<__nv_bfloat16, 128>(prm, st);
  } else if (dtype == HALO_DTYPE_F16) {
    if (D == 16) return launch_kd<__half, 16>(prm, st);
    if (D == 32) return launch_kd<__half, 32>(prm, st);
    if (D == 64) return launch_kd<__half, 64>(prm, st);
    if (D == 80) return launch_kd<__half, 80>(prm, st);
    if (D == 96) return launch_kd<__half, 96>(prm, st);
    if (D == 128) return launch_kd<__half, 128>(prm, st);
  } else {
    if (D == 16) return launch_kd<float, 16>(prm, st);
    if (D == 32) return launch_kd<float, 32>(prm, st);
    if (D == 64) return launch_kd<float, 64>(prm, st);
    if (D == 80) return launch_kd<float, 80>(prm, st);
    if (D == 96) return launch_kd<float, 96>(prm, st);
    if (D == 128) return launch_kd<float, 128>(prm, st);
  }
  return fail(HALO_ERR_UNSUPPORTED, "no kernel for dtype %d D %d", dtype, D);
}

static int encode_q_map(const halo_decode_problem_t& pb, CUtensorMap* out) {
  // q as a 3-D tensor {D, H, B}; box {128 bytes, q-heads per unit, 1}
  const int elt = elt_size(pb.dtype);
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(HALO_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(pb.q) & 15) || (pb.q_stride_h * elt) % 16 ||
      (pb.B > 1 && (pb.q_stride_b * elt) % 16))
    return fail(HALO_ERR_MISALIGNED, "q pointer/strides must be 16-byte aligned");
  cuuint64_t gdim[3] = {(cuuint64_t)pb.D, (cuuint64_t)pb.H, (cuuint64_t)pb.B};
  cuuint64_t gstr[2] = {(cuuint64_t)(pb.q_stride_h * elt),
                        (cuuint64_t)(pb.B > 1 ? pb.q_stride_b * elt : pb.q_stride_h * elt * pb.H)};
  const int inner = inner_bytes(pb.D, elt);
  cuuint32_t box[3] = {(cuuint32_t)(inner / elt), (cuuint32_t)gpb_for(pb.dtype), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = pb.dtype == HALO_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : pb.dtype == HALO_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(out, dt, 3, const_cast<void*>(pb.q), gdim, gstr, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_for(inner),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HALO_ERR_INVALID_ARG, "q tensor map encode failed (%d)", (int)r);
  return HALO_OK;
}

// ---------------------------------------------------------------- KIVI host side
template <typename T, int D, int BITS, bool TR>
static int kk_ctas_per_sm() {
  using KG = KGeom<T, D, BITS, TR>;
  static std::once_flag once[64];
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    cudaFuncSetAttribute(kk_kernel<T, D, BITS, TR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         KG::kSmemBytes);
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kk_kernel<T, D, BITS, TR>, kThreads,
                                                      KG::kSmemBytes) != cudaSuccess || n <= 0)
      n = 1;
    cache[dev & 63] = n;
  });
  return cache[dev & 63];
}

// The transposed tile math serves GQA groups of at most 8 q-heads.
static bool kk_transposed(int G) { return G <= 8; }

template <typename T, int D, int BITS>
static int kk_occupancy(int G) {
  return kk_transposed(G) ? kk_ctas_per_sm<T, D, BITS, true>() : kk_ctas_per_sm<T, D, BITS, false>();
}

static int kk_occupancy_for(int dtype, int D, int bits, int G) {
  const bool bf = dtype == HALO_DTYPE_BF16;
#define HALO_KK_OCC(DD, BB)                                                            \
  if (D == DD && bits == BB)                                                           \
    return bf ? kk_occupancy<__nv_bfloat16, DD, BB>(G) : kk_occupancy<__half, DD, BB>(G);
  HALO_KK_OCC(128, 2) HALO_KK_OCC(128, 4) HALO_KK_OCC(128, 8)
  HALO_KK_OCC(64, 2) HALO_KK_OCC(64, 4) HALO_KK_OCC(64, 8)
#undef HALO_KK_OCC
  return 2;
}

template <typename T, int D, int BITS, bool TR>
static int launch_kk(const KiviParams& prm, cudaStream_t st) {
  using KG = KGeom<T, D, BITS, TR>;
  const int64_t grid_max = (int64_t)device_sms() * kk_ctas_per_sm<T, D, BITS, TR>();
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(prm.n_units, grid_max));
  cudaError_t e =
      launch_dependent(kk_kernel<T, D, BITS, TR>, grid, kThreads, KG::kSmemBytes, st, prm);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "kk_kernel launch");
  count_launches();
  return HALO_OK;
}

template <typename T, int D, int BITS>
static int launch_kk_g(const KiviParams& prm, cudaStream_t st) {
  return kk_transposed(prm.G) ? launch_kk<T, D, BITS, true>(prm, st)
                              : launch_kk<T, D, BITS, false>(prm, st);
}

template <typename T>
static int dispatch_kk_t(int D, int bits, const KiviParams& prm, cudaStream_t st) {
  if (D == 128) {
    if (bits == 2) return launch_kk_g<T, 128, 2>(prm, st);
    if (bits == 4) return launch_kk_g<T, 128, 4>(prm, st);
    if (bits == 8) return launch_kk_g<T, 128, 8>(prm, st);
  } else if (D == 64) {
    if (bits == 2) return launch_kk_g<T, 64, 2>(prm, st);
    if (bits == 4) return launch_kk_g<T, 64, 4>(prm, st);
    if (bits == 8) return launch_kk_g<T, 64, 8>(prm, st);
  }
  return fail(HALO_ERR_UNSUPPORTED, "KIVI decode: D %d bits %d", D, bits);
}

// Rows per work item for the KIVI decode: the same cost model as the plain
// decode planner (persistent makespan + merge traffic), one segment.
static int64_t kivi_split_tiles(const halo_decode_problem_t* p, int64_t rows, int bits) {
  const int G = p->H / p->H_kv;
  const int64_t pairs = (int64_t)p->B * p->H_kv * ((G + 15) / 16);
  const int64_t grid =
      (int64_t)device_sms() * kk_occupancy_for(p->dtype, p->D, bits, G);
  const int64_t tiles = ceil_div64(rows, kBlockN);
  if (p->max_split_rows > 0) return std::max<int64_t>(1, p->max_split_rows / kBlockN);
  double best = 1e300;
  int64_t split = tiles;
  for (int64_t cand = std::max<int64_t>(1, tiles); cand >= 1;) {
    const int64_t items = ceil_div64(tiles, cand);
    const double span = (double)ceil_div64(items * pairs, grid) * ((double)std::min(cand, tiles) + 1.5);
    const double merge = (double)p->B * p->H * items * kConsumerWarps * (p->Dv + 2) * 8.0 /
                         (2.0 * kBlockN * p->D * 0.375 * (double)grid);
    if (items <= kMaxItems && span + merge < best * (1.0 - 1e-3)) {
      best = span + merge;
      split = cand;
    }
    if (cand == 1) break;
    cand = cand > 32 ? cand - std::max<int64_t>(1, cand / 32) : cand - 1;
  }
  return split;
}

static int validate_kivi(const halo_decode_problem_t* p, const halo_kivi_tensor_t* k,
                         const halo_kivi_tensor_t* v, int32_t rows, int32_t bits) {
  if (!p || !k || !v) return fail(HALO_ERR_INVALID_ARG, "NULL argument");
  if (p->B <= 0 || p->H <= 0 || p->H_kv <= 0 || p->H % p->H_kv || rows < 0)
    return fail(HALO_ERR_INVALID_ARG, "bad KIVI decode shape");
  if (p->dtype != HALO_DTYPE_F16 && p->dtype != HALO_DTYPE_BF16)
    return fail(HALO_ERR_UNSUPPORTED, "KIVI decode needs fp16/bf16");
  if ((p->D != 64 && p->D != 128) || p->Dv != p->D)
    return fail(HALO_ERR_UNSUPPORTED, "KIVI decode supports head_dim 64 and 128");
  if (bits != 2 && bits != 4 && bits != 8) return fail(HALO_ERR_UNSUPPORTED, "bits %d", bits);
  for (const halo_kivi_tensor_t* t : {k, v}) {
    if (rows > 0 && (!t->codes || !t->scale || !t->zero))
      return fail(HALO_ERR_INVALID_ARG, "NULL KIVI tensor");
    if (t->t_cap % kBlockN || t->t_cap < ceil_div64(rows, kBlockN) * kBlockN)
      return fail(HALO_ERR_INVALID_ARG, "t_cap must be a multiple of 64 covering the rows");
    if ((reinterpret_cast<uintptr_t>(t->codes) | reinterpret_cast<uintptr_t>(t->scale) |
         reinterpret_cast<uintptr_t>(t->zero)) & 15 ||
        t->codes_stride_b % 16 || t->codes_stride_h % 16 || (t->sz_stride_b * 2) % 16 ||
        (t->sz_stride_h * 2) % 16)
      return fail(HALO_ERR_MISALIGNED, "KIVI tensors need 16-byte aligned bases and strides");
  }
  return HALO_OK;
}

}  // namespace halo

using namespace halo;

extern "C" int64_t halo_decode_workspace_bytes(const halo_decode_problem_t* problem,
                                               const halo_kv_chunk_t* chunks, int32_t n_chunks) {
  int rc = validate_problem(problem, chunks, n_chunks);
  if (rc != HALO_OK) return rc;
  Plan plan = make_plan(problem, chunks, n_chunks);
  return workspace_for(problem, plan.S);
}

// The split-KV launches of a decode: partial (m, l, o) per split in the
// workspace (m [R][S], l [R][S], o [R][S][Dv], each block 256-byte aligned).
static int decode_splits(const halo_decode_problem_t* problem, const halo_kv_chunk_t* chunks,
                         int32_t n_chunks, void* workspace, int64_t workspace_bytes,
                         cudaStream_t st, int* S_out, float** m_out, float** l_out,
                         float** o_out) {
  const halo_decode_problem_t& pb = *problem;
  int rc = HALO_OK;
  Plan plan = make_plan(problem, chunks, n_chunks);
  const int64_t need = workspace_for(problem, plan.S);
  if (plan.S > 0 && (!workspace || workspace_bytes < need))
    return fail(HALO_ERR_WORKSPACE, "workspace %lld bytes < required %lld",
                (long long)workspace_bytes, (long long)need);
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(HALO_ERR_MISALIGNED, "workspace must be 256-byte aligned");

  const int64_t R = (int64_t)pb.B * pb.H;
  char* ws = static_cast<char*>(workspace);
  float* m_part = reinterpret_cast<float*>(ws + kCtrlBytes);
  float* l_part = reinterpret_cast<float*>(ws + kCtrlBytes + align256(R * plan.S * 4));
  float* o_part = reinterpret_cast<float*>(ws + kCtrlBytes + 2 * align256(R * plan.S * 4));

  if (plan.S > 0) {
    const int G = pb.H / pb.H_kv;
    const int gpb = gpb_for(pb.dtype);
    static thread_local DecodeParams prm;  // ~29 KB; kept off the stack
    rc = encode_q_map(pb, &prm.qmap);
    if (rc != HALO_OK) return rc;
    prm.q_pos = pb.q_pos;
    prm.m_part = m_part;
    prm.l_part = l_part;
    prm.o_part = o_part;
    prm.err = device_error_ptr();
    prm.B = pb.B;
    prm.H = pb.H;
    prm.H_kv = pb.H_kv;
    prm.G = G;
    prm.gblocks = (G + gpb - 1) / gpb;
    prm.S = plan.S;
    prm.scale_log2 = pb.scale * kLog2e;
    const int64_t pairs = (int64_t)pb.B * pb.H_kv * prm.gblocks;
    if (pb.event_begin) {
      cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(pb.event_begin), st);
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord(event_begin)");
    }
    if (plan.dyn) {
      prm.ctrl = reinterpret_cast<unsigned int*>(ws);
      prm.n_pairs = plan.n_pairs;
      prm.n_dyn_tiles = plan.n_tiles;
      prm.n_items = (int32_t)plan.items.size();
      prm.n_units = plan.grid;
      for (size_t si = 0; si < plan.segs.size(); ++si) {
        const Seg& sg = plan.segs[si];
        rc = encode_view(sg.view.k, sg.view.len, pb.H_kv, pb.B, pb.D, pb.dtype,
                         sg.view.k_stride_b, sg.view.k_stride_h, sg.view.k_stride_t,
                         &prm.maps[2 * si]);
        if (rc == HALO_OK)
          rc = encode_view(sg.view.v, sg.view.len, pb.H_kv, pb.B, pb.Dv, pb.dtype,
                           sg.view.v_stride_b, sg.view.v_stride_h, sg.view.v_stride_t,
                           &prm.maps[2 * si + 1]);
        if (rc != HALO_OK) return rc;
        prm.items[si] = plan.items[si];
      }
      rc = dispatch_kd_dyn(pb.dtype, pb.D, prm, plan.grid, st);
      if (rc != HALO_OK) return rc;
    }
    // One launch unless the segment or item tables overflow the parameter block.
    size_t i = plan.dyn ? plan.items.size() : 0;
    while (i < plan.items.size()) {
      int n_items = 0, n_seg = 0, last_seg = -1;
      while (i + n_items < plan.items.size() && n_items < kMaxItems) {
        const Item& it = plan.items[i + n_items];
        if (it.seg != last_seg) {
          if (n_seg == kMaxSegs) break;
          const Seg& sg = plan.segs[it.seg];
          rc = encode_view(sg.view.k, sg.view.len, pb.H_kv, pb.B, pb.D, pb.dtype,
                           sg.view.k_stride_b, sg.view.k_stride_h, sg.view.k_stride_t,
                           &prm.maps[2 * n_seg]);
          if (rc == HALO_OK)
            rc = encode_view(sg.view.v, sg.view.len, pb.H_kv, pb.B, pb.Dv, pb.dtype,
                             sg.view.v_stride_b, sg.view.v_stride_h, sg.view.v_stride_t,
                             &prm.maps[2 * n_seg + 1]);
          if (rc != HALO_OK) return rc;
          last_seg = it.seg;
          ++n_seg;
        }
        Item li = it;
        li.seg = n_seg - 1;
        prm.items[n_items] = li;
        ++n_items;
      }
      prm.n_items = n_items;
      prm.n_units = (int32_t)(pairs * n_items);
      rc = dispatch_kd(pb.dtype, pb.D, prm, st);
      if (rc != HALO_OK) return rc;
      i += n_items;
    }
    if (pb.event_end) {
      cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(pb.event_end), st);
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord(event_end)");
    }
  }
  *S_out = plan.S;
  *m_out = m_part;
  *l_out = l_part;
  *o_out = o_part;
  return HALO_OK;
}

extern "C" int32_t halo_chunked_decode(const halo_decode_problem_t* problem,
                                       const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                       void* workspace, int64_t workspace_bytes,
                                       const halo_merge_args_t* merge, halo_stream_t stream) {
  int rc = validate_problem(problem, chunks, n_chunks);
  if (rc != HALO_OK) return rc;
  rc = validate_merge(merge, problem->Dv);
  if (rc != HALO_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int S = 0;
  float *m_part = nullptr, *l_part = nullptr, *o_part = nullptr;
  rc = decode_splits(problem, chunks, n_chunks, workspace, workspace_bytes, st, &S, &m_part,
                     &l_part, &o_part);
  if (rc != HALO_OK) return rc;
  const halo_decode_problem_t& pb = *problem;
  MergeParams mp = merge_params(merge, pb.B, pb.H, pb.Dv, S, m_part, l_part, o_part, 1, S,
                                pb.Dv, (int64_t)S * pb.Dv);
  return launch_merge(mp, st);
}

extern "C" int32_t halo_sharded_merge(int32_t B, int32_t H, int32_t Dv, int32_t P,
                                      const float* m_parts, const float* l_parts,
                                      const float* o_parts, int64_t part_stride,
                                      int64_t row_stride, int64_t o_part_stride,
                                      int64_t o_row_stride, int32_t world, int32_t rank,
                                      void* const* bufs, int32_t out_dtype, void* out,
                                      int64_t out_stride_b, int64_t out_stride_h, float* lse,
                                      halo_stream_t stream);

namespace halo {
int validate_exchange(int32_t B, int32_t H, int32_t Dv, int32_t P, const float* m_parts,
                      const float* o_parts, int32_t world, int32_t rank, void* const* bufs,
                      int32_t out_dtype, const void* out);
}

// The split-KV launch, then the fused cross-GPU merge (kx_kernel, launched
// as a dependent so it is scheduled while the split-KV kernel drains).  The
// exchange arguments are checked before anything is launched.
extern "C" int32_t halo_sharded_decode(const halo_decode_problem_t* problem,
                                       const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                       void* workspace, int64_t workspace_bytes, int32_t world,
                                       int32_t rank, void* const* bufs, int32_t out_dtype,
                                       void* out, int64_t out_stride_b, int64_t out_stride_h,
                                       float* lse, halo_stream_t stream) {
  int rc = validate_problem(problem, chunks, n_chunks);
  if (rc != HALO_OK) return rc;
  const halo_decode_problem_t& pb = *problem;
  // P = 0 here: the partial arrays are the workspace's, placed below
  rc = validate_exchange(pb.B, pb.H, pb.Dv, 0, nullptr, nullptr, world, rank, bufs, out_dtype,
                         out);
  if (rc != HALO_OK) return rc;
  int S = 0;
  float *m_part = nullptr, *l_part = nullptr, *o_part = nullptr;
  rc = decode_splits(problem, chunks, n_chunks, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream), &S, &m_part, &l_part, &o_part);
  if (rc != HALO_OK) return rc;
  return halo_sharded_merge(pb.B, pb.H, pb.Dv, S, m_part, l_part, o_part, 1, S, pb.Dv,
                            (int64_t)S * pb.Dv, world, rank, bufs, out_dtype, out, out_stride_b,
                            out_stride_h, lse, stream);
}

extern "C" int32_t halo_chunked_decode_partials(const halo_decode_problem_t* problem,
                                                const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                                void* workspace, int64_t workspace_bytes,
                                                int32_t* n_parts, int64_t* offsets,
                                                halo_stream_t stream) {
  int rc = validate_problem(problem, chunks, n_chunks);
  if (rc != HALO_OK) return rc;
  if (!n_parts || !offsets) return fail(HALO_ERR_INVALID_ARG, "n_parts/offsets NULL");
  int S = 0;
  float *m_part = nullptr, *l_part = nullptr, *o_part = nullptr;
  rc = decode_splits(problem, chunks, n_chunks, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream), &S, &m_part, &l_part, &o_part);
  if (rc != HALO_OK) return rc;
  const char* ws = static_cast<const char*>(workspace);
  *n_parts = S;
  offsets[0] = reinterpret_cast<const char*>(m_part) - ws;
  offsets[1] = reinterpret_cast<const char*>(l_part) - ws;
  offsets[2] = reinterpret_cast<const char*>(o_part) - ws;
  return HALO_OK;
}

extern "C" int32_t halo_lse_merge(int32_t B, int32_t H, int32_t Dv, int32_t P,
                                  const float* m_parts, const float* l_parts,
                                  const float* o_parts, int64_t part_stride, int64_t row_stride,
                                  int64_t o_part_stride, int64_t o_row_stride,
                                  const halo_merge_args_t* merge, halo_stream_t stream) {
  if (B <= 0 || H <= 0 || Dv <= 0 || P < 0) return fail(HALO_ERR_INVALID_ARG, "bad merge shape");
  if (P > 0 && (!m_parts || !o_parts)) return fail(HALO_ERR_INVALID_ARG, "NULL partial arrays");
  if (Dv > 256 || (Dv > 32 && Dv % ((Dv + 31) / 32 > 2 ? ((Dv + 31) / 32 > 4 ? 8 : 4) : 2)))
    return fail(HALO_ERR_UNSUPPORTED, "Dv %d unsupported", Dv);
  int rc = validate_merge(merge, Dv);
  if (rc != HALO_OK) return rc;
  MergeParams mp = merge_params(merge, B, H, Dv, P, m_parts, l_parts, o_parts, part_stride,
                                row_stride, o_part_stride, o_row_stride);
  return launch_merge(mp, static_cast<cudaStream_t>(stream));
}

extern "C" const char* halo_last_error_string(void) { return halo::t_last_error.c_str(); }

extern "C" int32_t halo_device_error(int32_t* code_out, int32_t clear) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, halo::g_device_error, sizeof(v));
  if (e != cudaSuccess) return halo::cuda_fail(e, "read device error word");
  if (clear) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(halo::g_device_error, &z, sizeof(z));
    if (e != cudaSuccess) return halo::cuda_fail(e, "clear device error word");
  }
  if (code_out) *code_out = v ? -static_cast<int32_t>(v) : 0;
  return HALO_OK;
}

extern "C" int32_t halo_version(void) { return 100; }

extern "C" uint64_t halo_launch_count(void) {
  return halo::g_launch_count.load(std::memory_order_relaxed);
}

extern "C" int64_t halo_kivi_decode_workspace_bytes(const halo_decode_problem_t* problem,
                                                    int32_t rows) {
  if (!problem || rows < 0) return fail(HALO_ERR_INVALID_ARG, "bad arguments");
  // the split depends on the kernel variant's occupancy: size for the
  // largest over the code widths
  int64_t items = 0;
  for (int bits : {2, 4, 8}) {
    const int64_t split = kivi_split_tiles(problem, rows, bits);
    if (rows > 0) items = std::max(items, ceil_div64(ceil_div64(rows, kBlockN), split));
  }
  return workspace_for(problem, (int)(items * kConsumerWarps));
}

extern "C" int32_t halo_kivi_decode(const halo_decode_problem_t* problem,
                                    const halo_kivi_tensor_t* k, const halo_kivi_tensor_t* v,
                                    int32_t rows, int32_t bits, int64_t start, int32_t causal,
                                    void* workspace, int64_t workspace_bytes,
                                    const halo_merge_args_t* merge, halo_stream_t stream) {
  int rc = validate_kivi(problem, k, v, rows, bits);
  if (rc != HALO_OK) return rc;
  rc = validate_merge(merge, problem->Dv);
  if (rc != HALO_OK) return rc;
  if (causal && !problem->q_pos) return fail(HALO_ERR_INVALID_ARG, "causal needs q_pos");
  const halo_decode_problem_t& pb = *problem;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t split = kivi_split_tiles(problem, rows, bits);
  const int64_t tiles = ceil_div64(rows, kBlockN);
  const int n_items = rows > 0 ? (int)ceil_div64(tiles, split) : 0;
  if (n_items > kMaxItems) return fail(HALO_ERR_UNSUPPORTED, "too many KIVI work items");
  const int S = n_items * kConsumerWarps;
  const int64_t need = workspace_for(problem, S);
  if (S > 0 && (!workspace || workspace_bytes < need))
    return fail(HALO_ERR_WORKSPACE, "workspace %lld bytes < required %lld",
                (long long)workspace_bytes, (long long)need);
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(HALO_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  const int64_t R = (int64_t)pb.B * pb.H;
  char* ws = static_cast<char*>(workspace);
  float* m_part = reinterpret_cast<float*>(ws + kCtrlBytes);
  float* l_part = reinterpret_cast<float*>(ws + kCtrlBytes + align256(R * S * 4));
  float* o_part = reinterpret_cast<float*>(ws + kCtrlBytes + 2 * align256(R * S * 4));
  if (S > 0) {
    static thread_local KiviParams prm;
    rc = encode_q_map(pb, &prm.qmap);
    if (rc != HALO_OK) return rc;
    const int G = pb.H / pb.H_kv;
    prm.q_pos = pb.q_pos;
    prm.m_part = m_part;
    prm.l_part = l_part;
    prm.o_part = o_part;
    prm.err = device_error_ptr();
    prm.B = pb.B;
    prm.H = pb.H;
    prm.H_kv = pb.H_kv;
    prm.G = G;
    prm.gblocks = (G + 15) / 16;
    prm.S = S;
    prm.scale_log2 = pb.scale * kLog2e;
    prm.n_items = n_items;
    prm.n_units = (int32_t)((int64_t)pb.B * pb.H_kv * prm.gblocks * n_items);
    const halo_kivi_tensor_t* src[2] = {k, v};
    for (int w = 0; w < 2; ++w) {
      prm.kv[w].codes = src[w]->codes;
      prm.kv[w].scale = static_cast<const char*>(src[w]->scale);
      prm.kv[w].zero = static_cast<const char*>(src[w]->zero);
      prm.kv[w].c_sb = src[w]->codes_stride_b;
      prm.kv[w].c_sh = src[w]->codes_stride_h;
      prm.kv[w].s_sb = src[w]->sz_stride_b * 2;
      prm.kv[w].s_sh = src[w]->sz_stride_h * 2;
    }
    for (int i = 0; i < n_items; ++i) {
      Item& it = prm.items[i];
      it.seg = 0;
      it.row0 = (int32_t)(i * split * kBlockN);
      it.rows = (int32_t)std::min<int64_t>(split * kBlockN, rows - it.row0);
      it.start = start + it.row0;
      it.slot = i * kConsumerWarps;
      it.causal = causal;
      it.b_bcast = 0;
    }
    if (pb.event_begin) cudaEventRecord(static_cast<cudaEvent_t>(pb.event_begin), st);
    rc = pb.dtype == HALO_DTYPE_F16 ? dispatch_kk_t<__half>(pb.D, bits, prm, st)
                                    : dispatch_kk_t<__nv_bfloat16>(pb.D, bits, prm, st);
    if (rc != HALO_OK) return rc;
    if (pb.event_end) cudaEventRecord(static_cast<cudaEvent_t>(pb.event_end), st);
  }
  MergeParams mp = merge_params(merge, pb.B, pb.H, pb.Dv, S, m_part, l_part, o_part, 1, S, pb.Dv,
                                (int64_t)S * pb.Dv);
  return launch_merge(mp, st);
}
