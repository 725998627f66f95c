/*
 * halo_b200.h -- C ABI of libhalo_sm100.so, the B200 (sm_100a) kernels of
 * HALO's chunked-attention hot path.
 *
 * Conventions
 *  - Every entry point returns 0 (HALO_OK) or a negative HALO_ERR_* code;
 *    halo_last_error_string() describes the last failure of the calling
 *    thread.
 *  - Pointers marked "device" are CUDA device pointers; strides are in
 *    ELEMENTS; the innermost (head_dim) dimension is always contiguous.
 *  - All work is enqueued on the given stream; nothing synchronises the host.
 *  - The library allocates no device memory: callers pass workspaces sized by
 *    the matching *_workspace_bytes() query.  A decode workspace starts with
 *    a 4096-byte control block (the dynamic schedule's counters) that must
 *    be zero before the workspace's first use; every call leaves it zero, so
 *    zero a workspace once when allocating it and reuse it freely (one call
 *    in flight per workspace).
 *  - Kernels never wait without a limit: a wait that exceeds ~2 s records
 *    HALO_ERR_TIMEOUT in the per-device error word (halo_device_error) and
 *    the kernel returns.
 *
 * Reference interfaces replaced (paths relative to the lzbaclz/HALO root):
 *  - halo/triton_chunked.py:47-138   _chunked_lse_merge_kernel (Triton)
 *  - halo/triton_chunked.py:141-207  init_acc / update_chunk / finalize
 *  - halo/kv_cache_chunked.py:194-276 _lse_merge / _chunk_attention
 */
#ifndef HALO_B200_H_
#define HALO_B200_H_

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define HALO_OK 0
#define HALO_ERR_INVALID_ARG (-1)   /* bad shape, null pointer, bad enum     */
#define HALO_ERR_UNSUPPORTED (-2)   /* valid but not implemented (e.g. D)    */
#define HALO_ERR_MISALIGNED (-3)    /* pointer/stride not 16-byte aligned    */
#define HALO_ERR_CUDA (-4)          /* a CUDA runtime call failed            */
#define HALO_ERR_TIMEOUT (-5)       /* a device-side bounded wait expired    */
#define HALO_ERR_WORKSPACE (-6)     /* workspace missing or too small        */
#define HALO_ERR_SPLIT (-7)         /* reserved (no longer returned)          */

/* ------------------------------------------------------------------ dtypes */
#define HALO_DTYPE_F32 0
#define HALO_DTYPE_BF16 1
#define HALO_DTYPE_F16 2

/* Opaque CUDA stream (cudaStream_t); 0 = legacy default stream. */
typedef void* halo_stream_t;

/* One KV chunk: element (b, h, t, d) of K lives at
 *   k + b*k_stride_b + h*k_stride_h + t*k_stride_t + d      (elements)
 * and likewise for V.  `start` is the global position of row t = 0; when
 * `causal` is nonzero, key t is visible to batch row b iff
 * start + t <= q_pos[b].  Mirrors one (k, v, chunk_start, apply_causal)
 * tuple of triton_chunked_attention (halo/triton_chunked.py:210-267). */
typedef struct halo_kv_chunk {
  const void* k;
  const void* v;
  int64_t k_stride_b, k_stride_h, k_stride_t;
  int64_t v_stride_b, v_stride_h, v_stride_t;
  int64_t start;
  int32_t len;
  int32_t causal;
} halo_kv_chunk_t;

/* The decode query and its shape.  q is (B, H, D) with strides
 * (q_stride_b, q_stride_h, 1).  Query head h reads KV head h / (H / H_kv)
 * (GQA, halo/triton_chunked.py:73).  q_pos is a device int64 (B,) array of
 * global query positions, required when any chunk is causal. */
typedef struct halo_decode_problem {
  int32_t B, H, H_kv, D, Dv;
  int32_t dtype;               /* HALO_DTYPE_* of q, k and v */
  const void* q;
  int64_t q_stride_b, q_stride_h;
  const int64_t* q_pos;
  float scale;                 /* softmax scale, e.g. 1/sqrt(D) */
  int32_t max_split_rows;      /* 0 = automatic split size */
  /* Optional profiling hooks (cudaEvent_t or NULL): recorded on `stream`
   * right before the first and right after the last split-KV launch, so a
   * caller can time the decode kernel apart from the merge. */
  void* event_begin;
  void* event_end;
} halo_decode_problem_t;

/* Where the merged result goes.
 * mode HALO_MERGE_FINALIZE: out (B, H, Dv) in out_dtype with strides
 *   (out_stride_b, out_stride_h, 1) gets softmax(qk) @ v (zeros where no key
 *   is visible, halo/triton_chunked.py:195-207); lse (B, H) fp32 contiguous,
 *   optional, gets the natural-log log-sum-exp (-inf where no key is visible).
 *   If m/l/o are non-NULL they are folded in first as a prior running state.
 * mode HALO_MERGE_ACCUMULATE: the running fp32 accumulators m (B, H),
 *   l (B, H), o (B, H, Dv) (contiguous) of halo/triton_chunked.py:141-148 are
 *   updated in place: m = running max score, l = sum exp(s - m),
 *   o = sum exp(s - m) v, exactly the state update_chunk maintains. */
#define HALO_MERGE_FINALIZE 0
#define HALO_MERGE_ACCUMULATE 1
typedef struct halo_merge_args {
  int32_t mode;
  int32_t out_dtype;
  void* out;
  int64_t out_stride_b, out_stride_h;
  float* lse;
  float* m;
  float* l;
  float* o;
} halo_merge_args_t;

/* ------------------------------------------------------------------ decode */

/* Bytes of device workspace halo_chunked_decode needs for this problem and
 * chunk list: the zeroed control block, then the partial (m, l, o) per
 * split.  Returns < 0 on invalid input. */
int64_t halo_decode_workspace_bytes(const halo_decode_problem_t* problem,
                                    const halo_kv_chunk_t* chunks, int32_t n_chunks);

/* Split-KV chunked decode attention with a fused log-sum-exp merge.
 * Replaces the per-chunk Triton launches of update_chunk
 * (halo/triton_chunked.py:151-192, kernel :47-138) and the torch loop of
 * _chunk_attention + _lse_merge (halo/kv_cache_chunked.py:194-276) with one
 * split-KV launch over every chunk plus one merge launch (a programmatic
 * dependent launch, scheduled while the split-KV kernel drains; recording
 * an event between the two on the stream forfeits that overlap).  `chunks`
 * is a HOST array; K/V rows are staged through the async-copy engine, so
 * every row address must be 16-byte aligned.  The default schedule hands rows to CTAs at run time,
 * so results can differ between calls in the last bits of fp32;
 * max_split_rows > 0 selects a fixed split, bit-reproducible. */
int32_t halo_chunked_decode(const halo_decode_problem_t* problem,
                            const halo_kv_chunk_t* chunks, int32_t n_chunks,
                            void* workspace, int64_t workspace_bytes,
                            const halo_merge_args_t* merge, halo_stream_t stream);

/* Merge P partial states into R = B*H rows with the semantics of `merge`.
 * Part s of row r has max-score/LSE m_parts[s*part_stride + r*row_stride],
 * weight l_parts[same index] (l_parts NULL: every part is normalised, l = 1,
 * so m is its LSE) and output o_parts[s*o_part_stride + r*o_row_stride + d]
 * (fp32).  This is the LSE merge of halo/kv_cache_chunked.py:194-239
 * generalised to P parts; with (o, lse) parts gathered from several GPUs it
 * is the merge step of the sequence-sharded decode. */
int32_t halo_lse_merge(int32_t B, int32_t H, int32_t Dv, int32_t P,
                       const float* m_parts, const float* l_parts, const float* o_parts,
                       int64_t part_stride, int64_t row_stride,
                       int64_t o_part_stride, int64_t o_row_stride,
                       const halo_merge_args_t* merge, halo_stream_t stream);

/* Same as halo_chunked_decode, but allocates nothing and takes no workspace:
 * the partial (m, l, o) scratch lives in a fixed 8 MiB device array inside
 * the library.  No counterpart in the reference (its Triton path allocates
 * through torch); this exists for callers that cannot allocate device memory
 * when they need attention -- code whose framework owns every device
 * allocation, plugin hosts that forbid cudaMalloc on the hot path, C/FFI
 * callers without an allocator.  Problems needing more than 8 MiB of scratch
 * (halo_decode_workspace_bytes) are rejected with HALO_ERR_WORKSPACE.  Every
 * GPU that loads the library holds the array until exit.  All calls on a
 * device share it and it keeps the last call's contents; each call clears
 * its leading scheduler counters on `stream` before the kernels.  Calls that
 * overlap on the GPU race: serialise them.  The first call on each device
 * looks up the array's address (make it before any stream capture); the
 * address is kept for the life of the process, so do not use this entry
 * point on a device after cudaDeviceReset (or any other teardown of its
 * primary context) in the same process. */
int32_t halo_chunked_decode_noalloc(const halo_decode_problem_t* problem,
                                    const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                    const halo_merge_args_t* merge, halo_stream_t stream);

/* Only the split-KV launches of halo_chunked_decode: the per-split partial
 * state stays in `workspace` for the caller to merge (e.g. across GPUs with
 * halo_sharded_merge).  On return *n_parts = S and offsets[0..2] are the byte
 * offsets in the workspace of m [B*H][S], l [B*H][S] and o [B*H][S][Dv]
 * (fp32; m in natural-log score units, l = sum exp(s - m), o unnormalised).
 * Same inputs and workspace size as halo_chunked_decode. */
int32_t halo_chunked_decode_partials(const halo_decode_problem_t* problem,
                                     const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                     void* workspace, int64_t workspace_bytes,
                                     int32_t* n_parts, int64_t* offsets, halo_stream_t stream);

/* ------------------------------------------------------- multi-GPU merge */

/* Bytes of one rank's exchange buffer for `world` ranks, `rows` = B*H output
 * rows of Dv values: words[2][world][rows][Dv + 2] (64-bit: epoch tag and
 * fp32 value; o, lse, pad per row), then 16 bytes of control words (the
 * buffer's call epoch).  The
 * buffer must start zeroed (halo_ipc_alloc does) and serves one sequence
 * of calls with one (world, rows, Dv). */
int64_t halo_exchange_bytes(int32_t world, int32_t rows, int32_t Dv);

/* Exchange buffers shared across the processes of one node: halo_ipc_alloc
 * allocates and zeroes `bytes` of device memory on the current device and
 * writes its 64-byte CUDA IPC handle to handle_out; halo_ipc_open maps a
 * peer's handle into this process (peer access over NVLink); close/free
 * undo them. */
int32_t halo_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle_out);
int32_t halo_ipc_open(const void* handle, void** dev_ptr);
int32_t halo_ipc_close(void* dev_ptr);
int32_t halo_ipc_free(void* dev_ptr);

/* The cross-GPU step of a sequence-sharded decode in one kernel per rank:
 * merge this rank's P local partials (layout as halo_lse_merge), write the
 * normalised (o, lse) row, tagged with the call's epoch, into slot `rank`
 * of every rank's exchange buffer (bufs[j] = rank j's buffer mapped in this
 * process, bufs[rank] its own) through NVLink peer stores, wait for the
 * rows of all ranks (bounded: HALO_ERR_TIMEOUT in the device error word
 * after 2 s), and write the merged out (B, H, Dv) in out_dtype
 * and lse (B, H) (optional).  Every rank makes the same sequence of calls;
 * the epoch is counted on the device in the rank's own buffer, so the call
 * can be captured in a CUDA graph and replayed.  Replaces, for the sharded
 * decode, the local merge + all-gather + merge of (o, lse); the reference
 * (halo/kv_cache_chunked.py:194-239, single GPU) has no counterpart. */
int32_t halo_sharded_merge(int32_t B, int32_t H, int32_t Dv, int32_t P, const float* m_parts,
                           const float* l_parts, const float* o_parts, int64_t part_stride,
                           int64_t row_stride, int64_t o_part_stride, int64_t o_row_stride,
                           int32_t world, int32_t rank, void* const* bufs,
                           int32_t out_dtype, void* out, int64_t out_stride_b,
                           int64_t out_stride_h, float* lse, halo_stream_t stream);

/* One step of a sequence-sharded decode on this rank: attention of q over
 * this rank's chunks, merged with every rank's result through the exchange
 * buffers of halo_sharded_merge (same buffers, same call-sequence rule).
 * Two launches: the split-KV kernel, then halo_sharded_merge's kernel as a
 * programmatic dependent launch (scheduled while the first drains).
 * Inputs as halo_chunked_decode (workspace sized by
 * halo_decode_workspace_bytes, Dv == D); out (B, H, Dv) in out_dtype, lse
 * (B, H) optional.  No reference counterpart (the reference is single-GPU;
 * its merge identity is halo/kv_cache_chunked.py:194-239). */
int32_t halo_sharded_decode(const halo_decode_problem_t* problem,
                            const halo_kv_chunk_t* chunks, int32_t n_chunks, void* workspace,
                            int64_t workspace_bytes, int32_t world, int32_t rank,
                            void* const* bufs, int32_t out_dtype, void* out,
                            int64_t out_stride_b, int64_t out_stride_h, float* lse,
                            halo_stream_t stream);

/* ------------------------------------------------------------------ KIVI */

/* Per-group round-to-nearest quantisation of x (B, H, T, D) (element strides
 * x_sb, x_sh, x_st, fp16 or bf16) along head_dim in groups of `group`, to
 * `bits` (2/4/8) codes packed 8/bits per byte (4/8 bits: code i of a row at
 * byte i*bits/8, bit (i*bits)%8; 2 bits: 16 codes per little-endian 32-bit
 * word, code i at word i/16, bit 16*(e&1) + 2*(e>>1) with e = i%16, group a
 * multiple of 16; byte strides c_sb/c_sh/c_st) plus per-group
 * scale and zero in x's dtype (element strides s_sb/s_sh/s_st).  Bit-exact
 * with _quantize_per_group (baselines/kivi_cache.py:44-69), whose every op
 * rounds to the tensor dtype. */
int32_t halo_kivi_quantize(const void* x, int64_t x_sb, int64_t x_sh, int64_t x_st,
                           int32_t B, int32_t H, int32_t T, int32_t D, int32_t dtype,
                           int32_t bits, int32_t group, uint8_t* codes, int64_t c_sb,
                           int64_t c_sh, int64_t c_st, void* scale, void* zero, int64_t s_sb,
                           int64_t s_sh, int64_t s_st, halo_stream_t stream);

/* Inverse: x = rnd(fl32(code * scale) + zero), bit-exact with
 * _dequantize_per_group (baselines/kivi_cache.py:72-78). */
int32_t halo_kivi_dequantize(const uint8_t* codes, int64_t c_sb, int64_t c_sh, int64_t c_st,
                             const void* scale, const void* zero, int64_t s_sb, int64_t s_sh,
                             int64_t s_st, int32_t B, int32_t H, int32_t T, int32_t D,
                             int32_t dtype, int32_t bits, int32_t group, void* x, int64_t x_sb,
                             int64_t x_sh, int64_t x_st, halo_stream_t stream);

/* A KIVI-packed K or V: codes (B, H_kv, t_cap, D*bits/8) bytes with
 * contiguous rows, scale/zero (B, H_kv, t_cap, D/32) in the problem dtype
 * with contiguous rows; t_cap a multiple of 64 (tiles are read whole). */
typedef struct halo_kivi_tensor {
  const uint8_t* codes;
  const void* scale;
  const void* zero;
  int64_t codes_stride_b, codes_stride_h;   /* bytes */
  int64_t sz_stride_b, sz_stride_h;         /* elements */
  int64_t t_cap;
} halo_kivi_tensor_t;

int64_t halo_kivi_decode_workspace_bytes(const halo_decode_problem_t* problem, int32_t rows);

/* Fused 2/4/8-bit dequantise-and-attend decode over rows [0, rows) of a
 * KIVI-packed K/V (group 32, head_dim 64 or 128, fp16/bf16), rows at global
 * positions start + t, then the LSE merge described by `merge`.  Replaces
 * the per-step full dequantisation of KIVICache.update + SDPA
 * (baselines/kivi_cache.py:187-195). */
int32_t halo_kivi_decode(const halo_decode_problem_t* problem, const halo_kivi_tensor_t* k,
                         const halo_kivi_tensor_t* v, int32_t rows, int32_t bits, int64_t start,
                         int32_t causal, void* workspace, int64_t workspace_bytes,
                         const halo_merge_args_t* merge, halo_stream_t stream);

/* ------------------------------------------------------------------ scorer */

/* Per-page channel-wise min/max of K (B, H_kv, T, D) for pages
 * [page_begin, page_begin + n_pages) of `page_size` rows, written to
 * kmin/kmax at element (b, h, page, d) = b*o_sb + h*o_sh + page*o_sp + d, in
 * K's dtype (exact).  Replaces _QuestScorerAdapter.observe_keys
 * (baselines/quest_path_d.py:125-150). */
int32_t halo_page_summary(const void* k, int64_t k_sb, int64_t k_sh, int64_t k_st,
                          int32_t B, int32_t H_kv, int32_t D, int32_t dtype,
                          int32_t page_size, int32_t page_begin, int32_t n_pages,
                          void* kmin, void* kmax, int64_t o_sb, int64_t o_sh, int64_t o_sp,
                          halo_stream_t stream);

/* Quest upper-bound page scores and top-k.  q is (B, H, T_q, D) with element
 * strides (q_sb, q_sh, q_st, 1); it is mean-pooled over each GQA group in
 * fp32 and rounded once to its dtype, then scores[b][h_kv][t][p] =
 * sum_d max(q_d * kmin_d, q_d * kmax_d) in fp32 (contiguous (B, H_kv, T_q, P)
 * output).  With k > 0, per_page (optional, (P,)) gets the max over
 * (b, h_kv, t) and topk ((k,) int64) the k best pages, largest first, ties
 * to the lower index, skipping pages with exclude[p] != 0 (optional).
 * P <= 16384 when k > 0.  Replaces _QuestScorerAdapter.score_pages and
 * select_hot_pages (baselines/quest_path_d.py:153-205). */
int32_t halo_page_score_topk(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                             int32_t B, int32_t H, int32_t T_q, int32_t H_kv, int32_t D,
                             int32_t dtype, const void* kmin, const void* kmax, int64_t o_sb,
                             int64_t o_sh, int64_t o_sp, int32_t P, float* scores,
                             const uint8_t* exclude, int32_t k, float* per_page, int64_t* topk,
                             halo_stream_t stream);

/* Per-page mean key of the HALOPress ablation scorer (observe_keys of
 * baselines/scorer_ablations.py:208-218): for pages page_begin ..
 * page_begin + n_pages - 1 of K (B, H_kv, T, D), kmean[b][h][p][d] = fp32 sum
 * over the page's rows in row order, divided by page_size, rounded once to
 * the key dtype.  Strides as halo_page_summary. */
int32_t halo_page_mean(const void* k, int64_t k_sb, int64_t k_sh, int64_t k_st, int32_t B,
                       int32_t H_kv, int32_t D, int32_t dtype, int32_t page_size,
                       int32_t page_begin, int32_t n_pages, void* kmean, int64_t o_sb,
                       int64_t o_sh, int64_t o_sp, halo_stream_t stream);

/* HALOPress page selection (select_hot_pages of
 * baselines/scorer_ablations.py:220-268): scores[b][h_kv][t][p] = q_g . kmean
 * (fp32; q_g the GQA mean rounded to q's dtype, as halo_page_score_topk);
 * attn = max over (b, h_kv, t), minus its min, divided by its max when
 * positive; rec = exp(-(P-1-p)/refresh_window) over its sum (+1e-12) over
 * its max (+1e-12); sink = 1 for the first n_sink_pages pages; score =
 * alpha*attn + beta*rec + gamma*sink (one rounding per operation) into
 * per_page (optional); topk ((k,) int64) gets the k best pages, largest
 * first, ties to the lower index.  P <= 8192. */
int32_t halo_page_press_topk(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, int32_t B,
                             int32_t H, int32_t T_q, int32_t H_kv, int32_t D, int32_t dtype,
                             const void* kmean, int64_t o_sb, int64_t o_sh, int64_t o_sp,
                             int32_t P, float alpha, float beta, float gamma,
                             int32_t refresh_window, int32_t n_sink_pages, float* scores,
                             int32_t k, float* per_page, int64_t* topk, halo_stream_t stream);

/* ---------------------------------------------------------------- prefill */
/* Multi-query (chunked-prefill) attention on the 5th-generation tensor cores:
 * T_q query rows per (b, h) at global positions q_pos0 .. q_pos0 + T_q - 1
 * attend to a list of K/V chunks (a chunk's `causal` flag hides keys after
 * each query row).  Replaces the T_q > 1 branch of
 * HALOCacheChunked.compute_attention (halo/kv_cache_chunked.py:873-942) that
 * halo/chunked_prefill.py:73-135 drives slice by slice.  q is
 * (B, H, T_q, D) with element strides (q_stride_b, q_stride_h, q_stride_t, 1);
 * query head h reads KV head h / (H / H_kv).  bf16 or fp16, D = 64 or 128,
 * value head dim equal to D.  Chunks that continue each other in memory and
 * position are coalesced; at most 48 remain per call (HALO_ERR_UNSUPPORTED
 * beyond: split the list and carry the running state). */
typedef struct halo_prefill_problem {
  int32_t B, H, H_kv, T_q, D;
  int32_t dtype;               /* HALO_DTYPE_BF16 or HALO_DTYPE_F16 */
  const void* q;
  int64_t q_stride_b, q_stride_h, q_stride_t;
  int64_t q_pos0;
  float scale;
  void* event_begin;           /* optional cudaEvent_t around the kernel */
  void* event_end;
} halo_prefill_problem_t;

/* Result of halo_prefill_attention, per (b, h, t) row:
 * mode HALO_MERGE_FINALIZE: out (B, H, T_q, D) in out_dtype (F32 or the input
 *   dtype) with element strides (out_stride_b, out_stride_h, out_stride_t, 1);
 *   lse (B, H, T_q) fp32 contiguous, optional.  Rows with no visible key get
 *   zeros and -inf.  If m/l/o are non-NULL they are folded in first.
 * mode HALO_MERGE_ACCUMULATE: the running state m, l (B, H, T_q) and
 *   o (B, H, T_q, D), fp32 contiguous, with the meaning of halo_merge_args_t,
 *   is updated in place. */
typedef struct halo_prefill_out {
  int32_t mode;
  int32_t out_dtype;
  void* out;
  int64_t out_stride_b, out_stride_h, out_stride_t;
  float* lse;
  float* m;
  float* l;
  float* o;
} halo_prefill_out_t;

/* Any chunk order is accepted: the kernel's single MMA issuer polls its
 * inputs and never waits on one step while another could go (a CTA's two
 * query tiles walk the union of their K/V tiles; the earlier tile sits out
 * the tiles only the later one can see).  Without a workspace, bf16 inputs
 * run P V as two bf16 MMAs (P as high part + residual); see
 * halo_prefill_attention_ws for the single-MMA route. */
int32_t halo_prefill_attention(const halo_prefill_problem_t* problem,
                               const halo_kv_chunk_t* chunks, int32_t n_chunks,
                               const halo_prefill_out_t* out, halo_stream_t stream);

/* Workspace bytes halo_prefill_attention_ws needs for this problem and chunk
 * list: 256 bytes of flags, then for bf16 inputs an fp16 copy of V
 * (B x H_kv x rows x D x 2 bytes per coalesced segment, each rounded up to
 * 256), then, when there are more query-tile pairs x heads than SMs with a
 * remainder, fp32 partials for the last wave's pairs, which run as two
 * half-walk CTAs each (2 x 2 x 128 rows x (D + 4) floats per such pair).
 * 0 when none of these apply (fp16 inputs, a single wave).  Negative status
 * on bad arguments. */
int64_t halo_prefill_workspace_bytes(const halo_prefill_problem_t* problem,
                                     const halo_kv_chunk_t* chunks, int32_t n_chunks);

/* halo_prefill_attention with a caller workspace (256-byte aligned, at least
 * halo_prefill_workspace_bytes; its contents need no initialisation and are
 * overwritten).  For bf16 inputs a pre-pass writes an fp16 copy of V into
 * the workspace, so P enters P V as one fp16 operand (one MMA instead of
 * two; max error well inside 2e-3).  If V holds a finite |v| >= 65536, which
 * fp16 cannot represent, the pre-pass raises a flag in the workspace and the
 * kernel takes the two-MMA bf16 route with the original V: same result
 * contract, no host round trip.  For a finalising call without a running
 * state, the last partial wave's query-tile pairs run as two CTAs over half
 * of their keys each, merged by one more launch (fills the SMs the last wave
 * would leave idle).  Same semantics as halo_prefill_attention otherwise.
 * Same reference interface as halo_prefill_attention. */
int32_t halo_prefill_attention_ws(const halo_prefill_problem_t* problem,
                                  const halo_kv_chunk_t* chunks, int32_t n_chunks,
                                  const halo_prefill_out_t* out, void* workspace,
                                  int64_t workspace_bytes, halo_stream_t stream);

/* ------------------------------------------------------------------ tiers */

/* Pitched async copy of `height` rows of `width_bytes` between any two of
 * pinned host / device memory (cudaMemcpyDefault), on `stream`.  Moves a
 * (B, H_kv, rows, D) slice of a (B, H_kv, T_cap, D) tier in one DMA.
 * Replaces the strided slice copies of halo/kv_cache_chunked.py:441-446,
 * :469-483 (peel to host) and :716-717, :884-885 (refetch to HBM). */
int32_t halo_copy2d_async(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                          int64_t width_bytes, int64_t height, halo_stream_t stream);

/* ------------------------------------------------------------------ misc */
const char* halo_last_error_string(void);
/* Read (and optionally clear) the device error word of the current device.
 * Synchronises the current device. */
int32_t halo_device_error(int32_t* code_out, int32_t clear);
/* ABI version: major*10000 + minor*100 + patch. */
int32_t halo_version(void);
/* Number of kernels this library has launched in this process (all devices,
 * all streams).  A counter for benchmarks and tests; no reference
 * counterpart. */
uint64_t halo_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* HALO_B200_H_ */
