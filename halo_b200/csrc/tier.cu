// Tier movement between the pinned host cold tier and HBM.
//
// A cold tier stores one layer as (B, H_kv, T_cap, D) in pinned memory; a
// row range [a, b) of it is B*H_kv pieces of (b-a)*D contiguous elements
// spaced T_cap*D apart.  One pitched copy moves the whole range with the DMA
// engines (no contiguous staging copy, no host synchronisation), in either
// direction.  Replaces the strided `.to(device)` / `.to("cpu")` slice copies
// of halo/kv_cache_chunked.py:441-446, :469-483 (peel) and :716-717, :884-885
// (per-chunk refetch) in lzbaclz/HALO.
#include "halo_common.cuh"

namespace halo {
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
}  // namespace halo

extern "C" int32_t halo_copy2d_async(void* dst, int64_t dst_pitch, const void* src,
                                     int64_t src_pitch, int64_t width_bytes, int64_t height,
                                     halo_stream_t stream) {
  if (width_bytes < 0 || height < 0 || dst_pitch < width_bytes || src_pitch < width_bytes)
    return halo::fail(HALO_ERR_INVALID_ARG, "bad 2-D copy geometry");
  if (width_bytes == 0 || height == 0) return HALO_OK;
  if (!dst || !src) return halo::fail(HALO_ERR_INVALID_ARG, "NULL copy pointer");
  cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)dst_pitch, src, (size_t)src_pitch,
                                    (size_t)width_bytes, (size_t)height, cudaMemcpyDefault,
                                    static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HALO_OK : halo::cuda_fail(e, "cudaMemcpy2DAsync");
}
