// KIVI per-group quantise / dequantise for B200, bit-exact with the
// reference's torch ops (baselines/kivi_cache.py:44-78 in lzbaclz/HALO).
//
// Every torch op there rounds its exact result once to the tensor dtype
// (fp16 or bf16).  Here each step is an IEEE fp32 operation (exact or
// correctly rounded; fp32 keeps enough bits for the second rounding to be
// innocuous) followed by one round-to-nearest-even into the 16-bit type:
//   mn, mx    = min / max of the group                      (exact)
//   d         = rnd(mx - mn); d = max(d, rnd(1e-8))         (scalar cast first)
//   s         = rnd(d / qmax);  z = mn
//   q         = clamp(rint(rnd(rnd(x - z) / s)), 0, qmax)   (NaN -> 0)
//   dequant   = rnd(fl32(q * s) + z)                        (no fused multiply-add)
// Codes are packed 8/bits per byte along head_dim.  4 and 8 bits: code i of
// a row sits in byte i*bits/8 at bit (i*bits) % 8.  2 bits: each
// little-endian 32-bit word holds 16 codes laid out for the decoder -- code
// i of the row sits in word i/16 at bit 16*(e & 1) + 2*(e >> 1), e = i % 16
// -- so the two codes of each consecutive pair (2q, 2q+1) share bit 2q of
// the word's two 16-bit halves and one mask yields both as a packed pair
// (halo_b200.h documents the layout).  Scale and zero are stored per group
// in the 16-bit type, as the reference stores them.
#include <cstdint>

#include "halo_common.cuh"

namespace halo {

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return Elem<T>::to_f32(Elem<T>::from_f32(x));
}

struct QuantParams {
  const char* x;            // (B, H, T, D) rows, element strides
  int64_t x_sb, x_sh, x_st;
  uint8_t* codes;           // (B, H, T, D*bits/8) bytes
  int64_t c_sb, c_sh, c_st;
  char* scale;              // (B, H, T, D/group), element strides
  char* zero;
  int64_t s_sb, s_sh, s_st;
  int32_t H, T, D, group, bits;
  int64_t n_groups;         // B*H*T*(D/group)
};

// One thread per (row, group).
template <typename T>
__global__ void __launch_bounds__(256) kivi_quantize_kernel(const QuantParams p) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= p.n_groups) return;
  const int gpr = p.D / p.group;
  const int g = (int)(gid % gpr);
  int64_t row = gid / gpr;
  const int t = (int)(row % p.T);
  row /= p.T;
  const int h = (int)(row % p.H);
  const int b = (int)(row / p.H);
  const T* x = reinterpret_cast<const T*>(p.x) + b * p.x_sb + h * p.x_sh + (int64_t)t * p.x_st +
               g * p.group;
  const float qmax = (float)((1 << p.bits) - 1);
  float mn = Elem<T>::to_f32(x[0]), mx = mn;
  for (int i = 1; i < p.group; ++i) {
    const float v = Elem<T>::to_f32(x[i]);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  float d = rnd<T>(mx - mn);
  const float eps = rnd<T>(1e-8f);
  d = d < eps ? eps : d;
  const float s = rnd<T>(__fdiv_rn(d, qmax));
  T* sc = reinterpret_cast<T*>(p.scale) + b * p.s_sb + h * p.s_sh + (int64_t)t * p.s_st + g;
  T* ze = reinterpret_cast<T*>(p.zero) + b * p.s_sb + h * p.s_sh + (int64_t)t * p.s_st + g;
  *sc = Elem<T>::from_f32(s);
  *ze = Elem<T>::from_f32(mn);
  uint8_t* out = p.codes + b * p.c_sb + h * p.c_sh + (int64_t)t * p.c_st +
                 (int64_t)g * p.group * p.bits / 8;
  auto code = [&](int i) -> uint32_t {
    const float tt = rnd<T>(__fsub_rn(Elem<T>::to_f32(x[i]), mn));
    const float u = rnd<T>(__fdiv_rn(tt, s));
    const float r = rintf(u);
    return isnan(r) ? 0u : (uint32_t)fminf(fmaxf(r, 0.f), qmax);
  };
  if (p.bits == 2) {
    // groups are whole 16-code words (group % 16 == 0 is checked)
    for (int w = 0; w < p.group / 16; ++w) {
      uint32_t word = 0;
      for (int e = 0; e < 16; ++e) word |= code(16 * w + e) << (16 * (e & 1) + 2 * (e >> 1));
      for (int bb = 0; bb < 4; ++bb) out[4 * w + bb] = (uint8_t)(word >> (8 * bb));
    }
    return;
  }
  const int per_byte = 8 / p.bits;
  for (int i0 = 0; i0 < p.group; i0 += per_byte) {
    uint32_t byte = 0;
    for (int j = 0; j < per_byte; ++j) byte |= code(i0 + j) << (j * p.bits);
    out[i0 / per_byte] = (uint8_t)byte;
  }
}

// One thread per (row, group): rnd(fl32(q * s) + z).
template <typename T>
__global__ void __launch_bounds__(256) kivi_dequantize_kernel(const QuantParams p) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= p.n_groups) return;
  const int gpr = p.D / p.group;
  const int g = (int)(gid % gpr);
  int64_t row = gid / gpr;
  const int t = (int)(row % p.T);
  row /= p.T;
  const int h = (int)(row % p.H);
  const int b = (int)(row / p.H);
  T* x = const_cast<T*>(reinterpret_cast<const T*>(p.x)) + b * p.x_sb + h * p.x_sh +
         (int64_t)t * p.x_st + g * p.group;
  const float s = Elem<T>::to_f32(
      *(reinterpret_cast<const T*>(p.scale) + b * p.s_sb + h * p.s_sh + (int64_t)t * p.s_st + g));
  const float z = Elem<T>::to_f32(
      *(reinterpret_cast<const T*>(p.zero) + b * p.s_sb + h * p.s_sh + (int64_t)t * p.s_st + g));
  const uint8_t* in = p.codes + b * p.c_sb + h * p.c_sh + (int64_t)t * p.c_st +
                      (int64_t)g * p.group * p.bits / 8;
  const int per_byte = 8 / p.bits;
  const uint32_t mask = (1u << p.bits) - 1;
  for (int i = 0; i < p.group; ++i) {
    const int e = i & 15;
    const uint32_t c =
        p.bits == 2 ? (in[4 * (i >> 4) + 2 * (e & 1) + (e >> 3)] >> (2 * ((e >> 1) & 3))) & 3u
                    : (in[i / per_byte] >> ((i % per_byte) * p.bits)) & mask;
    x[i] = Elem<T>::from_f32(__fadd_rn(__fmul_rn((float)c, s), z));
  }
}

}  // namespace halo

using namespace halo;

static int kivi_check(int32_t B, int32_t H, int32_t T, int32_t D, int32_t dtype, int32_t bits,
                      int32_t group) {
  if (B <= 0 || H <= 0 || T < 0 || D <= 0) return fail(HALO_ERR_INVALID_ARG, "bad KIVI shape");
  if (dtype != HALO_DTYPE_F16 && dtype != HALO_DTYPE_BF16)
    return fail(HALO_ERR_UNSUPPORTED, "KIVI needs fp16 or bf16 (dtype %d)", dtype);
  if (bits != 2 && bits != 4 && bits != 8)
    return fail(HALO_ERR_UNSUPPORTED, "KIVI bits must be 2, 4 or 8 (got %d)", bits);
  if (group <= 0 || D % group || (group * bits) % 8)
    return fail(HALO_ERR_INVALID_ARG, "group %d must divide D=%d and pack to bytes", group, D);
  if (bits == 2 && group % 16)
    return fail(HALO_ERR_UNSUPPORTED, "2-bit groups must be multiples of 16 (got %d)", group);
  return HALO_OK;
}

static int kivi_launch(bool quantize, const void* x, int64_t x_sb, int64_t x_sh, int64_t x_st,
                       int32_t B, int32_t H, int32_t T, int32_t D, int32_t dtype, int32_t bits,
                       int32_t group, void* codes, int64_t c_sb, int64_t c_sh, int64_t c_st,
                       void* scale, void* zero, int64_t s_sb, int64_t s_sh, int64_t s_st,
                       halo_stream_t stream) {
  int rc = kivi_check(B, H, T, D, dtype, bits, group);
  if (rc != HALO_OK) return rc;
  if (T == 0) return HALO_OK;
  if (!x || !codes || !scale || !zero) return fail(HALO_ERR_INVALID_ARG, "NULL pointer");
  QuantParams p{static_cast<const char*>(x), x_sb, x_sh, x_st, static_cast<uint8_t*>(codes),
                c_sb, c_sh, c_st, static_cast<char*>(scale), static_cast<char*>(zero),
                s_sb, s_sh, s_st, H, T, D, group, bits,
                (int64_t)B * H * T * (D / group)};
  const int64_t blocks = (p.n_groups + 255) / 256;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (quantize) {
    if (dtype == HALO_DTYPE_F16) kivi_quantize_kernel<__half><<<blocks, 256, 0, st>>>(p);
    else kivi_quantize_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(p);
  } else {
    if (dtype == HALO_DTYPE_F16) kivi_dequantize_kernel<__half><<<blocks, 256, 0, st>>>(p);
    else kivi_dequantize_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "KIVI kernel launch");
  count_launches();
  return HALO_OK;
}

extern "C" int32_t halo_kivi_quantize(const void* x, int64_t x_sb, int64_t x_sh, int64_t x_st,
                                      int32_t B, int32_t H, int32_t T, int32_t D, int32_t dtype,
                                      int32_t bits, int32_t group, uint8_t* codes, int64_t c_sb,
                                      int64_t c_sh, int64_t c_st, void* scale, void* zero,
                                      int64_t s_sb, int64_t s_sh, int64_t s_st,
                                      halo_stream_t stream) {
  return kivi_launch(true, x, x_sb, x_sh, x_st, B, H, T, D, dtype, bits, group, codes, c_sb,
                     c_sh, c_st, scale, zero, s_sb, s_sh, s_st, stream);
}

extern "C" int32_t halo_kivi_dequantize(const uint8_t* codes, int64_t c_sb, int64_t c_sh,
                                        int64_t c_st, const void* scale, const void* zero,
                                        int64_t s_sb, int64_t s_sh, int64_t s_st, int32_t B,
                                        int32_t H, int32_t T, int32_t D, int32_t dtype,
                                        int32_t bits, int32_t group, void* x, int64_t x_sb,
                                        int64_t x_sh, int64_t x_st, halo_stream_t stream) {
  return kivi_launch(false, x, x_sb, x_sh, x_st, B, H, T, D, dtype, bits, group,
                     const_cast<uint8_t*>(codes), c_sb, c_sh, c_st, const_cast<void*>(scale),
                     const_cast<void*>(zero), s_sb, s_sh, s_st, stream);
}
