/*
 * CPU oracle: KIVI per-group quantise / dequantise in plain C.
 * TEST INFRASTRUCTURE ONLY -- never linked into the shipped library.
 *
 * Restates baselines/kivi_cache.py:44-78 (lzbaclz/HALO) with explicit
 * per-op rounding: every torch op on an fp16 / bf16 tensor rounds its
 * result once to that type, so each step is an IEEE float32 operation
 * followed by one round-to-nearest-even into the 16-bit storage type.
 * float32 keeps >= 2p+2 bits for both 16-bit formats, so that double
 * rounding equals a single correct rounding of the exact result.
 *
 * Layout: rows of D contiguous elements (raw 16-bit patterns); D is split
 * into D/group groups.  Outputs: codes int8 [rows][D], scale/zero 16-bit
 * [rows][D/group].
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* IEEE binary16 -> float (exact). */
static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    if (exp == 0) {                       /* zero / subnormal: mant * 2^-24 */
        float v = ldexpf((float)mant, -24);
        return sign ? -v : v;
    }
    if (exp == 31) return bits_to_f32(sign | 0x7F800000u | (mant << 13));
    return bits_to_f32(sign | ((exp - 15 + 127) << 23) | (mant << 13));
}

/* float -> IEEE binary16, round to nearest even. */
static uint16_t f32_to_f16_rn(float f) {
    uint32_t u = f32_to_bits(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return sign | 0x7E00u;          /* NaN */
    if (a >= 0x477FF000u) return sign | 0x7C00u;         /* >= 65520 -> inf */
    if (a < 0x38800000u) {                               /* below 2^-14 */
        uint32_t e = a >> 23;
        if (a == 0 || e < 102) return sign;              /* < 2^-25: to zero */
        uint32_t mant = (a & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126 - e;                        /* units of 2^-24 */
        uint32_t r = mant >> shift, rem = mant & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return sign | (uint16_t)r;
    }
    uint32_t r = (((a >> 23) - 127 + 15) << 10) | ((a & 0x7FFFFFu) >> 13);
    uint32_t rem = a & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return sign | (uint16_t)r;
}

static float bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

static uint16_t f32_to_bf16_rn(float f) {
    uint32_t u = f32_to_bits(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

typedef float (*to_f32_fn)(uint16_t);
typedef uint16_t (*from_f32_fn)(float);

static void quantize_rows(const uint16_t *x, int64_t rows, int D, int group, int bits,
                          int8_t *codes, uint16_t *scale, uint16_t *zero,
                          to_f32_fn to32, from_f32_fn from32) {
    const float qmax = (float)((1 << bits) - 1);
    const float eps = to32(from32(1e-8f));  /* clamp_min scalar cast to dtype */
    const int ng = D / group;
    for (int64_t r = 0; r < rows; ++r) {
        for (int g = 0; g < ng; ++g) {
            const uint16_t *xg = x + r * D + (int64_t)g * group;
            float mn = to32(xg[0]), mx = mn;
            for (int i = 1; i < group; ++i) {
                float v = to32(xg[i]);
                mn = v < mn ? v : mn;
                mx = v > mx ? v : mx;
            }
            float d = to32(from32(mx - mn));
            if (d < eps) d = eps;
            uint16_t s_bits = from32(d / qmax);
            float s = to32(s_bits);
            scale[r * ng + g] = s_bits;
            zero[r * ng + g] = from32(mn);
            for (int i = 0; i < group; ++i) {
                float t = to32(from32(to32(xg[i]) - mn));
                float u = to32(from32(t / s));
                float q = rintf(u);
                int8_t c;
                if (isnan(q)) c = 0;
                else c = (int8_t)(q < 0.f ? 0.f : (q > qmax ? qmax : q));
                codes[r * D + (int64_t)g * group + i] = c;
            }
        }
    }
}

static void dequantize_rows(const int8_t *codes, const uint16_t *scale, const uint16_t *zero,
                            int64_t rows, int D, int group, uint16_t *out,
                            to_f32_fn to32, from_f32_fn from32) {
    const int ng = D / group;
    for (int64_t r = 0; r < rows; ++r)
        for (int i = 0; i < D; ++i) {
            float s = to32(scale[r * ng + i / group]), z = to32(zero[r * ng + i / group]);
            volatile float prod = (float)codes[r * D + i] * s;   /* no FMA contraction */
            out[r * D + i] = from32(prod + z);
        }
}

/* dtype: 0 = fp16, 1 = bf16 */
void oracle_kivi_quantize(const uint16_t *x, int64_t rows, int D, int group, int bits,
                          int dtype, int8_t *codes, uint16_t *scale, uint16_t *zero) {
    if (dtype == 0)
        quantize_rows(x, rows, D, group, bits, codes, scale, zero, f16_to_f32, f32_to_f16_rn);
    else
        quantize_rows(x, rows, D, group, bits, codes, scale, zero, bf16_to_f32, f32_to_bf16_rn);
}

void oracle_kivi_dequantize(const int8_t *codes, const uint16_t *scale, const uint16_t *zero,
                            int64_t rows, int D, int group, int dtype, uint16_t *out) {
    if (dtype == 0)
        dequantize_rows(codes, scale, zero, rows, D, group, out, f16_to_f32, f32_to_f16_rn);
    else
        dequantize_rows(codes, scale, zero, rows, D, group, out, bf16_to_f32, f32_to_bf16_rn);
}
