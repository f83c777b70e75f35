/* oracle/shim/rad_plugin.h -- TEST INFRASTRUCTURE, used only to compile the checker (oracle/_ref).
 *
 * A stand-in for radiance's rad_plugin.h, which the reference tree does not vendor: it declares just the
 * helpers the reference's quant family (src/adjoint/host/quant.cpp) calls, so that file compiles into the
 * checker beside the other host rows. Each is written here from the format it converts:
 *   bf16  the top 16 bits of an f32, rounded to nearest even (NaN kept quiet);
 *   E4M3  OCP FP8 E4M3FN (sign, 4 exponent bits of bias 7, 3 mantissa bits, no infinities, 448 the
 *         largest finite), rounded to nearest even and saturated at +-448, NaN to 0x7F.
 * The int8 quantisers this repository pins its kernels to use only the bf16 pair; the E4M3 pair serves the
 * family's fp8 rows, which are not a parity anchor here. */
#ifndef R97_ORACLE_SHIM_RAD_PLUGIN_H
#define R97_ORACLE_SHIM_RAD_PLUGIN_H

#include <math.h>
#include <stdint.h>
#include <string.h>

typedef enum RadDtype {
    RAD_DTYPE_NONE = 0,
    RAD_DTYPE_I8,
    RAD_DTYPE_U8,
    RAD_DTYPE_FP8,
    RAD_DTYPE_BF16,
    RAD_DTYPE_F16,
    RAD_DTYPE_I32,
    RAD_DTYPE_F32,
    RAD_DTYPE_F64,
} RadDtype;

static inline RadDtype rad_dtype_parse(const char* s) {
    if (!s) return RAD_DTYPE_NONE;
    if (!strcmp(s, "i8") || !strcmp(s, "int8")) return RAD_DTYPE_I8;
    if (!strcmp(s, "u8") || !strcmp(s, "uint8")) return RAD_DTYPE_U8;
    if (!strcmp(s, "fp8") || !strcmp(s, "e4m3") || !strcmp(s, "fp8e4m3")) return RAD_DTYPE_FP8;
    if (!strcmp(s, "bf16")) return RAD_DTYPE_BF16;
    if (!strcmp(s, "f16") || !strcmp(s, "fp16")) return RAD_DTYPE_F16;
    if (!strcmp(s, "i32") || !strcmp(s, "int32")) return RAD_DTYPE_I32;
    if (!strcmp(s, "f32") || !strcmp(s, "fp32")) return RAD_DTYPE_F32;
    if (!strcmp(s, "f64") || !strcmp(s, "fp64")) return RAD_DTYPE_F64;
    return RAD_DTYPE_NONE;
}

static inline int rad_dtype_bits(RadDtype d) {
    switch (d) {
    case RAD_DTYPE_I8: case RAD_DTYPE_U8: case RAD_DTYPE_FP8: return 8;
    case RAD_DTYPE_BF16: case RAD_DTYPE_F16: return 16;
    case RAD_DTYPE_I32: case RAD_DTYPE_F32: return 32;
    case RAD_DTYPE_F64: return 64;
    default: return 0;
    }
}

static inline uint16_t rad_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float rad_bf16_to_f32(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint8_t rad_f32_to_fp8e4m3(float f) {
    if (isnan(f)) return 0x7F;
    const uint8_t sign = signbit(f) ? 0x80 : 0x00;
    float a = fabsf(f);
    if (a >= 448.0f) return (uint8_t)(sign | 0x7E);
    /* the grid spacing at a: 2^(e - 3) for a normal of exponent e >= -6, 2^-9 below (subnormals) */
    int e;
    frexpf(a, &e);  /* a = m 2^e, m in [0.5, 1): the leading bit is 2^(e - 1) */
    int lead = e - 1;
    if (lead < -6) lead = -6;
    const float step = ldexpf(1.0f, lead - 3);
    float q = nearbyintf(a / step) * step; /* a / step is exact (a power-of-two divide); ties to even */
    if (q >= 448.0f) return (uint8_t)(sign | 0x7E);
    if (q == 0.0f) return sign;
    int qe;
    frexpf(q, &qe);
    const int ql = qe - 1;
    if (ql < -6) return (uint8_t)(sign | (uint8_t)(q / ldexpf(1.0f, -9))); /* subnormal: mantissa count */
    const int mant = (int)(q / ldexpf(1.0f, ql - 3)) - 8;
    return (uint8_t)(sign | (uint8_t)((ql + 7) << 3) | (uint8_t)mant);
}

static inline float rad_fp8e4m3_to_f32(uint8_t b) {
    const float sign = (b & 0x80) ? -1.0f : 1.0f;
    const int ex = (b >> 3) & 0xF, mant = b & 7;
    if (ex == 0xF && mant == 7) return NAN;
    if (ex == 0) return sign * ldexpf((float)mant, -9);
    return sign * ldexpf((float)(8 + mant), ex - 10);
}

#endif
