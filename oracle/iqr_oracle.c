/* oracle/iqr_oracle.c -- TEST INFRASTRUCTURE: a plain-C restatement of the stored IQR decode.
 *
 * Each function names the reference lines it restates (reference src/iqr_decode.h). The
 * algorithm is libquant's grid_tcq_decode as the reference restates it (radiance pinned at
 * 451b136874084650992668bed9e8662deb58de88, un-vendored here); parity is pinned against the
 * reference's own r97_iqr_decode_host built from its sources in oracle/_ref.
 *
 * Not part of the product: only tests, the bench's CPU baseline and the smoke check call it.
 */
#include "iqr_oracle.h"

#include <math.h>
#include <string.h>

/* ---------------------------------------------------------------- scalar formats */

/* Nearest-even bf16 of an f32, NaN kept quiet (reference src/iqr_decode.h:118-124). */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE half to f32, subnormals included (reference src/iqr_decode.h:133-152). */
static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int32_t e = (h >> 10) & 0x1F;
    uint32_t m = h & 0x3FFu, u;
    if (e == 0) {
        if (m == 0) {
            u = sign;
        } else {
            /* value = m * 2^-24: normalise the mantissa */
            int32_t ex = 1 - 15;
            while (!(m & 0x400u)) {
                m <<= 1;
                --ex;
            }
            u = sign | ((uint32_t)(ex + 127) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        u = sign | 0x7F800000u | (m << 13);
    } else {
        u = sign | ((uint32_t)(e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* OCP FP8 E4M3 to f32: bias 7, no infinities, S.1111.111 the only NaN
 * (reference src/iqr_decode.h:156-180). */
static float e4m3_to_f32(uint8_t b) {
    const float sign = (b & 0x80u) ? -1.0f : 1.0f;
    const int e = (b >> 3) & 0xF;
    const int m = b & 0x7;
    if (e == 0xF && m == 0x7) return sign * NAN;
    if (e == 0) return sign * ldexpf((float)m, -9); /* m/8 * 2^-6 */
    return sign * ldexpf(1.0f + (float)m / 8.0f, e - 7);
}

static float load_scalar(const uint8_t* base, int32_t dtype, int64_t i) {
    switch (dtype) {
        case R97_IQR_F32: {
            float f;
            memcpy(&f, base + 4 * i, 4);
            return f;
        }
        case R97_IQR_BF16: {
            uint16_t b;
            memcpy(&b, base + 2 * i, 2);
            return bf16_to_f32(b);
        }
        case R97_IQR_F8E4M3: return e4m3_to_f32(base[i]);
        case R97_IQR_F16: {
            uint16_t h;
            memcpy(&h, base + 2 * i, 2);
            return f16_to_f32(h);
        }
        default: return 0.0f;
    }
}

/* Code `i` of a packed row, `bits` wide, lowest bits first (reference src/iqr_decode.h:194-203). */
static uint32_t load_bits(const uint8_t* row, int32_t bits, int64_t i) {
    const int64_t bit = i * (int64_t)bits;
    uint64_t w = 0;
    const int64_t first = bit >> 3;
    const int64_t last = (bit + bits - 1) >> 3;
    for (int64_t b = first; b <= last; ++b) w |= (uint64_t)row[b] << (8 * (b - first));
    return (uint32_t)((w >> (bit & 7)) & ((1ull << bits) - 1ull));
}

/* ---------------------------------------------------------------- one value */

/* The state's grid value: the mad hash's byte sum less 126, or the stored LUT
 * (reference src/iqr_decode.h:207-214). */
static int32_t state_value(const R97IqrDecodeDesc* d, uint32_t st) {
    if (d->mad) {
        uint32_t h = (st & 0xFFFFFFu) * (d->mad_a & 0xFFFFFFu) + d->mad_b;
        h &= 0x3F3F3F3Fu;
        return (int32_t)((h & 0xFF) + ((h >> 8) & 0xFF) + ((h >> 16) & 0xFF) + (h >> 24)) - 126;
    }
    return (int32_t)d->lut[st];
}

static int64_t block_cols(const R97IqrDecodeDesc* d) {
    return d->scale_block_cols > 0 ? d->scale_block_cols : d->cols;
}

/* The scale-plane group of 128-column block kb (reference src/iqr_decode.h:218-221). */
static int64_t scale_group(const R97IqrDecodeDesc* d, int64_t kb) {
    const int64_t bc = block_cols(d);
    return bc == d->cols ? 0 : (kb * 128) / bc;
}

/* Row r's first-level scale for block kb, times the second level settled to bf16
 * (reference src/iqr_decode.h:225-237). */
static float block_scale(const R97IqrDecodeDesc* d, int64_t r, int64_t kb) {
    const int64_t gb = scale_group(d, kb);
    float v = load_scalar(d->scale + (r - d->row0) * d->scale_row_bytes, d->scale_dtype, gb);
    if (d->scale2) {
        const int64_t i2 = d->scale2_block_rows > 0 ? r / d->scale2_block_rows : 0;
        const int64_t j2 = d->scale2_block_cols > 0 ? (gb * block_cols(d)) / d->scale2_block_cols : 0;
        const float s2 = load_scalar(d->scale2 + i2 * d->scale2_row_bytes, d->scale2_dtype, j2);
        v = bf16_to_f32(oracle_f32_to_bf16(v * s2));
    }
    return v;
}

/* The largest scale of row r's rb block, floored at zero (reference src/iqr_decode.h:241-252). */
static float block_max(const R97IqrDecodeDesc* d, int64_t r, int64_t kb) {
    const int64_t r0 = (r / d->rb) * d->rb;
    int64_t r1 = r0 + d->rb;
    if (r1 > d->rows_all) r1 = d->rows_all;
    float m = 0.0f;
    for (int64_t q = r0; q < r1; ++q) {
        const float v = block_scale(d, q, kb);
        if (v > m) m = v;
    }
    return m;
}

/* tcq_rb's re-rounding of a code onto the block's shared scale (reference src/iqr_decode.h:255-258):
 * the mad form rounds with the 1.5*2^23 magic number through one fused multiply-add. */
static int32_t rb_round(int32_t v, float ratio, int32_t round_mad) {
    if (round_mad) return (int32_t)(fmaf((float)v, ratio, 12582912.0f) - 12582912.0f);
    return (int32_t)rintf((float)v * ratio);
}

/* ---------------------------------------------------------------- the decode */

static void put(const R97IqrDecodeDesc* d, int64_t r, int64_t j, int32_t code, float scale) {
    d->out_codes[(r - d->row0) * d->cols + j] = (int8_t)code;
    if ((j & 127) == 0) d->out_scale[(r - d->row0) * (d->cols >> 7) + (j >> 7)] = oracle_f32_to_bf16(scale);
}

/* One run [r0, r1) of column j (reference src/iqr_decode.h:281-315). */
static void decode_run_column(const R97IqrDecodeDesc* d, int64_t r0, int64_t r1, int64_t j) {
    const int64_t kb = j >> 7;
    if (d->affine) {
        for (int64_t r = r0; r < r1; ++r) {
            const uint32_t code = load_bits(d->codes + (r - d->row0) * d->codes_row_bytes, d->bits, j);
            const uint32_t zero = load_bits(d->zero + (r - d->row0) * d->zero_row_bytes, d->zero_bits,
                                            scale_group(d, kb));
            put(d, r, j, (int32_t)code - (int32_t)zero, block_scale(d, r, kb));
        }
        return;
    }
    const int32_t c = (d->state_bits + d->bits - 1) / d->bits;
    const uint32_t mask = (uint32_t)((1ull << d->state_bits) - 1ull);
    uint32_t st = 0;
    /* tail-biting seam: the run's last c codes precede its first row */
    for (int32_t q = 0; q < c; ++q) {
        const int64_t t = r1 - c + q;
        st = ((st << d->bits) | load_bits(d->codes + (t - d->row0) * d->codes_row_bytes, d->bits, j)) & mask;
    }
    float cur = 0.0f;
    for (int64_t r = r0; r < r1; ++r) {
        st = ((st << d->bits) | load_bits(d->codes + (r - d->row0) * d->codes_row_bytes, d->bits, j)) & mask;
        const int32_t v = state_value(d, st);
        if (d->rb > 1) {
            if (r % d->rb == 0) cur = block_max(d, r, kb);
            const float sr = block_scale(d, r, kb);
            put(d, r, j, cur <= 0.0f ? 0 : rb_round(v, sr / cur, d->round_mad), cur);
        } else {
            put(d, r, j, v, block_scale(d, r, kb));
        }
    }
}

/* reference src/iqr_decode.h:321-362 */
int32_t oracle_iqr_validate(const R97IqrDecodeDesc* d) {
    if (!d->codes || !d->out_codes || !d->out_scale) return 1;
    if (d->rows <= 0 || d->row0 < 0 || d->rows_all <= 0 || d->rows > d->rows_all - d->row0) return 1;
    if (d->cols <= 0 || (d->cols & 127) != 0) return 1;
    if (d->run_rows <= 0 || d->rb <= 0 || d->run_rows % d->rb != 0) return 1;
    if (d->row0 % d->run_rows != 0) return 1;
    if (d->rows % d->run_rows != 0 && d->row0 + d->rows != d->rows_all) return 1;
    const int64_t bc = block_cols(d);
    if (bc != 128 && bc != d->cols) return 1;
    if (d->affine) {
        if (!d->zero || d->bits < 1 || d->bits > 7 || d->zero_bits < 1 || d->zero_bits > 8) return 1;
        if (d->run_rows != 1 || d->rb != 1 || d->scale2) return 1;
        return 0;
    }
    if (d->bits < 1 || d->bits > 16 || d->state_bits < 1 || d->state_bits > 24) return 1;
    if (!d->mad && !d->lut) return 1;
    if (d->scale2 && (d->scale2_block_rows < 0 || d->scale2_block_cols < 0)) return 1;
    if (d->scale2 && d->scale2_block_cols > 0 && d->scale2_block_cols % 128 != 0) return 1;
    const int32_t c = (d->state_bits + d->bits - 1) / d->bits;
    for (int64_t r0 = d->row0; r0 < d->row0 + d->rows; r0 += d->run_rows) {
        int64_t r1 = r0 + d->run_rows;
        if (r1 > d->rows_all) r1 = d->rows_all;
        if (r1 - r0 < c) return 1;
    }
    return 0;
}

int32_t oracle_iqr_decode(const R97IqrDecodeDesc* d) {
    if (oracle_iqr_validate(d)) return 1;
    for (int64_t r0 = d->row0; r0 < d->row0 + d->rows; r0 += d->run_rows) {
        int64_t r1 = r0 + d->run_rows;
        if (r1 > d->rows_all) r1 = d->rows_all;
        for (int64_t j = 0; j < d->cols; ++j) decode_run_column(d, r0, r1, j);
    }
    return 0;
}
