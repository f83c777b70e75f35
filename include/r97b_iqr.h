/* include/r97b_iqr.h -- the stored IQR weight description shared by the B200 decode kernels, the
 * C-ABI entry point r97_iqr_decode and the CPU oracle.
 *
 * The struct keeps the field order, meaning and units of the reference's R97IqrDecodeDesc
 * (reference src/iqr_decode.h:59-114) so that a caller built against the reference passes the same
 * bytes: it is an interface, not an implementation, and has to be alike. Plain C, no CUDA types.
 *
 * A weight is N = rows_all output rows by K = cols input columns (K a multiple of 128), stored as
 * `bits`-wide codes packed along each row, lowest bits first. Down each column the codes drive a
 * tail-biting trellis: the state at row r is the last ceil(state_bits/bits) codes of that column
 * (rows r-c+1..r), masked to state_bits; a run of run_rows rows seeds its first state from its own
 * last codes. The state's value is an int8 grid point (a computed "mad" hash or a stored LUT) and
 * the block scale (one per row and 128 columns) multiplies it. The decode writes the int8 grid
 * [rows, cols] and the scale as bf16 bits [rows, cols/128].
 */
#ifndef R97B_IQR_H
#define R97B_IQR_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum R97IqrScaleType {
    R97_IQR_F32 = 0,
    R97_IQR_BF16 = 1,
    R97_IQR_F8E4M3 = 2,
    R97_IQR_F16 = 3,
};

typedef struct R97IqrDecodeDesc {
    int64_t rows_all;
    int64_t cols;
    int64_t row0;
    int64_t rows;

    int32_t bits;
    int32_t state_bits;
    int32_t run_rows;
    int32_t rb;

    int32_t mad;
    int32_t round_mad;
    uint32_t mad_a;
    uint32_t mad_b;
    const int8_t* lut;

    const uint8_t* codes;
    int64_t codes_row_bytes;

    const uint8_t* scale;
    int32_t scale_dtype;
    int64_t scale_block_cols;
    int64_t scale_row_bytes;

    int32_t affine;
    const uint8_t* zero;
    int32_t zero_bits;
    int64_t zero_row_bytes;

    const uint8_t* scale2;
    int32_t scale2_dtype;
    int64_t scale2_row_bytes;
    int64_t scale2_block_rows;
    int64_t scale2_block_cols;

    int8_t* out_codes;
    uint16_t* out_scale;
} R97IqrDecodeDesc;

typedef void* R97IqrStream;

/* ---- a stored weight's encoding, read as the description above (reference src/iqr_form.h) ----
 * The fields of a container encoding (radiance's RadEncoding; not in this tree) that the derivation reads:
 * each plane's role ("codes", "scale", "trellis", "trellis.mad", "zero", "scale.1", "scale.col"), its
 * element type, its block (block[0] rows, block[1] columns an element; 0 = the whole extent) and, for a
 * table, its extent (extent[0] entries). */
enum R97bEncDtype {
    R97B_ENC_U1 = 1, /* .. R97B_ENC_U12 = 12: packed unsigned codes of that many bits */
    R97B_ENC_U12 = 12,
    R97B_ENC_I8 = 20,
    R97B_ENC_U32 = 21,
    R97B_ENC_F32 = 30,
    R97B_ENC_BF16 = 31,
    R97B_ENC_F16 = 32,
    R97B_ENC_F8E4M3 = 33,
};
#define R97B_ENC_MAX_PLANES 8
typedef struct R97bEncPlane {
    char role[24];
    int32_t dtype;
    int64_t block[2];
    int64_t extent[2];
} R97bEncPlane;
typedef struct R97bEncoding {
    int32_t n_planes;
    R97bEncPlane plane[R97B_ENC_MAX_PLANES];
} R97bEncoding;
/* One encoding plane's bytes as stored (rows of packed elements, each row rounded up to a byte); a plane the
 * caller does not hold is {null, 0}. */
typedef struct R97bStoredPlane {
    const void* data;
    int64_t bytes;
} R97bStoredPlane;

/* The description of the whole weight [rows, cols] from an encoding's planes (plane[i] = encoding plane i):
 * the form is derived from the planes by role (codes -> bits; a trellis table -> state_bits = log2(extent),
 * run_rows, rb; a zero plane -> the affine grid; scale / scale.1 layouts; trellis.mad -> the computed
 * codebook; trellis.mad or scale.col -> rounded codes). 0, or 1 when the encoding is not a form the decode
 * reads or a plane it needs is missing or short. planes_on_device: the planes are device memory (the
 * computed codebook's A and B are then read with one blocking copy, so the planes must already be written,
 * not pending on another stream). The output pointers are left to the caller.
 * Replaces: reference src/iqr_form.h:87-175 r97_iqr_desc_from_planes. */
int r97b_iqr_desc_from_planes(const R97bEncoding* enc, const R97bStoredPlane* plane, int64_t rows, int64_t cols,
                              int32_t planes_on_device, R97IqrDecodeDesc* out);
/* The whole weight decoded on the device from device planes: out_codes int8 [rows, cols], out_scale bf16 bits
 * [rows, cols / 128], with a scale.col plane's factor folded into the scale as bf16(row f32 x factor), one
 * rounding (it is refused beside any scale but an f32 one a row). 0, or 1 as above.
 * Replaces: reference src/iqr_form.h:189-217 r97_iqr_decode_planes (host), on the device. */
int r97b_iqr_decode_planes(const R97bEncoding* enc, const R97bStoredPlane* plane, int64_t rows, int64_t cols,
                           int8_t* out_codes, uint16_t* out_scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* R97B_IQR_H */
