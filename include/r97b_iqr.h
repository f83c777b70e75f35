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

#ifdef __cplusplus
}
#endif

#endif /* R97B_IQR_H */
