/* oracle/iqr_oracle.h -- TEST INFRASTRUCTURE: the CPU restatement of the IQR decode.
 *
 * Used only by tests/, bench.py's cpu_baseline leg and __graft_entry__.smoke() as the checker of
 * the CUDA decode; the product never links it. Parity pin: tests/test_oracle_pin.py holds this
 * restatement bit-exact against the reference's own r97_iqr_decode_host compiled from the
 * reference tree (oracle/_ref), over every stored form that function accepts.
 */
#ifndef R97B_IQR_ORACLE_H
#define R97B_IQR_ORACLE_H

#include "../include/r97b_iqr.h"

#ifdef __cplusplus
extern "C" {
#endif

/* 0 when the description is decodable, 1 otherwise (reference src/iqr_decode.h:321-362). */
int32_t oracle_iqr_validate(const R97IqrDecodeDesc* d);

/* Decodes rows [row0, row0+rows) into out_codes / out_scale (reference src/iqr_decode.h:291-315,
 * 366-376). Returns the validate result. */
int32_t oracle_iqr_decode(const R97IqrDecodeDesc* d);

/* The f32 -> bf16 rounding the decode settles scales with (nearest-even, quiet NaN). */
uint16_t oracle_f32_to_bf16(float f);

#ifdef __cplusplus
}
#endif

#endif
