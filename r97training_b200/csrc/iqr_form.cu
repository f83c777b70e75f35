// iqr_form.cu -- a stored IQR weight's encoding, read as the decode's own description, and the device decode
// of a whole weight from its planes (the reference's src/iqr_form.h: r97_iqr_desc_from_planes,
// r97_iqr_decode_planes).
//
// The form is derived from the encoding's planes by role, as the reference derives it:
//   codes   packed unsigned codes (u1 .. u12), one a weight -> bits, codes_row_bytes
//   scale   f32 / bf16 / f16 / e4m3; block[1] = 0 one a row, else one a block[1] columns
//   trellis a table of 2^state_bits int8 states (extent[0]), run_rows = block[0], rb = block[1] (or 1)
//   zero    the affine grid instead of a trellis: an integer zero a scale block (1 .. 8 bits)
//   scale.1 a second scale level (not with the affine grid)
//   trellis.mad the computed codebook's A and B (two u32); it, or a scale.col plane, makes the codes round
//   scale.col one f32 a 128 columns that the description cannot carry: the decode folds it into the bf16
//           scale it writes, bf16(row scale x factor) with one rounding, and only for an f32 row scale
// Anything else -- a missing plane, a plane shorter than the weight needs, a state count that is not a power
// of two, a column count that is not a multiple of 128, zero and trellis together -- is refused.
//
// The encoding struct (include/r97b_iqr.h R97bEncoding) carries the fields of radiance's RadEncoding that the
// derivation reads (each plane's role, dtype, block and extent); radiance itself is not in this tree.
#include "r97b_internal.h"
#include "../../include/r97b_iqr.h"

#include <cuda_bf16.h>
#include <cstring>

namespace {

int code_bits(int32_t dt) { return dt >= R97B_ENC_U1 && dt <= R97B_ENC_U12 ? dt - R97B_ENC_U1 + 1 : 0; }

int dtype_bits(int32_t dt) {
    if (code_bits(dt)) return code_bits(dt);
    switch (dt) {
        case R97B_ENC_I8: case R97B_ENC_F8E4M3: return 8;
        case R97B_ENC_BF16: case R97B_ENC_F16: return 16;
        case R97B_ENC_F32: case R97B_ENC_U32: return 32;
        default: return 0;
    }
}

// Bytes of one row of n elements of dtype dt: packed bits, the row rounded up to a byte.
int64_t row_bytes(int32_t dt, int64_t n) { return (n * dtype_bits(dt) + 7) / 8; }

int32_t scale_type(int32_t dt) {
    switch (dt) {
        case R97B_ENC_F32: return R97_IQR_F32;
        case R97B_ENC_BF16: return R97_IQR_BF16;
        case R97B_ENC_F8E4M3: return R97_IQR_F8E4M3;
        case R97B_ENC_F16: return R97_IQR_F16;
        default: return -1;
    }
}

int32_t log2_exact(int64_t n) {
    int32_t l = 0;
    while (l < 62 && (int64_t(1) << l) < n) ++l;
    return (int64_t(1) << l) == n ? l : -1;
}

int plane_of(const R97bEncoding& e, const char* role) {
    for (int i = 0; i < e.n_planes && i < R97B_ENC_MAX_PLANES; ++i)
        if (std::strncmp(e.plane[i].role, role, sizeof e.plane[i].role) == 0) return i;
    return -1;
}

bool held(const R97bStoredPlane* p, int i, int64_t need) { return i >= 0 && p[i].data && p[i].bytes >= need; }

// bf16 bits of x, round to nearest even (the decode's own rounding of a scale).
__global__ void fold_scale_col_kernel(const float* __restrict__ row, const float* __restrict__ factor, int64_t rows,
                                      int64_t nkb, uint16_t* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nkb) return;
    const __nv_bfloat16 b = __float2bfloat16_rn(row[i / nkb] * factor[i % nkb]);
    out[i] = *reinterpret_cast<const uint16_t*>(&b);
}

}  // namespace

extern "C" int r97b_iqr_desc_from_planes(const R97bEncoding* enc, const R97bStoredPlane* plane, int64_t rows,
                                         int64_t cols, int32_t planes_on_device, R97IqrDecodeDesc* out) {
    if (!enc || !plane || !out || rows <= 0 || cols <= 0 || (cols & 127) || enc->n_planes < 0 ||
        enc->n_planes > R97B_ENC_MAX_PLANES)
        return 1;
    const R97bEncoding& e = *enc;
    const int64_t nkb = cols / 128;
    const int ic = plane_of(e, "codes"), is = plane_of(e, "scale"), it = plane_of(e, "trellis"),
              iz = plane_of(e, "zero");
    if (ic < 0 || is < 0 || (it < 0 && iz < 0)) return 1;
    R97IqrDecodeDesc d;
    std::memset(&d, 0, sizeof d);
    d.rows_all = rows, d.cols = cols, d.row0 = 0, d.rows = rows;
    d.bits = code_bits(e.plane[ic].dtype);
    if (d.bits <= 0) return 1;
    d.codes_row_bytes = row_bytes(e.plane[ic].dtype, cols);
    if (!held(plane, ic, rows * d.codes_row_bytes)) return 1;
    if (iz >= 0) {  // the affine grid: a zero a block beside the scale, no trellis, a row a run of its own
        if (it >= 0) return 1;
        d.zero_bits = dtype_bits(e.plane[iz].dtype);
        if (d.zero_bits < 1 || d.zero_bits > 8) return 1;
        if (e.plane[iz].block[0] != e.plane[is].block[0] || e.plane[iz].block[1] != e.plane[is].block[1]) return 1;
        d.affine = 1, d.run_rows = 1, d.rb = 1;
        d.zero_row_bytes = row_bytes(e.plane[iz].dtype, e.plane[iz].block[1] > 0 ? nkb : 1);
        if (!held(plane, iz, rows * d.zero_row_bytes)) return 1;
        d.zero = static_cast<const uint8_t*>(plane[iz].data);
    } else {
        d.state_bits = log2_exact(e.plane[it].extent[0]);
        if (d.state_bits < 1) return 1;
        d.run_rows = (int32_t)e.plane[it].block[0];
        d.rb = e.plane[it].block[1] > 0 ? (int32_t)e.plane[it].block[1] : 1;
        if (d.run_rows < 1 || d.rb < 1) return 1;
    }
    d.scale_dtype = scale_type(e.plane[is].dtype);
    if (d.scale_dtype < 0) return 1;
    d.scale_block_cols = e.plane[is].block[1];
    d.scale_row_bytes = row_bytes(e.plane[is].dtype, d.scale_block_cols > 0 ? nkb : 1);
    if (!held(plane, is, rows * d.scale_row_bytes)) return 1;
    const int is2 = plane_of(e, "scale.1");
    if (is2 >= 0) {
        if (iz >= 0) return 1;
        d.scale2_dtype = scale_type(e.plane[is2].dtype);
        if (d.scale2_dtype < 0) return 1;
        d.scale2_block_rows = e.plane[is2].block[0];
        d.scale2_block_cols = e.plane[is2].block[1];
        d.scale2_row_bytes = row_bytes(e.plane[is2].dtype, d.scale2_block_cols > 0 ? nkb : 1);
        const int64_t rows2 = d.scale2_block_rows > 0 ? (rows + d.scale2_block_rows - 1) / d.scale2_block_rows : 1;
        if (!held(plane, is2, rows2 * d.scale2_row_bytes)) return 1;
        d.scale2 = static_cast<const uint8_t*>(plane[is2].data);
    }
    const int im = plane_of(e, "trellis.mad");
    d.mad = im >= 0;
    d.round_mad = d.mad || plane_of(e, "scale.col") >= 0;
    if (it >= 0) {
        if (!held(plane, it, e.plane[it].extent[0])) return 1;
        d.lut = static_cast<const int8_t*>(plane[it].data);
        if (d.mad) {
            if (!held(plane, im, 8)) return 1;
            uint32_t ab[2];
            if (planes_on_device) {
                if (cudaMemcpy(ab, plane[im].data, sizeof ab, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
            } else {
                std::memcpy(ab, plane[im].data, sizeof ab);
            }
            d.mad_a = ab[0], d.mad_b = ab[1];
        }
    }
    d.codes = static_cast<const uint8_t*>(plane[ic].data);
    d.scale = static_cast<const uint8_t*>(plane[is].data);
    *out = d;
    return 0;
}

extern "C" int r97b_iqr_decode_planes(const R97bEncoding* enc, const R97bStoredPlane* plane, int64_t rows,
                                      int64_t cols, int8_t* out_codes, uint16_t* out_scale, void* stream) {
    R97IqrDecodeDesc d;
    if (!out_codes || !out_scale || r97b_iqr_desc_from_planes(enc, plane, rows, cols, 1, &d)) return 1;
    const int icf = plane_of(*enc, "scale.col");
    const int64_t nkb = cols / 128;
    if (icf >= 0) {  // the factor needs an f32 row scale to fold into; any other pairing has no form
        if (enc->plane[icf].dtype != R97B_ENC_F32 || !held(plane, icf, nkb * 4)) return 1;
        if (d.scale_dtype != R97_IQR_F32 || d.scale_block_cols > 0) return 1;
    }
    d.out_codes = out_codes;
    d.out_scale = out_scale;
    if (r97_iqr_decode(&d, stream) != 0) return 1;
    if (icf < 0) return 0;
    const int64_t n = rows * nkb;
    fold_scale_col_kernel<<<(unsigned)((n + 255) / 256), 256, 0, r97b::as_stream(stream)>>>(
        static_cast<const float*>(plane[plane_of(*enc, "scale")].data), static_cast<const float*>(plane[icf].data),
        rows, nkb, out_scale);
    return r97b::launch_status() == R97B_OK ? 0 : 1;
}
