// iqr.cu -- the stored IQR weight decode on sm_100a.
//
// Two kernels:
//   * iqr_decode_general: every form the reference's r97_iqr_validate accepts (any code width up to 16
//     bits, computed or stored codebook, f32/bf16/e4m3/f16 scales, a second scale level, tcq_rb row
//     blocks, the affine grid). One thread walks one column of one trellis run, the reference's own
//     unit of work (reference src/iqr_decode.h:281-315).
//   * iqr_decode_u4: the trunk form the configs store (4-bit codes, 16 state bits, computed "mad"
//     codebook, one f32/bf16 scale per row and 128 columns, rb = 1). A thread owns 8 adjacent columns
//     (one 32-bit word of codes a row) over an 8-row segment of a run; the state a segment enters with
//     comes from the 3 codes above it, or from the run's tail-biting seam for the run's first rows, so
//     segments decode independently. It writes either the reference's int8 grid + bf16 scale, or the
//     bf16 product code * scale the GEMM reads.
//
// Both produce the reference's values bit for bit (checked against the CPU oracle in tests/).
#include "r97b_internal.h"
#include "sm100.cuh"

#include <cuda_bf16.h>

namespace r97b {

namespace {

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// Nearest-even f32 -> bf16 bits with NaN kept quiet, the rounding the decode settles scales with.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

__device__ float f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int32_t e = (h >> 10) & 0x1F;
    uint32_t m = h & 0x3FFu, u;
    if (e == 0) {
        if (m == 0) {
            u = sign;
        } else {
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
    return __uint_as_float(u);
}

__device__ float e4m3_bits_to_f32(uint8_t b) {
    const uint32_t s = (uint32_t)(b >> 7) << 31;
    const int e = (b >> 3) & 0xF;
    const int m = b & 0x7;
    if (e == 0xF && m == 0x7) return __uint_as_float(s | 0x7FC00000u);
    if (e == 0) return (s ? -1.0f : 1.0f) * ldexpf((float)m, -9);
    return (s ? -1.0f : 1.0f) * ldexpf(1.0f + (float)m * 0.125f, e - 7);
}

__device__ float load_scalar(const uint8_t* base, int32_t dtype, int64_t i) {
    switch (dtype) {
        case R97_IQR_F32: return reinterpret_cast<const float*>(base)[i];
        case R97_IQR_BF16: return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(base)[i]);
        case R97_IQR_F8E4M3: return e4m3_bits_to_f32(base[i]);
        case R97_IQR_F16: return f16_bits_to_f32(reinterpret_cast<const uint16_t*>(base)[i]);
        default: return 0.0f;
    }
}

__device__ __forceinline__ uint32_t load_bits(const uint8_t* row, int32_t bits, int64_t i) {
    const int64_t bit = i * (int64_t)bits;
    const int64_t first = bit >> 3;
    const int64_t last = (bit + bits - 1) >> 3;
    uint64_t w = 0;
    for (int64_t b = first; b <= last; ++b) w |= (uint64_t)row[b] << (8 * (b - first));
    return (uint32_t)((w >> (bit & 7)) & ((1ull << bits) - 1ull));
}

__device__ __forceinline__ int32_t mad_value(uint32_t st, uint32_t a, uint32_t b) {
    const uint32_t h = ((st & 0xFFFFFFu) * (a & 0xFFFFFFu) + b) & 0x3F3F3F3Fu;
    return (int32_t)__dp4a(h, 0x01010101u, 0u) - 126;
}

__device__ __forceinline__ int64_t block_cols(const R97IqrDecodeDesc& d) {
    return d.scale_block_cols > 0 ? d.scale_block_cols : d.cols;
}

__device__ __forceinline__ int64_t scale_group(const R97IqrDecodeDesc& d, int64_t kb) {
    const int64_t bc = block_cols(d);
    return bc == d.cols ? 0 : (kb * 128) / bc;
}

__device__ float block_scale(const R97IqrDecodeDesc& d, int64_t r, int64_t kb) {
    const int64_t gb = scale_group(d, kb);
    float v = load_scalar(d.scale + (r - d.row0) * d.scale_row_bytes, d.scale_dtype, gb);
    if (d.scale2) {
        const int64_t i2 = d.scale2_block_rows > 0 ? r / d.scale2_block_rows : 0;
        const int64_t j2 = d.scale2_block_cols > 0 ? (gb * block_cols(d)) / d.scale2_block_cols : 0;
        const float s2 = load_scalar(d.scale2 + i2 * d.scale2_row_bytes, d.scale2_dtype, j2);
        v = bf16_bits_to_f32(f32_to_bf16_bits(v * s2));
    }
    return v;
}

__device__ float block_max(const R97IqrDecodeDesc& d, int64_t r, int64_t kb) {
    const int64_t r0 = (r / d.rb) * d.rb;
    int64_t r1 = r0 + d.rb;
    if (r1 > d.rows_all) r1 = d.rows_all;
    float m = 0.0f;
    for (int64_t q = r0; q < r1; ++q) {
        const float v = block_scale(d, q, kb);
        m = v > m ? v : m;
    }
    return m;
}

__device__ __forceinline__ int32_t rb_round(int32_t v, float ratio, int32_t round_mad) {
    if (round_mad) return (int32_t)(__fmaf_rn((float)v, ratio, 12582912.0f) - 12582912.0f);
    return (int32_t)rintf((float)v * ratio);
}

// Output sinks: the reference's int8 grid + bf16 scale, or the bf16 GEMM operand.
struct Sink {
    int8_t* codes;
    uint16_t* scale;
    uint16_t* w;
    int64_t ld_w;
};

__device__ __forceinline__ void emit(const R97IqrDecodeDesc& d, const Sink& s, int64_t r, int64_t j, int32_t code,
                                     float sc) {
    const int64_t lr = r - d.row0;
    if (s.w) {
        const float sb = bf16_bits_to_f32(f32_to_bf16_bits(sc));
        s.w[lr * s.ld_w + j] = f32_to_bf16_bits((float)code * sb);
        return;
    }
    s.codes[lr * d.cols + j] = (int8_t)code;
    if ((j & 127) == 0) s.scale[lr * (d.cols >> 7) + (j >> 7)] = f32_to_bf16_bits(sc);
}

__global__ void iqr_decode_general(const R97IqrDecodeDesc d, const Sink s) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= d.cols) return;
    for (int64_t run = blockIdx.y; run * d.run_rows < d.rows; run += gridDim.y) {
        const int64_t r0 = d.row0 + run * d.run_rows;
        int64_t r1 = r0 + d.run_rows;
        if (r1 > d.rows_all) r1 = d.rows_all;
        const int64_t kb = j >> 7;
        if (d.affine) {
            for (int64_t r = r0; r < r1; ++r) {
                const uint32_t code = load_bits(d.codes + (r - d.row0) * d.codes_row_bytes, d.bits, j);
                const uint32_t zero =
                    load_bits(d.zero + (r - d.row0) * d.zero_row_bytes, d.zero_bits, scale_group(d, kb));
                emit(d, s, r, j, (int32_t)code - (int32_t)zero, block_scale(d, r, kb));
            }
            continue;
        }
        const int32_t c = (d.state_bits + d.bits - 1) / d.bits;
        const uint32_t mask = (uint32_t)((1ull << d.state_bits) - 1ull);
        uint32_t st = 0;
        for (int32_t q = 0; q < c; ++q) {
            const int64_t t = r1 - c + q;
            st = ((st << d.bits) | load_bits(d.codes + (t - d.row0) * d.codes_row_bytes, d.bits, j)) & mask;
        }
        float cur = 0.0f;
        for (int64_t r = r0; r < r1; ++r) {
            st = ((st << d.bits) | load_bits(d.codes + (r - d.row0) * d.codes_row_bytes, d.bits, j)) & mask;
            const int32_t v = d.mad ? mad_value(st, d.mad_a, d.mad_b) : (int32_t)d.lut[st];
            if (d.rb > 1) {
                if (r % d.rb == 0) cur = block_max(d, r, kb);
                const float sr = block_scale(d, r, kb);
                emit(d, s, r, j, cur <= 0.0f ? 0 : rb_round(v, sr / cur, d.round_mad), cur);
            } else {
                emit(d, s, r, j, v, block_scale(d, r, kb));
            }
        }
    }
}

constexpr int kSegRows = 8;

// The trunk form: u4 codes, 16 state bits, mad codebook, per-(row, 128 col) f32/bf16 scale, rb = 1.
// A thread requests every code word and scale of its segment (and the 3 words above it) before the first
// row's arithmetic: 19 loads in flight per thread (8 words, 8 scales, 3 halo words), 4 CTAs of 256 threads per
// SM (measured 4-5 % faster than 16-row segments at 3 CTAs an SM).
template <bool kBf16Out>
__global__ void __launch_bounds__(256, 4) iqr_decode_u4(const R97IqrDecodeDesc d, const Sink s, int64_t nseg_per_run) {
    const int64_t groups = d.cols >> 3;  // 8-column groups
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nruns = (d.rows + d.run_rows - 1) / d.run_rows;
    const int64_t total = groups * nruns * nseg_per_run;
    if (gid >= total) return;
    int64_t g, seg, run;
    if (total <= 0xFFFFFFFFll) {  // 32-bit splits: a 64-bit division is a long subroutine
        const uint32_t ng = (uint32_t)groups, ns = (uint32_t)nseg_per_run;
        const uint32_t q = (uint32_t)gid / ng, q2 = q / ns;
        g = (uint32_t)gid - q * ng;
        seg = q - q2 * ns;
        run = q2;
    } else {
        g = gid % groups;
        seg = (gid / groups) % nseg_per_run;
        run = gid / (groups * nseg_per_run);
    }
    const int64_t r0 = d.row0 + run * d.run_rows;
    int64_t r1 = r0 + d.run_rows;
    if (r1 > d.rows_all) r1 = d.rows_all;
    const int64_t len = r1 - r0;
    const int64_t sr0 = r0 + seg * kSegRows;
    if (sr0 >= r1) return;
    const int64_t sr1 = sr0 + kSegRows < r1 ? sr0 + kSegRows : r1;
    const int64_t j0 = g * 8;
    const uint8_t* cbase = d.codes + j0 / 2;
    auto word = [&](int64_t r) -> uint32_t {
        return *reinterpret_cast<const uint32_t*>(cbase + (r - d.row0) * d.codes_row_bytes);
    };
    const int64_t kb = j0 >> 7;
    const int nrow = (int)(sr1 - sr0);
    // the 3 words above the segment's first row, wrapping to the run's tail (the seam)
    uint32_t halo[3];
#pragma unroll
    for (int q = 3; q >= 1; --q) {
        int64_t t = sr0 - q;
        if (t < r0) t += len;
        halo[3 - q] = word(t);
    }
    uint32_t wb[kSegRows];
    float sb[kSegRows];
    {
        const uint8_t* cp = cbase + (sr0 - d.row0) * d.codes_row_bytes;
        const int crb = (int)d.codes_row_bytes, srb = (int)d.scale_row_bytes;
        const bool f32s = d.scale_dtype == R97_IQR_F32;
        const uint8_t* sp = d.scale + (sr0 - d.row0) * d.scale_row_bytes + kb * (f32s ? 4 : 2);
#pragma unroll
        for (int b = 0; b < kSegRows; ++b) {
            const int rb = b < nrow ? b : nrow - 1;
            wb[b] = *reinterpret_cast<const uint32_t*>(cp + rb * crb);
            sb[b] = f32s ? *reinterpret_cast<const float*>(sp + rb * srb)
                         : bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sp + rb * srb));
        }
    }
    // A column's 16-bit state at row r is its nibbles of rows r-3 .. r. They are formed from "pair bytes":
    // for rows (a, b), E holds (a's nibble << 4 | b's nibble) of the even columns (byte j: column 2j) and O
    // of the odd ones (byte j: column 2j + 1); the state of column 2j is then E(r-3, r-2).byte_j << 8 |
    // E(r-1, r).byte_j -- one byte permute yields two columns' states, so a row's eight states take four
    // permutes and eight half-extractions instead of a shift / mask / merge chain per column.
    auto pair_e = [](uint32_t a, uint32_t b) { return ((a << 4) & 0xF0F0F0F0u) | (b & 0x0F0F0F0Fu); };
    auto pair_o = [](uint32_t a, uint32_t b) { return (a & 0xF0F0F0F0u) | ((b >> 4) & 0x0F0F0F0Fu); };
    uint32_t e2 = pair_e(halo[0], halo[1]), o2 = pair_o(halo[0], halo[1]);  // rows (r-3, r-2)
    uint32_t e1 = pair_e(halo[1], halo[2]), o1 = pair_o(halo[1], halo[2]);  // rows (r-2, r-1)
    uint32_t prev = halo[2];
    const uint32_t A = d.mad_a & 0xFFFFFFu, B = d.mad_b;
    uint16_t* wrow = kBf16Out ? s.w + (sr0 - d.row0) * s.ld_w + j0 : nullptr;
#pragma unroll
    for (int b = 0; b < kSegRows; ++b) {
        if (b >= nrow) break;
        const uint32_t w = wb[b];
        const int64_t lr = sr0 + b - d.row0;
        const uint32_t e0 = pair_e(prev, w), o0 = pair_o(prev, w);  // rows (r-1, r)
        const uint32_t pe01 = __byte_perm(e0, e2, 0x5140u), pe23 = __byte_perm(e0, e2, 0x7362u);
        const uint32_t po01 = __byte_perm(o0, o2, 0x5140u), po23 = __byte_perm(o0, o2, 0x7362u);
        const uint32_t st[8] = {pe01 & 0xFFFFu, po01 & 0xFFFFu, pe01 >> 16, po01 >> 16,
                                pe23 & 0xFFFFu, po23 & 0xFFFFu, pe23 >> 16, po23 >> 16};
        e2 = e1;
        o2 = o1;
        e1 = e0;
        o1 = o0;
        prev = w;
        if (kBf16Out) {
            // value = (byte sum of the hash) - 126, formed exactly as a float: the dot product's
            // accumulator starts at 2^23's bit pattern, so the sum lands in the mantissa
            const float sc = bf16_bits_to_f32(f32_to_bf16_bits(sb[b]));
            float vf[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t h = (st[i] * A + B) & 0x3F3F3F3Fu;
                vf[i] = __uint_as_float(__dp4a(h, 0x01010101u, 0x4B000000u)) - 8388734.0f;
            }
            // code * scale rounded to nearest-even bf16 by the hardware conversion (finite and infinite
            // products round exactly as f32_to_bf16_bits does)
            uint32_t pk[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __nv_bfloat162 p2 = __floats2bfloat162_rn(vf[2 * i] * sc, vf[2 * i + 1] * sc);
                pk[i] = *reinterpret_cast<const uint32_t*>(&p2);
            }
            *reinterpret_cast<uint4*>(wrow) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            wrow += s.ld_w;
        } else {
            int32_t v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = mad_value(st[i], A, B);
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                lo |= ((uint32_t)(uint8_t)(int8_t)v[i]) << (8 * i);
                hi |= ((uint32_t)(uint8_t)(int8_t)v[4 + i]) << (8 * i);
            }
            *reinterpret_cast<uint2*>(s.codes + lr * d.cols + j0) = make_uint2(lo, hi);
            if ((j0 & 127) == 0) s.scale[lr * (d.cols >> 7) + kb] = f32_to_bf16_bits(sb[b]);
        }
    }
}

// Host-side mirror of the reference's r97_iqr_validate (reference src/iqr_decode.h:321-362): it reads
// only the description's fields, never the planes.
int validate(const R97IqrDecodeDesc& d, bool need_outputs) {
    if (!d.codes) return 1;
    if (need_outputs && (!d.out_codes || !d.out_scale)) return 1;
    if (d.rows <= 0 || d.row0 < 0 || d.rows_all <= 0 || d.rows > d.rows_all - d.row0) return 1;
    if (d.cols <= 0 || (d.cols & 127) != 0) return 1;
    if (d.run_rows <= 0 || d.rb <= 0 || d.run_rows % d.rb != 0) return 1;
    if (d.row0 % d.run_rows != 0) return 1;
    if (d.rows % d.run_rows != 0 && d.row0 + d.rows != d.rows_all) return 1;
    const int64_t bc = d.scale_block_cols > 0 ? d.scale_block_cols : d.cols;
    if (bc != 128 && bc != d.cols) return 1;
    if (d.affine) {
        if (!d.zero || d.bits < 1 || d.bits > 7 || d.zero_bits < 1 || d.zero_bits > 8) return 1;
        if (d.run_rows != 1 || d.rb != 1 || d.scale2) return 1;
        return 0;
    }
    if (d.bits < 1 || d.bits > 16 || d.state_bits < 1 || d.state_bits > 24) return 1;
    if (!d.mad && !d.lut) return 1;
    if (d.scale2 && (d.scale2_block_rows < 0 || d.scale2_block_cols < 0)) return 1;
    if (d.scale2 && d.scale2_block_cols > 0 && d.scale2_block_cols % 128 != 0) return 1;
    const int32_t c = (d.state_bits + d.bits - 1) / d.bits;
    for (int64_t r0 = d.row0; r0 < d.row0 + d.rows; r0 += d.run_rows) {
        int64_t r1 = r0 + d.run_rows;
        if (r1 > d.rows_all) r1 = d.rows_all;
        if (r1 - r0 < c) return 1;
    }
    return 0;
}

bool is_trunk_form(const R97IqrDecodeDesc& d) {
    return !d.affine && d.bits == 4 && d.state_bits == 16 && d.mad && d.rb == 1 && !d.scale2 &&
           (d.scale_dtype == R97_IQR_F32 || d.scale_dtype == R97_IQR_BF16) &&
           (d.scale_block_cols == 128 || (d.scale_block_cols <= 0 && d.cols == 128)) &&
           (reinterpret_cast<uintptr_t>(d.codes) & 3) == 0 && (d.codes_row_bytes & 3) == 0 &&
           d.run_rows >= 4;
}

int run_decode(const R97IqrDecodeDesc& d, const Sink& s, cudaStream_t stream) {
    if (is_trunk_form(d)) {
        const bool bf16 = s.w != nullptr;
        if (bf16 && ((reinterpret_cast<uintptr_t>(s.w) & 15) != 0 || (s.ld_w & 7) != 0)) goto general;
        if (!bf16 && ((reinterpret_cast<uintptr_t>(s.codes) & 7) != 0)) goto general;
        {
            const int64_t nseg = (d.run_rows + kSegRows - 1) / kSegRows;
            const int64_t nruns = (d.rows + d.run_rows - 1) / d.run_rows;
            const int64_t total = (d.cols >> 3) * nruns * nseg;
            const int threads = 256;
            const int64_t blocks = (total + threads - 1) / threads;
            if (bf16)
                iqr_decode_u4<true><<<(unsigned)blocks, threads, 0, stream>>>(d, s, nseg);
            else
                iqr_decode_u4<false><<<(unsigned)blocks, threads, 0, stream>>>(d, s, nseg);
            return launch_status();
        }
    }
general : {
    const int64_t nruns = (d.rows + d.run_rows - 1) / d.run_rows;
    dim3 grid((unsigned)((d.cols + 127) / 128), (unsigned)(nruns < 65535 ? nruns : 65535));
    iqr_decode_general<<<grid, 128, 0, stream>>>(d, s);
    return launch_status();
}
}

}  // namespace

}  // namespace r97b


namespace r97b {
namespace {
// W[r, k] = bf16(code[r, k] * scale[r, k / group]): the stored (codes, scale) pair of a decoded weight as
// the GEMM operand, with the same product and rounding the fused decode uses. 8 columns a thread.
__global__ void codes_dequant_kernel(const int8_t* __restrict__ codes, const uint16_t* __restrict__ scale,
                                     int64_t rows, int64_t cols, int64_t group, int64_t groups,
                                     uint16_t* __restrict__ out, int64_t ld) {
    const int64_t per_row = (cols + 7) / 8;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= rows * per_row) return;
    const int64_t r = t / per_row, c0 = (t % per_row) * 8;
    for (int64_t c = c0; c < c0 + 8 && c < cols; ++c) {
        const float sb = bf16_bits_to_f32(scale[r * groups + c / group]);
        out[r * ld + c] = f32_to_bf16_bits((float)codes[r * cols + c] * sb);
    }
}
}  // namespace
}  // namespace r97b

extern "C" int r97b_codes_dequant_bf16(const int8_t* codes, const uint16_t* scale, int64_t rows, int64_t cols,
                                       int64_t group, uint16_t* out_w, int64_t ld_w, void* stream) {
    if (!codes || !scale || !out_w || rows <= 0 || cols <= 0 || group <= 0 || ld_w < cols) return R97B_EINVAL;
    const int64_t groups = (cols + group - 1) / group;
    const int64_t threads = rows * ((cols + 7) / 8);
    if (threads / 256 + 1 > 0x7FFFFFFF) return R97B_EINVAL;
    r97b::codes_dequant_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, r97b::as_stream(stream)>>>(
        codes, scale, rows, cols, group, groups, out_w, ld_w);
    return r97b::launch_status();
}

extern "C" int r97_iqr_decode(const R97IqrDecodeDesc* desc, R97IqrStream stream) {
    if (!desc || r97b::validate(*desc, true)) return 1;
    r97b::Sink s{desc->out_codes, desc->out_scale, nullptr, 0};
    return r97b::run_decode(*desc, s, reinterpret_cast<cudaStream_t>(stream)) == R97B_OK ? 0 : 1;
}

extern "C" int r97b_iqr_dequant_bf16(const R97IqrDecodeDesc* desc, uint16_t* out_w, int64_t ld_w, void* stream) {
    if (!desc || !out_w || ld_w < desc->cols || r97b::validate(*desc, false)) return R97B_EINVAL;
    r97b::Sink s{nullptr, nullptr, out_w, ld_w};
    return r97b::run_decode(*desc, s, r97b::as_stream(stream));
}
