// quant.cu -- the int8 activation quantisers of the w8a8 trunk and their straight-through adjoints.
//
// quant_act_i8g / had_quant_act_i8g (reference src/adjoint/host/quant.cpp:43-370; docs/adjoints/quant.md
// s1, s3): per row and group of t columns, v = the group (for the rotated op: W x, W the unnormalised
// Walsh-Hadamard matrix of order t, W W = t I), s = amax|v| / 127 (1 for a zero group), codes =
// rint(clamp(v / s, +-127)) (nearest even), one f32 scale per group. The adjoint takes the codes'
// cotangent g straight through the rounding, zero where the clamp engaged (|v / s| > 127), divides by the
// scale (g (1 / s), one reciprocal a group) and rotates back: dx = W (m . g / s) (W^T = W); the scale's
// cotangent is dropped.
//
// The rotated op is HBM-bound elementwise work. A warp owns 32 E consecutive columns of a row, a lane E of
// them, so the transform's stages below E are in-lane butterflies and the rest are shuffles (lane ^ h / E);
// E = 4 serves every group up to 128 with 8-byte bf16 loads, E = 8 groups of 256. The stages run in
// ascending h with the lower index's sum first, the order the reference's fwht loop uses, in f32; the
// reciprocal is taken once a group (inv = 1 / s, u = v inv), as the reference's kernel does.
#include "r97b_internal.h"

#include <cuda_bf16.h>
#include <stdint.h>

namespace r97b {
namespace {

constexpr float kTop = 127.0f;

// E bf16 of a row into f32 (E = 4: one 8-byte load; E = 8: one 16-byte load).
template <int E>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* p, float (&v)[E]) {
    uint32_t w[E / 2];
    if constexpr (E == 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        w[0] = u.x, w[1] = u.y;
    } else {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        w[0] = u.x, w[1] = u.y, w[2] = u.z, w[3] = u.w;
    }
#pragma unroll
    for (int k = 0; k < E / 2; ++k) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
        v[2 * k] = f.x, v[2 * k + 1] = f.y;
    }
}

// E int8 codes to one 4- or 8-byte store.
template <int E>
__device__ __forceinline__ void store_codes(int8_t* p, const int (&q)[E]) {
    uint32_t w[E / 4];
#pragma unroll
    for (int k = 0; k < E / 4; ++k)
        w[k] = (uint32_t)(q[4 * k] & 0xFF) | ((uint32_t)(q[4 * k + 1] & 0xFF) << 8) |
               ((uint32_t)(q[4 * k + 2] & 0xFF) << 16) | ((uint32_t)(q[4 * k + 3] & 0xFF) << 24);
    if constexpr (E == 4) *reinterpret_cast<uint32_t*>(p) = w[0];
    else *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
}

// The unnormalised transform of every t-wide group of the warp's 32 E columns (t <= 32 E, a power of two).
template <int E>
__device__ __forceinline__ void fwht_warp(float (&v)[E], int t, int lane) {
#pragma unroll
    for (int h = 1; h < E; h <<= 1) {
        if (h >= t) break;
#pragma unroll
        for (int i = 0; i < E; ++i)
            if (!(i & h)) {
                const float a = v[i], b = v[i + h];
                v[i] = a + b;
                v[i + h] = a - b;
            }
    }
    for (int x = 1; x * E < t; x <<= 1) {  // stage h = x E: the partner is lane ^ x
        const float sgn = (lane & x) ? -1.0f : 1.0f;  // the upper index keeps (lower - upper) = -v + o
#pragma unroll
        for (int i = 0; i < E; ++i) v[i] = fmaf(sgn, v[i], __shfl_xor_sync(0xFFFFFFFFu, v[i], x));
    }
}

// em[i] = the max of |v| over element i's t-wide group (lanes of one group end with the same values).
template <int E>
__device__ __forceinline__ void group_amax(const float (&v)[E], int t, float (&em)[E]) {
    if (t >= E) {
        float m = 0.0f;
#pragma unroll
        for (int i = 0; i < E; ++i) m = fmaxf(m, fabsf(v[i]));
        for (int x = 1; x * E < t; x <<= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, x));
#pragma unroll
        for (int i = 0; i < E; ++i) em[i] = m;
        return;
    }
#pragma unroll
    for (int i = 0; i < E; ++i) em[i] = fabsf(v[i]);
#pragma unroll
    for (int h = 1; h < E; h <<= 1) {
        if (h >= t) break;
        float o[E];
#pragma unroll
        for (int i = 0; i < E; ++i) o[i] = fmaxf(em[i], em[i ^ h]);
#pragma unroll
        for (int i = 0; i < E; ++i) em[i] = o[i];
    }
}

// s = a / 127, one correctly rounded division (then inv = 1 / s and u = v inv: at the amax u is
// a (1 / (a / 127)), one rounding either side of 127, the arithmetic docs/adjoints/quant.md s1 describes).
__device__ __forceinline__ float scale_of_amax(float amax) { return amax > 0.0f ? amax / kTop : 1.0f; }

struct QuantArgs {
    const __nv_bfloat16* x;
    int64_t ldx, rows, n;
    int t;        // group width (a power of two for the rotated kernel)
    int lt;       // log2(t) when t is a power of two
    int rotate;
    int64_t ngrp;
};

// Forward, rotated or power-of-two plain groups. Grid (rows, ceil(chunks / (8 U))): a warp takes U chunks
// of 32 E columns of its row, all their loads issued before the first transform.
template <int E, int U>
__global__ void __launch_bounds__(256) quant_fwd_kernel(QuantArgs a, int8_t* __restrict__ codes, int64_t ldc,
                                                         float* __restrict__ scale) {
    const int lane = threadIdx.x & 31;
    const int64_t r = blockIdx.x;
    const int64_t chunk0 = ((int64_t)blockIdx.y * 8 + (threadIdx.x >> 5)) * U;
    if (chunk0 * 32 * E >= a.n) return;  // whole warps
    float v[U][E];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t c0 = (chunk0 + u) * 32 * E + (int64_t)lane * E;
        if (c0 < a.n) load_bf16<E>(a.x + r * a.ldx + c0, v[u]);  // n % E == 0: a lane is all in or out
        else
#pragma unroll
            for (int i = 0; i < E; ++i) v[u][i] = 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t c0 = (chunk0 + u) * 32 * E + (int64_t)lane * E;
        if (a.rotate) fwht_warp<E>(v[u], a.t, lane);
        float em[E];
        group_amax<E>(v[u], a.t, em);
        int q[E];
        if (a.t >= E) {  // one group across the lane: one scale, one reciprocal
            const float inv = 1.0f / scale_of_amax(em[0]);
#pragma unroll
            for (int i = 0; i < E; ++i) q[i] = __float2int_rn(fminf(fmaxf(v[u][i] * inv, -kTop), kTop));
        } else {
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const float inv = 1.0f / scale_of_amax(em[i]);
                q[i] = __float2int_rn(fminf(fmaxf(v[u][i] * inv, -kTop), kTop));
            }
        }
        if (c0 >= a.n) continue;
        store_codes<E>(codes + r * ldc + c0, q);
#pragma unroll
        for (int i = 0; i < E; ++i)  // the first column of each group writes its scale
            if (((c0 + i) & (a.t - 1)) == 0) scale[r * a.ngrp + ((c0 + i) >> a.lt)] = scale_of_amax(em[i]);
    }
}

// Adjoint, same layout: dx = W (m . g / s).
template <int E, int U>
__global__ void __launch_bounds__(256) quant_bwd_kernel(QuantArgs a, const float* __restrict__ scale,
                                                         const float* __restrict__ g, int64_t ldg, float* __restrict__ dx,
                                                         int64_t lddx, int accumulate) {
    const int lane = threadIdx.x & 31;
    const int64_t r = blockIdx.x;
    const int64_t chunk0 = ((int64_t)blockIdx.y * 8 + (threadIdx.x >> 5)) * U;
    if (chunk0 * 32 * E >= a.n) return;
    float v[U][E], d[U][E];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t c0 = (chunk0 + u) * 32 * E + (int64_t)lane * E;
        if (c0 < a.n) {
            load_bf16<E>(a.x + r * a.ldx + c0, v[u]);
#pragma unroll
            for (int i = 0; i < E; i += 4) {
                const float4 f = *reinterpret_cast<const float4*>(g + r * ldg + c0 + i);
                d[u][i] = f.x, d[u][i + 1] = f.y, d[u][i + 2] = f.z, d[u][i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < E; ++i) v[u][i] = d[u][i] = 0.0f;
        }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int64_t c0 = (chunk0 + u) * 32 * E + (int64_t)lane * E;
        const bool on = c0 < a.n;
        if (a.rotate) fwht_warp<E>(v[u], a.t, lane);
        if (a.t >= E) {
            const float inv = on ? 1.0f / scale[r * a.ngrp + (c0 >> a.lt)] : 1.0f;
#pragma unroll
            for (int i = 0; i < E; ++i) d[u][i] = fabsf(v[u][i] * inv) > kTop ? 0.0f : d[u][i] * inv;
        } else {
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const float inv = on ? 1.0f / scale[r * a.ngrp + ((c0 + i) >> a.lt)] : 1.0f;
                d[u][i] = fabsf(v[u][i] * inv) > kTop ? 0.0f : d[u][i] * inv;
            }
        }
        if (a.rotate) fwht_warp<E>(d[u], a.t, lane);
        if (!on) continue;
#pragma unroll
        for (int i = 0; i < E; i += 4) {
            float4* p = reinterpret_cast<float4*>(dx + r * lddx + c0 + i);
            float4 o = make_float4(d[u][i], d[u][i + 1], d[u][i + 2], d[u][i + 3]);
            if (accumulate) {
                const float4 prev = *p;
                o.x += prev.x, o.y += prev.y, o.z += prev.z, o.w += prev.w;
            }
            *p = o;
        }
    }
}

// The plain op with any group width (a short last group when it does not divide n): a warp a group.
__global__ void __launch_bounds__(256) quant_plain_fwd_kernel(QuantArgs a, int8_t* __restrict__ codes, int64_t ldc,
                                                               float* __restrict__ scale) {
    const int lane = threadIdx.x & 31;
    const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (wid >= a.rows * a.ngrp) return;
    const int64_t r = wid / a.ngrp, k0 = (wid % a.ngrp) * a.t;
    const int64_t w = min((int64_t)a.t, a.n - k0);
    const __nv_bfloat16* xr = a.x + r * a.ldx + k0;
    float m = 0.0f;
    for (int64_t i = lane; i < w; i += 32) m = fmaxf(m, fabsf(__bfloat162float(xr[i])));
#pragma unroll
    for (int x = 16; x > 0; x >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, x));
    const float s = scale_of_amax(m), inv = 1.0f / s;
    for (int64_t i = lane; i < w; i += 32)
        codes[r * ldc + k0 + i] = (int8_t)__float2int_rn(fminf(fmaxf(__bfloat162float(xr[i]) * inv, -kTop), kTop));
    if (lane == 0) scale[r * a.ngrp + k0 / a.t] = s;
}

__global__ void __launch_bounds__(256) quant_plain_bwd_kernel(QuantArgs a, const float* __restrict__ scale,
                                                               const float* __restrict__ g, int64_t ldg,
                                                               float* __restrict__ dx, int64_t lddx, int accumulate) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.rows * a.n) return;
    const int64_t r = i / a.n, c = i % a.n;
    const float s = scale[r * a.ngrp + c / a.t], inv = 1.0f / s;
    const float v = __bfloat162float(a.x[r * a.ldx + c]);
    float d = fabsf(v * inv) > kTop ? 0.0f : g[r * ldg + c] / s;
    if (accumulate) d += dx[r * lddx + c];
    dx[r * lddx + c] = d;
}

// y[r, c] = x[r, c] s[r, c / group], f32 in, f32 or bf16 out (y may be x for f32): the group scales of the
// int8 trunk's products applied to a float operand or result.
__global__ void __launch_bounds__(256) group_scale_kernel(const float* __restrict__ x, int64_t ldx, int64_t rows,
                                                          int64_t cols, int64_t group, const float* __restrict__ s,
                                                          int64_t lds, void* y, int64_t ldy, int y_bf16) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * cols) return;
    const int64_t r = i / cols, c = i % cols;
    const float v = x[r * ldx + c] * s[r * lds + c / group];
    if (y_bf16) reinterpret_cast<__nv_bfloat16*>(y)[r * ldy + c] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(y)[r * ldy + c] = v;
}

unsigned blocks_of_warps(int64_t warps) { return (unsigned)((warps * 32 + 255) / 256); }

// One block a row and 8 chunks of `cols` columns.
dim3 chunk_grid(int64_t rows, int64_t n, int cols) {
    return dim3((unsigned)rows, (unsigned)(((n + cols - 1) / cols + 7) / 8));
}

// The shared argument rules; fills the geometry. 0 when the call is valid.
int quant_args(const uint16_t* x, int64_t ldx, int64_t rows, int64_t n, int64_t group, int32_t rotate, QuantArgs* a) {
    if (!x || rows < 0 || n <= 0 || ldx < n) return R97B_EINVAL;
    a->x = reinterpret_cast<const __nv_bfloat16*>(x);
    a->ldx = ldx, a->rows = rows, a->n = n, a->rotate = rotate ? 1 : 0;
    if (rotate) {
        if (group <= 0 || group > 1024 || (group & (group - 1)) || n % group) return R97B_EINVAL;
    } else if (group <= 0 || group > n) {
        group = n;
    }
    a->t = (int)group;
    a->lt = 0;
    while ((1ll << (a->lt + 1)) <= group) ++a->lt;
    a->ngrp = (n + group - 1) / group;
    return R97B_OK;
}

// Which warp layout serves the call (power-of-two groups up to 256 that divide n): E = 8 columns a lane when
// n and the x rows allow 16-byte loads, else E = 4 (groups up to 128); 0 when neither (the plain op then
// takes its general kernel).
int lanes_cols(const QuantArgs& a) {
    if ((a.t & (a.t - 1)) || a.n % a.t || a.n % 4 || a.t > 256) return 0;
    const uintptr_t xp = reinterpret_cast<uintptr_t>(a.x);
    if (a.n % 8 == 0 && a.ldx % 8 == 0 && (xp & 15) == 0) return 8;
    if (a.t <= 128 && a.ldx % 4 == 0 && (xp & 7) == 0) return 4;
    return 0;
}

// The E = 4 layout's own rule (8-byte x rows), for a call whose codes / g / dx rows do not allow E = 8.
bool lanes_cols4(const QuantArgs& a) {
    return a.ldx % 4 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 7) == 0;
}

bool aligned(const void* p, int64_t ld, int elems, int bytes) {
    return (reinterpret_cast<uintptr_t>(p) & (uintptr_t)(bytes - 1)) == 0 && ld % elems == 0;
}

}  // namespace
}  // namespace r97b

using namespace r97b;

extern "C" int r97b_quant_act_i8g(const uint16_t* x, int64_t ldx, int64_t rows, int64_t n, int64_t group,
                                  int32_t rotate, int8_t* codes, int64_t ldc, float* scale, void* stream) {
    QuantArgs a{};
    if (quant_args(x, ldx, rows, n, group, rotate, &a) != R97B_OK || !codes || !scale || ldc < n) return R97B_EINVAL;
    if (rows == 0) return R97B_OK;
    if (rows > INT32_MAX || (n + 255) / 256 / 8 >= 65535) return R97B_EINVAL;
    const cudaStream_t s = as_stream(stream);
    const int e = lanes_cols(a);
    if (e == 8 && aligned(codes, ldc, 8, 8)) {
        quant_fwd_kernel<8, 2><<<chunk_grid(rows, n, 256 * 2), 256, 0, s>>>(a, codes, ldc, scale);
    } else if (e && a.t <= 128 && lanes_cols4(a) && aligned(codes, ldc, 4, 4)) {
        quant_fwd_kernel<4, 2><<<chunk_grid(rows, n, 128 * 2), 256, 0, s>>>(a, codes, ldc, scale);
    } else if (!rotate) {
        quant_plain_fwd_kernel<<<blocks_of_warps(rows * a.ngrp), 256, 0, s>>>(a, codes, ldc, scale);
    } else {
        return R97B_EINVAL;  // a rotation wider than 256 columns, or rows off the 4 / 8-column alignment
    }
    return launch_status();
}

extern "C" int r97b_quant_act_i8g_bwd(const uint16_t* x, int64_t ldx, int64_t rows, int64_t n, int64_t group,
                                      int32_t rotate, const float* scale, const float* g, int64_t ldg, float* dx,
                                      int64_t lddx, int32_t accumulate, void* stream) {
    QuantArgs a{};
    if (quant_args(x, ldx, rows, n, group, rotate, &a) != R97B_OK || !scale || !g || !dx || ldg < n || lddx < n)
        return R97B_EINVAL;
    if (rows == 0) return R97B_OK;
    if (rows > INT32_MAX || (n + 255) / 256 / 8 >= 65535) return R97B_EINVAL;
    const cudaStream_t s = as_stream(stream);
    const int e = lanes_cols(a);
    const bool vec = aligned(g, ldg, 4, 16) && aligned(dx, lddx, 4, 16);
    if (e == 8 && vec) {
        quant_bwd_kernel<8, 2><<<chunk_grid(rows, n, 256 * 2), 256, 0, s>>>(a, scale, g, ldg, dx, lddx, accumulate);
    } else if (e && a.t <= 128 && lanes_cols4(a) && vec) {
        quant_bwd_kernel<4, 2><<<chunk_grid(rows, n, 128 * 2), 256, 0, s>>>(a, scale, g, ldg, dx, lddx, accumulate);
    } else if (!rotate) {
        quant_plain_bwd_kernel<<<(unsigned)((rows * n + 255) / 256), 256, 0, s>>>(a, scale, g, ldg, dx, lddx,
                                                                                  accumulate);
    } else {
        return R97B_EINVAL;
    }
    return launch_status();
}

extern "C" int r97b_group_scale(const float* x, int64_t ldx, int64_t rows, int64_t cols, int64_t group, const float* s,
                                int64_t lds, void* y, int64_t ldy, int32_t y_bf16, void* stream) {
    if (!x || !s || !y || rows < 0 || cols < 0 || group <= 0 || ldx < cols || ldy < cols ||
        lds < (cols + group - 1) / group)
        return R97B_EINVAL;
    if (rows == 0 || cols == 0) return R97B_OK;
    const int64_t blocks = (rows * cols + 255) / 256;
    if (blocks > INT32_MAX) return R97B_EINVAL;
    group_scale_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(x, ldx, rows, cols, group, s, lds, y, ldy,
                                                                        y_bf16 ? 1 : 0);
    return launch_status();
}
