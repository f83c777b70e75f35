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

// ------------------------------------------------------------------------ the fused int8 producers
// rmsnorm_had_quant_i8g, gated_had_quant_i8g, gate_had_quant_i8g (reference src/adjoint/host/quant.cpp:821-1100,
// fused_twin / fused_adjoint): an elementwise part, then the rotated quantiser above over the part's f32 value,
// which is also stored as bf16 when the caller asks (the record's `out` write):
//   part 0  rmsnorm      v = x s (w + wadd) mult, s = 1 / sqrt(mean(x^2) + eps)  (elementwise.cpp:459-530)
//   part 1  silu_mul     v = silu(g) u, g and u the halves of one [rows, 2 n] row  (elementwise.cpp:278-293)
//   part 2  sigmoid mul  v = sigmoid(a) b                                          (act_mul, act "sigmoid")
// The adjoint recomputes v, takes the codes' cotangent straight through (masked where |v / s| > 127, over s,
// rotated back), adds the `out` write's cotangent, and then applies the part's adjoint:
//   rmsnorm  dx_j = mult (s c_j dv_j - (s^3 x_j / n) sum_i dv_i x_i c_i), c = w + wadd   (elementwise.cpp:531-541)
//   silu_mul dg = dv u silu'(g), du = dv silu(g);   sigmoid mul da = dv b sig'(a), db = dv sig(a)
// One CTA a row, a warp a 256-column chunk (8 columns a lane, the rotation's stages below 8 in-lane, the rest
// shuffles); the rmsnorm adjoint holds the row's dv in shared memory between its two passes.
struct FusedArgs {
    int part;
    const __nv_bfloat16* x;
    int64_t ldx;
    const __nv_bfloat16* x2;
    int64_t ldx2;
    const float* w;
    float eps, wadd, mult;
    int64_t n;
    int t, lt;
};

__device__ __forceinline__ float silu_of(float g) { return g / (1.0f + __expf(-g)); }
__device__ __forceinline__ float sig_of(float a) { return 1.0f / (1.0f + __expf(-a)); }

// The row's rmsnorm factor 1 / sqrt(mean(x^2) + eps), every thread of the block.
__device__ float row_rstd(const FusedArgs& a, int64_t r, float* red) {
    float ss = 0.0f;
    for (int64_t c = (int64_t)threadIdx.x * 8; c < a.n; c += 256 * 8) {
        float x[8];
        load_bf16<8>(a.x + r * a.ldx + c, x);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    __syncthreads();
    return 1.0f / sqrtf(tot / (float)a.n + a.eps);
}

// The part's inputs and value at columns c0 .. c0 + 7 of row r: p = x (part 0), the gate (1), a (2); u = the
// up half (1), b (2).
__device__ __forceinline__ void part_value(const FusedArgs& a, int64_t r, int64_t c0, float rstd, float (&p)[8],
                                           float (&u)[8], float (&v)[8]) {
    load_bf16<8>(a.x + r * a.ldx + c0, p);
    if (a.part == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = p[i] * rstd * (a.w ? a.w[c0 + i] + a.wadd : 1.0f) * a.mult;
    } else {
        load_bf16<8>(a.part == 1 ? a.x + r * a.ldx + a.n + c0 : a.x2 + r * a.ldx2 + c0, u);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (a.part == 1 ? silu_of(p[i]) : sig_of(p[i])) * u[i];
    }
}

__device__ __forceinline__ void load8f(const float* src, float (&d)[8]) {
    const float4 x = *reinterpret_cast<const float4*>(src), y = *reinterpret_cast<const float4*>(src + 4);
    d[0] = x.x, d[1] = x.y, d[2] = x.z, d[3] = x.w, d[4] = y.x, d[5] = y.y, d[6] = y.z, d[7] = y.w;
}
__device__ __forceinline__ void store8f(float* dst, const float (&v)[8], int accumulate) {
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = v[i];
    if (accumulate) {
        float prev[8];
        load8f(dst, prev);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] += prev[i];
    }
    *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(o[4], o[5], o[6], o[7]);
}

__global__ void __launch_bounds__(256) fused_quant_fwd_kernel(FusedArgs a, int8_t* __restrict__ codes, int64_t ldc,
                                                              float* __restrict__ scale, int64_t lds,
                                                              __nv_bfloat16* __restrict__ out, int64_t ldo) {
    __shared__ float red[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t r = blockIdx.x;
    const float rstd = a.part == 0 ? row_rstd(a, r, red) : 1.0f;
    for (int64_t ch = warp; ch * 256 < a.n; ch += 8) {  // whole warps: the rotation shuffles
        const int64_t c0 = ch * 256 + (int64_t)lane * 8;
        const bool on = c0 < a.n;  // n % 8 == 0: a lane is all in or out
        float p[8], u[8], v[8];
        if (on) {
            part_value(a, r, c0, rstd, p, u, v);
            if (out) {
                uint32_t w4[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
                    w4[k] = *reinterpret_cast<const uint32_t*>(&b2);
                }
                *reinterpret_cast<uint4*>(out + r * ldo + c0) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        }
        fwht_warp<8>(v, a.t, lane);
        float em[8];
        group_amax<8>(v, a.t, em);
        int q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float inv = 1.0f / scale_of_amax(em[i]);
            q[i] = __float2int_rn(fminf(fmaxf(v[i] * inv, -kTop), kTop));
        }
        if (!on) continue;
        store_codes<8>(codes + r * ldc + c0, q);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (((c0 + i) & (a.t - 1)) == 0) scale[r * lds + ((c0 + i) >> a.lt)] = scale_of_amax(em[i]);
    }
}

__global__ void __launch_bounds__(256) fused_quant_bwd_kernel(FusedArgs a, const float* __restrict__ scale,
                                                              int64_t lds, const float* __restrict__ g, int64_t ldg,
                                                              const float* __restrict__ go, int64_t ldgo,
                                                              float* __restrict__ dx, int64_t lddx,
                                                              float* __restrict__ dx2, int64_t lddx2, int accumulate) {
    extern __shared__ float dv_row[];  // part 0: the row's dv
    __shared__ float red[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t r = blockIdx.x;
    const float rstd = a.part == 0 ? row_rstd(a, r, red) : 1.0f;
    float dot = 0.0f;  // part 0: this thread's share of sum_i dv_i x_i c_i
    for (int64_t ch = warp; ch * 256 < a.n; ch += 8) {
        const int64_t c0 = ch * 256 + (int64_t)lane * 8;
        const bool on = c0 < a.n;
        float p[8], u[8], v[8], d[8];
        if (on) {
            part_value(a, r, c0, rstd, p, u, v);
            load8f(g + r * ldg + c0, d);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) p[i] = u[i] = v[i] = d[i] = 0.0f;
        }
        float vr[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) vr[i] = v[i];
        fwht_warp<8>(vr, a.t, lane);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float inv = on ? 1.0f / scale[r * lds + ((c0 + i) >> a.lt)] : 1.0f;
            d[i] = fabsf(vr[i] * inv) > kTop ? 0.0f : d[i] * inv;
        }
        fwht_warp<8>(d, a.t, lane);
        if (!on) continue;
        if (go) {
            float o[8];
            load8f(go + r * ldgo + c0, o);
#pragma unroll
            for (int i = 0; i < 8; ++i) d[i] += o[i];
        }
        if (a.part == 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                dv_row[c0 + i] = d[i];
                dot = fmaf(d[i] * p[i], a.w ? a.w[c0 + i] + a.wadd : 1.0f, dot);
            }
        } else if (a.part == 1) {
            float dg[8], du[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float s = sig_of(p[i]);
                dg[i] = d[i] * u[i] * (s * (1.0f + p[i] * (1.0f - s)));
                du[i] = d[i] * (p[i] * s);
            }
            store8f(dx + r * lddx + c0, dg, accumulate);
            store8f(dx + r * lddx + a.n + c0, du, accumulate);
        } else {
            float da[8], db[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float s = sig_of(p[i]);
                da[i] = d[i] * u[i] * (s * (1.0f - s));
                db[i] = d[i] * s;
            }
            store8f(dx + r * lddx + c0, da, accumulate);
            store8f(dx2 + r * lddx2 + c0, db, accumulate);
        }
    }
    if (a.part != 0) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xFFFFFFFFu, dot, o);
    if (lane == 0) red[warp] = dot;
    __syncthreads();  // also: the row's dv is complete
    float S = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) S += red[i];
    const float k2 = rstd * rstd * rstd / (float)a.n * S;
    for (int64_t c = (int64_t)threadIdx.x * 8; c < a.n; c += 256 * 8) {
        float x[8], o[8];
        load_bf16<8>(a.x + r * a.ldx + c, x);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float cg = a.w ? a.w[c + i] + a.wadd : 1.0f;
            o[i] = a.mult * (rstd * cg * dv_row[c + i] - k2 * x[i]);
        }
        store8f(dx + r * lddx + c, o, accumulate);
    }
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

namespace {

// The rules both fused entry points share; fills the geometry.
int fused_args(int32_t part, const uint16_t* x, int64_t ldx, const uint16_t* x2, int64_t ldx2, const float* w,
               float eps, float wadd, float mult, int64_t rows, int64_t n, int64_t group, FusedArgs* a) {
    if (part < 0 || part > 2 || !x || rows < 0 || n <= 0 || n % 8 || group <= 0 || group > 256 ||
        (group & (group - 1)) || n % group || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
        ldx < (part == 1 ? 2 * n : n) || rows > INT32_MAX)
        return R97B_EINVAL;
    if (part == 2 && (!x2 || ldx2 < n || ldx2 % 8 || (reinterpret_cast<uintptr_t>(x2) & 15))) return R97B_EINVAL;
    if (part == 0 && !w && wadd != 0.0f) return R97B_EINVAL;  // an offset without a gain (the twin refuses it)
    a->part = part, a->x = reinterpret_cast<const __nv_bfloat16*>(x), a->ldx = ldx;
    a->x2 = reinterpret_cast<const __nv_bfloat16*>(x2), a->ldx2 = ldx2;
    a->w = part == 0 ? w : nullptr, a->eps = eps, a->wadd = wadd, a->mult = mult;
    a->n = n, a->t = (int)group, a->lt = 0;
    while ((1 << (a->lt + 1)) <= group) ++a->lt;
    return R97B_OK;
}

bool al16(const void* p, int64_t ld) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && ld % 4 == 0; }

}  // namespace

extern "C" int r97b_fused_quant_i8g(int32_t part, const uint16_t* x, int64_t ldx, const uint16_t* x2, int64_t ldx2,
                                    const float* w, float eps, float wadd, float mult, int64_t rows, int64_t n,
                                    int64_t group, int8_t* codes, int64_t ldc, float* scale, int64_t lds,
                                    uint16_t* out, int64_t ldo, void* stream) {
    FusedArgs a{};
    if (fused_args(part, x, ldx, x2, ldx2, w, eps, wadd, mult, rows, n, group, &a) != R97B_OK) return R97B_EINVAL;
    if (!codes || !scale || ldc < n || ldc % 8 || (reinterpret_cast<uintptr_t>(codes) & 7) || lds < n / group)
        return R97B_EINVAL;
    if (out && (ldo < n || ldo % 8 || (reinterpret_cast<uintptr_t>(out) & 15))) return R97B_EINVAL;
    if (rows == 0) return R97B_OK;
    fused_quant_fwd_kernel<<<(unsigned)rows, 256, 0, as_stream(stream)>>>(
        a, codes, ldc, scale, lds, reinterpret_cast<__nv_bfloat16*>(out), ldo);
    return launch_status();
}

extern "C" int r97b_fused_quant_i8g_bwd(int32_t part, const uint16_t* x, int64_t ldx, const uint16_t* x2,
                                        int64_t ldx2, const float* w, float eps, float wadd, float mult, int64_t rows,
                                        int64_t n, int64_t group, const float* scale, int64_t lds, const float* g,
                                        int64_t ldg, const float* g_out, int64_t ldgo, float* dx, int64_t lddx,
                                        float* dx2, int64_t lddx2, int32_t accumulate, void* stream) {
    FusedArgs a{};
    if (fused_args(part, x, ldx, x2, ldx2, w, eps, wadd, mult, rows, n, group, &a) != R97B_OK) return R97B_EINVAL;
    if (!scale || lds < n / group || !g || ldg < n || !al16(g, ldg) || !dx || !al16(dx, lddx) ||
        lddx < (part == 1 ? 2 * n : n))
        return R97B_EINVAL;
    if (g_out && (ldgo < n || !al16(g_out, ldgo))) return R97B_EINVAL;
    if (part == 2 && (!dx2 || lddx2 < n || !al16(dx2, lddx2))) return R97B_EINVAL;
    const int smem = part == 0 ? (int)(n * 4) : 0;
    if (part == 0 && n > 16384) return R97B_EINVAL;
    if (rows == 0) return R97B_OK;
    if (smem > 48 * 1024 && !smem_opt_in(fused_quant_bwd_kernel, smem)) return R97B_ELAUNCH;
    fused_quant_bwd_kernel<<<(unsigned)rows, 256, smem, as_stream(stream)>>>(a, scale, lds, g, ldg, g_out, ldgo, dx,
                                                                             lddx, dx2, lddx2, accumulate ? 1 : 0);
    return launch_status();
}
