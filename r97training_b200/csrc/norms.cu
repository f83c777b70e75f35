// norms.cu -- RMSNorm and gated RMSNorm, forward and backward, on sm_100a.
//
// HBM-bound row kernels: a row is split over a group of lanes (a whole warp for wide rows, half a
// warp for the 128-wide head rows of the gated norm), each lane moving 16-byte vectors, and the
// row's sums are warp-shuffle reductions. All arithmetic is f32; inputs and outputs are bf16.
//
//   rmsnorm:       y = x * rsqrt(mean(x^2) + eps) * (w + wadd) * mult
//                  dx = mult * (s c dy - s^3 x / n * sum(dy x c)),  c = w + wadd
//                  (reference src/adjoint/host/elementwise.cpp:459-670)
//   gated rmsnorm: o = x * rsqrt(mean(x^2) + eps) * w * act(z),  act = silu (or sigmoid)
//                  dx = w g sc do - x sc^3 / n * sum(x w g do),  dz = do x sc w g'
//                  (reference src/adjoint/host/gdn_prep.cpp:501-592)
#include "r97b_internal.h"
#include "fastmath.cuh"

#include <cuda_bf16.h>

namespace r97b {
namespace {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ void loadw8(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

template <int W>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return sigmoid_ftz(x); }

// One row per group of W lanes; VPL = 8-element vectors per lane, runtime loop over the row.
template <int W>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                          int64_t rows, int n, float eps, float wadd, float mult) {
    const int lane = threadIdx.x & (W - 1);
    const int64_t grow = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / W;
    // lanes past the last row still join the shuffles, on a clamped row, and store nothing
    const bool valid = grow < rows;
    const int64_t row = valid ? grow : rows - 1;
    const __nv_bfloat16* xr = x + row * n;
    float ss = 0.0f;
    for (int c = lane * 8; c < n; c += W * 8) {
        float v[8];
        load8(xr + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
    }
    ss = group_sum<W>(ss);
    const float s = rsqrtf(ss / (float)n + eps);
    if (rstd && lane == 0 && valid) rstd[row] = s;
    for (int c = lane * 8; c < n; c += W * 8) {
        float v[8], g[8];
        load8(xr + c, v);
        if (w) loadw8(w + c, g);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = v[i] * s * (w ? g[i] + wadd : 1.0f) * mult;
        if (valid) store8(y + row * n + c, v);
    }
}

template <int W>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                                          const __nv_bfloat16* __restrict__ dy,
                                                          const __nv_bfloat16* __restrict__ addend,
                                                          __nv_bfloat16* __restrict__ dx, int64_t rows, int n, float eps,
                                                          float wadd, float mult) {
    const int lane = threadIdx.x & (W - 1);
    const int64_t grow = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / W;
    // lanes past the last row still join the shuffles, on a clamped row, and store nothing
    const bool valid = grow < rows;
    const int64_t row = valid ? grow : rows - 1;
    const __nv_bfloat16* xr = x + row * n;
    const __nv_bfloat16* dyr = dy + row * n;
    float ss = 0.0f, t = 0.0f;
    for (int c = lane * 8; c < n; c += W * 8) {
        float v[8], d[8], g[8];
        load8(xr + c, v);
        load8(dyr + c, d);
        if (w) loadw8(w + c, g);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            ss = fmaf(v[i], v[i], ss);
            t = fmaf(d[i] * v[i], w ? g[i] + wadd : 1.0f, t);
        }
    }
    ss = group_sum<W>(ss);
    t = group_sum<W>(t);
    const float s = rsqrtf(ss / (float)n + eps);
    const float k = s * s * s * t / (float)n;
    for (int c = lane * 8; c < n; c += W * 8) {
        float v[8], d[8], g[8], a[8];
        load8(xr + c, v);
        load8(dyr + c, d);
        if (w) loadw8(w + c, g);
        if (addend) load8(addend + row * n + c, a);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float cc = w ? g[i] + wadd : 1.0f;
            v[i] = mult * (s * cc * d[i] - k * v[i]) + (addend ? a[i] : 0.0f);
        }
        if (valid) store8(dx + row * n + c, v);
    }
}

// z rows may live inside a wider token row: row r of z is at (r / zh) * zts + (r % zh) * n when zh > 0
// The z row of gated row r: token r / zh (row stride zts), head r % zh (n columns each); 32-bit division
// (the launchers keep rows below 2^32).
__device__ __forceinline__ int64_t zrow(int64_t r, int n, int64_t zts, int zh) {
    if (zh <= 0) return r * (int64_t)n;
    const uint32_t q = (uint32_t)r / (uint32_t)zh, m = (uint32_t)r - q * (uint32_t)zh;
    return (int64_t)q * zts + (int64_t)m * n;
}

template <int W>
__global__ void __launch_bounds__(256) gated_rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                                const __nv_bfloat16* __restrict__ z,
                                                                const float* __restrict__ w, __nv_bfloat16* __restrict__ o,
                                                                int64_t rows, int n, float eps, int sig, int64_t zts,
                                                                int zh) {
    const int lane = threadIdx.x & (W - 1);
    const int64_t grow = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / W;
    // lanes past the last row still join the shuffles, on a clamped row, and store nothing
    const bool valid = grow < rows;
    const int64_t row = valid ? grow : rows - 1;
    float ss = 0.0f;
    for (int c = lane * 8; c < n; c += W * 8) {
        float v[8];
        load8(x + row * n + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
    }
    ss = group_sum<W>(ss);
    const float s = rsqrtf(ss / (float)n + eps);
    for (int c = lane * 8; c < n; c += W * 8) {
        float v[8], zz[8], g[8];
        load8(x + row * n + c, v);
        load8(z + zrow(row, n, zts, zh) + c, zz);
        loadw8(w + c, g);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float sg = sigmoidf_(zz[i]);
            v[i] = v[i] * s * g[i] * (sig ? sg : zz[i] * sg);
        }
        if (valid) store8(o + row * n + c, v);
    }
}

template <int W>
__global__ void __launch_bounds__(256) gated_rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                                const __nv_bfloat16* __restrict__ z,
                                                                const float* __restrict__ w,
                                                                const __nv_bfloat16* __restrict__ dout,
                                                                __nv_bfloat16* __restrict__ dx, __nv_bfloat16* __restrict__ dz,
                                                                int64_t rows, int n, float eps, int sig, int64_t zts,
                                                                int zh) {
    const int lane = threadIdx.x & (W - 1);
    const int64_t grow = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / W;
    // lanes past the last row still join the shuffles, on a clamped row, and store nothing
    const bool valid = grow < rows;
    const int64_t row = valid ? grow : rows - 1;
    float ss = 0.0f, a = 0.0f;
    for (int c = lane * 8; c < n; c += W * 8) {
        float v[8], zz[8], g[8], d[8];
        load8(x + row * n + c, v);
        load8(z + zrow(row, n, zts, zh) + c, zz);
        load8(dout + row * n + c, d);
        loadw8(w + c, g);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float sg = sigmoidf_(zz[i]);
            const float gate = sig ? sg : zz[i] * sg;
            ss = fmaf(v[i], v[i], ss);
            a = fmaf(v[i] * d[i], g[i] * gate, a);
        }
    }
    ss = group_sum<W>(ss);
    a = group_sum<W>(a);
    const float s = rsqrtf(ss / (float)n + eps);
    const float k = s * s * s * a / (float)n;
    for (int c = lane * 8; c < n; c += W * 8) {
        float v[8], zz[8], g[8], d[8], ox[8], oz[8];
        load8(x + row * n + c, v);
        load8(z + zrow(row, n, zts, zh) + c, zz);
        load8(dout + row * n + c, d);
        loadw8(w + c, g);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float sg = sigmoidf_(zz[i]);
            const float gate = sig ? sg : zz[i] * sg;
            const float dgate = sig ? sg * (1.0f - sg) : sg * (1.0f + zz[i] * (1.0f - sg));
            ox[i] = g[i] * gate * s * d[i] - v[i] * k;
            oz[i] = d[i] * v[i] * s * g[i] * dgate;
        }
        if (valid) {
            store8(dx + row * n + c, ox);
            store8(dz + zrow(row, n, zts, zh) + c, oz);
        }
    }
}

// ---- wide rows held in registers: 128 threads a row (two rows a 256-thread block), VPT 8-vectors each
// (n = 1024 VPT); every load of the row is in flight at once and x is read once.
template <int VPT>
__device__ __forceinline__ float row_sum128(float v, float* red) {
    v = group_sum<32>(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    const int b = (threadIdx.x >> 7) * 4;
    return red[b] + red[b + 1] + red[b + 2] + red[b + 3];
}

template <int VPT>
__global__ void __launch_bounds__(256) rmsnorm_fwd_row(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                                       __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                       int64_t rows, float eps, float wadd, float mult) {
    __shared__ float red[8];
    constexpr int n = VPT * 1024;
    const int t = threadIdx.x & 127;
    const int64_t grow = (int64_t)blockIdx.x * 2 + (threadIdx.x >> 7);
    const bool valid = grow < rows;
    const int64_t row = valid ? grow : rows - 1;
    float v[VPT][8];
#pragma unroll
    for (int i = 0; i < VPT; ++i) load8(x + row * n + (i * 128 + t) * 8, v[i]);
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(v[i][e], v[i][e], ss);
    ss = row_sum128<VPT>(ss, red);
    const float s = rsqrtf(ss / (float)n + eps);
    if (rstd && t == 0 && valid) rstd[row] = s;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int c = (i * 128 + t) * 8;
        float g[8];
        if (w) loadw8(w + c, g);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = v[i][e] * s * (w ? g[e] + wadd : 1.0f) * mult;
        if (valid) store8(y + row * n + c, v[i]);
    }
}

template <int VPT>
__global__ void __launch_bounds__(256) rmsnorm_bwd_row(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                                       const __nv_bfloat16* __restrict__ dy,
                                                       const __nv_bfloat16* __restrict__ addend,
                                                       __nv_bfloat16* __restrict__ dx, int64_t rows, float eps,
                                                       float wadd, float mult) {
    __shared__ float red[2][8];
    constexpr int n = VPT * 1024;
    const int t = threadIdx.x & 127;
    const int64_t grow = (int64_t)blockIdx.x * 2 + (threadIdx.x >> 7);
    const bool valid = grow < rows;
    const int64_t row = valid ? grow : rows - 1;
    float v[VPT][8], d[VPT][8], ad[VPT][8];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        load8(x + row * n + (i * 128 + t) * 8, v[i]);
        load8(dy + row * n + (i * 128 + t) * 8, d[i]);
    }
    if (addend)  // the residual addend's loads fly during the reduction
#pragma unroll
        for (int i = 0; i < VPT; ++i) load8(addend + row * n + (i * 128 + t) * 8, ad[i]);
    float ss = 0.0f, tt = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        float g[8];
        if (w) loadw8(w + (i * 128 + t) * 8, g);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            ss = fmaf(v[i][e], v[i][e], ss);
            tt = fmaf(d[i][e] * v[i][e], w ? g[e] + wadd : 1.0f, tt);
        }
    }
    ss = group_sum<32>(ss);
    tt = group_sum<32>(tt);
    if ((threadIdx.x & 31) == 0) {
        red[0][threadIdx.x >> 5] = ss;
        red[1][threadIdx.x >> 5] = tt;
    }
    __syncthreads();
    const int b = (threadIdx.x >> 7) * 4;
    ss = red[0][b] + red[0][b + 1] + red[0][b + 2] + red[0][b + 3];
    tt = red[1][b] + red[1][b + 1] + red[1][b + 2] + red[1][b + 3];
    const float s = rsqrtf(ss / (float)n + eps);
    const float k = s * s * s * tt / (float)n;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int c = (i * 128 + t) * 8;
        float g[8];
        if (w) loadw8(w + c, g);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float cc = w ? g[e] + wadd : 1.0f;
            v[i][e] = mult * (s * cc * d[i][e] - k * v[i][e]) + (addend ? ad[i][e] : 0.0f);
        }
        if (valid) store8(dx + row * n + c, v[i]);
    }
}

// ---- the gated norm's 128-wide head rows: 16 lanes a row, each lane-group R rows with every load of its
// rows issued before the first reduction.
template <int R>
__global__ void __launch_bounds__(256) gated_fwd128(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ z,
                                                    const float* __restrict__ w, __nv_bfloat16* __restrict__ o,
                                                    int64_t rows, float eps, int sig, int64_t zts, int zh) {
    const int lane = threadIdx.x & 15;
    const int64_t grp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
    float g[8];
    loadw8(w + lane * 8, g);
    float xv[R][8], zv[R][8];
    int64_t rr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t row = grp * R + r;
        rr[r] = row < rows ? row : rows - 1;
        load8(x + rr[r] * 128 + lane * 8, xv[r]);
        load8(z + zrow(rr[r], 128, zts, zh) + lane * 8, zv[r]);
    }
    float ss[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        ss[r] = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss[r] = fmaf(xv[r][e], xv[r][e], ss[r]);
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1)
#pragma unroll
        for (int r = 0; r < R; ++r) ss[r] += __shfl_xor_sync(0xFFFFFFFFu, ss[r], off);
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float s = rsqrtf(ss[r] / 128.0f + eps);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float sg = sigmoidf_(zv[r][e]);
            xv[r][e] = xv[r][e] * s * g[e] * (sig ? sg : zv[r][e] * sg);
        }
        if (grp * R + r < rows) store8(o + rr[r] * 128 + lane * 8, xv[r]);
    }
}

template <int R>
__global__ void __launch_bounds__(256) gated_bwd128(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ z,
                                                    const float* __restrict__ w, const __nv_bfloat16* __restrict__ dout,
                                                    __nv_bfloat16* __restrict__ dx, __nv_bfloat16* __restrict__ dz,
                                                    int64_t rows, float eps, int sig, int64_t zts, int zh) {
    const int lane = threadIdx.x & 15;
    const int64_t grp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
    float g[8];
    loadw8(w + lane * 8, g);
    float xv[R][8], zv[R][8], dv[R][8];
    int64_t rr[R], zr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t row = grp * R + r;
        rr[r] = row < rows ? row : rows - 1;
        zr[r] = zrow(rr[r], 128, zts, zh);
        load8(x + rr[r] * 128 + lane * 8, xv[r]);
        load8(z + zr[r] + lane * 8, zv[r]);
        load8(dout + rr[r] * 128 + lane * 8, dv[r]);
    }
    float ss[R], a[R], sgv[R][8];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        ss[r] = 0.0f;
        a[r] = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float sg = sgv[r][e] = sigmoidf_(zv[r][e]);
            const float gate = sig ? sg : zv[r][e] * sg;
            ss[r] = fmaf(xv[r][e], xv[r][e], ss[r]);
            a[r] = fmaf(xv[r][e] * dv[r][e], g[e] * gate, a[r]);
        }
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1)
#pragma unroll
        for (int r = 0; r < R; ++r) {
            ss[r] += __shfl_xor_sync(0xFFFFFFFFu, ss[r], off);
            a[r] += __shfl_xor_sync(0xFFFFFFFFu, a[r], off);
        }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const float s = rsqrtf(ss[r] / 128.0f + eps);
        const float k = s * s * s * a[r] / 128.0f;
        float ox[8], oz[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float sg = sgv[r][e];
            const float gate = sig ? sg : zv[r][e] * sg;
            const float dgate = sig ? sg * (1.0f - sg) : sg * (1.0f + zv[r][e] * (1.0f - sg));
            ox[e] = g[e] * gate * s * dv[r][e] - xv[r][e] * k;
            oz[e] = dv[r][e] * xv[r][e] * s * g[e] * dgate;
        }
        if (grp * R + r < rows) {
            store8(dx + rr[r] * 128 + lane * 8, ox);
            store8(dz + zr[r] + lane * 8, oz);
        }
    }
}

constexpr int kGatedFwdRows = 2;
constexpr int kGatedBwdRows = 1;

int group_width(int n) {
    // lanes per row: a full warp once the row has 256+ elements, else one 8-vector per lane
    int w = n / 8;
    if (w >= 32) return 32;
    if (w >= 16) return 16;
    if (w >= 8) return 8;
    if (w >= 4) return 4;
    return 0;
}

#define R97B_DISPATCH_W(W, CALL)                  \
    switch (W) {                                  \
        case 32: { constexpr int kW = 32; CALL; } break; \
        case 16: { constexpr int kW = 16; CALL; } break; \
        case 8: { constexpr int kW = 8; CALL; } break;   \
        case 4: { constexpr int kW = 4; CALL; } break;   \
        default: return R97B_EINVAL;              \
    }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace r97b

using namespace r97b;

extern "C" int r97b_rmsnorm_fwd(const uint16_t* x, const float* w, uint16_t* y, float* rstd, int64_t rows, int64_t n,
                                float eps, float wadd, float mult, void* stream) {
    if (!x || !y || rows <= 0 || n <= 0 || n % 8 || !aligned16(x) || !aligned16(y) || (w && !aligned16(w)))
        return R97B_EINVAL;
    if (n == 1024 || n == 2048 || n == 4096 || n == 8192) {
        const unsigned blocks = (unsigned)((rows + 1) / 2);
        auto xb = reinterpret_cast<const __nv_bfloat16*>(x);
        auto yb = reinterpret_cast<__nv_bfloat16*>(y);
        cudaStream_t st = as_stream(stream);
        if (n == 1024) rmsnorm_fwd_row<1><<<blocks, 256, 0, st>>>(xb, w, yb, rstd, rows, eps, wadd, mult);
        else if (n == 2048) rmsnorm_fwd_row<2><<<blocks, 256, 0, st>>>(xb, w, yb, rstd, rows, eps, wadd, mult);
        else if (n == 4096) rmsnorm_fwd_row<4><<<blocks, 256, 0, st>>>(xb, w, yb, rstd, rows, eps, wadd, mult);
        else rmsnorm_fwd_row<8><<<blocks, 256, 0, st>>>(xb, w, yb, rstd, rows, eps, wadd, mult);
        return launch_status();
    }
    const int W = group_width((int)n);
    const int64_t threads = rows * (W ? W : 1);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    R97B_DISPATCH_W(W, (rmsnorm_fwd_kernel<kW><<<blocks, 256, 0, as_stream(stream)>>>(
                            reinterpret_cast<const __nv_bfloat16*>(x), w, reinterpret_cast<__nv_bfloat16*>(y), rstd,
                            rows, (int)n, eps, wadd, mult)));
    return launch_status();
}

extern "C" int r97b_rmsnorm_bwd(const uint16_t* x, const float* w, const uint16_t* dy, const uint16_t* addend,
                                uint16_t* dx, int64_t rows, int64_t n, float eps, float wadd, float mult, void* stream) {
    if (!x || !dy || !dx || rows <= 0 || n <= 0 || n % 8 || !aligned16(x) || !aligned16(dy) || !aligned16(dx) ||
        (w && !aligned16(w)) || (addend && !aligned16(addend)))
        return R97B_EINVAL;
    if (n == 1024 || n == 2048 || n == 4096 || n == 8192) {
        const unsigned blocks = (unsigned)((rows + 1) / 2);
        auto xb = reinterpret_cast<const __nv_bfloat16*>(x);
        auto db = reinterpret_cast<const __nv_bfloat16*>(dy);
        auto ab = reinterpret_cast<const __nv_bfloat16*>(addend);
        auto ob = reinterpret_cast<__nv_bfloat16*>(dx);
        cudaStream_t st = as_stream(stream);
        if (n == 1024) rmsnorm_bwd_row<1><<<blocks, 256, 0, st>>>(xb, w, db, ab, ob, rows, eps, wadd, mult);
        else if (n == 2048) rmsnorm_bwd_row<2><<<blocks, 256, 0, st>>>(xb, w, db, ab, ob, rows, eps, wadd, mult);
        else if (n == 4096) rmsnorm_bwd_row<4><<<blocks, 256, 0, st>>>(xb, w, db, ab, ob, rows, eps, wadd, mult);
        else rmsnorm_bwd_row<8><<<blocks, 256, 0, st>>>(xb, w, db, ab, ob, rows, eps, wadd, mult);
        return launch_status();
    }
    const int W = group_width((int)n);
    const int64_t threads = rows * (W ? W : 1);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    R97B_DISPATCH_W(W, (rmsnorm_bwd_kernel<kW><<<blocks, 256, 0, as_stream(stream)>>>(
                            reinterpret_cast<const __nv_bfloat16*>(x), w, reinterpret_cast<const __nv_bfloat16*>(dy),
                            reinterpret_cast<const __nv_bfloat16*>(addend), reinterpret_cast<__nv_bfloat16*>(dx), rows,
                            (int)n, eps, wadd, mult)));
    return launch_status();
}

extern "C" int r97b_gated_rmsnorm_fwd(const uint16_t* x, const uint16_t* z, int64_t z_tok_stride, int32_t z_heads,
                                      const float* w, uint16_t* o, int64_t rows, int64_t n, float eps,
                                      int32_t act_sigmoid, void* stream) {
    if (z_heads < 0 || (z_heads > 0 && (rows % z_heads || z_tok_stride % 8))) return R97B_EINVAL;
    if (rows > (int64_t)UINT32_MAX) return R97B_EINVAL;  // zrow divides in 32 bits
    if (!x || !z || !w || !o || rows <= 0 || n <= 0 || n % 8 || !aligned16(x) || !aligned16(z) || !aligned16(w) ||
        !aligned16(o))
        return R97B_EINVAL;
    if (n == 128) {
        const int64_t groups = (rows + kGatedFwdRows - 1) / kGatedFwdRows;
        gated_fwd128<kGatedFwdRows><<<(unsigned)((groups * 16 + 255) / 256), 256, 0, as_stream(stream)>>>(
            reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(z), w,
            reinterpret_cast<__nv_bfloat16*>(o), rows, eps, act_sigmoid, z_tok_stride, z_heads);
        return launch_status();
    }
    const int W = group_width((int)n);
    const int64_t threads = rows * (W ? W : 1);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    R97B_DISPATCH_W(W, (gated_rmsnorm_fwd_kernel<kW><<<blocks, 256, 0, as_stream(stream)>>>(
                            reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(z), w,
                            reinterpret_cast<__nv_bfloat16*>(o), rows, (int)n, eps, act_sigmoid, z_tok_stride,
                            z_heads)));
    return launch_status();
}

extern "C" int r97b_gated_rmsnorm_bwd(const uint16_t* x, const uint16_t* z, int64_t z_tok_stride, int32_t z_heads,
                                      const float* w, const uint16_t* dout, uint16_t* dx, uint16_t* dz, int64_t rows,
                                      int64_t n, float eps, int32_t act_sigmoid, void* stream) {
    if (z_heads < 0 || (z_heads > 0 && (rows % z_heads || z_tok_stride % 8))) return R97B_EINVAL;
    if (rows > (int64_t)UINT32_MAX) return R97B_EINVAL;  // zrow divides in 32 bits
    if (!x || !z || !w || !dout || !dx || !dz || rows <= 0 || n <= 0 || n % 8 || !aligned16(x) || !aligned16(z) ||
        !aligned16(w) || !aligned16(dout) || !aligned16(dx) || !aligned16(dz))
        return R97B_EINVAL;
    if (n == 128) {
        const int64_t groups = (rows + kGatedBwdRows - 1) / kGatedBwdRows;
        gated_bwd128<kGatedBwdRows><<<(unsigned)((groups * 16 + 255) / 256), 256, 0, as_stream(stream)>>>(
            reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(z), w,
            reinterpret_cast<const __nv_bfloat16*>(dout), reinterpret_cast<__nv_bfloat16*>(dx),
            reinterpret_cast<__nv_bfloat16*>(dz), rows, eps, act_sigmoid, z_tok_stride, z_heads);
        return launch_status();
    }
    const int W = group_width((int)n);
    const int64_t threads = rows * (W ? W : 1);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    R97B_DISPATCH_W(W, (gated_rmsnorm_bwd_kernel<kW><<<blocks, 256, 0, as_stream(stream)>>>(
                            reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(z), w,
                            reinterpret_cast<const __nv_bfloat16*>(dout), reinterpret_cast<__nv_bfloat16*>(dx),
                            reinterpret_cast<__nv_bfloat16*>(dz), rows, (int)n, eps, act_sigmoid, z_tok_stride,
                            z_heads)));
    return launch_status();
}
