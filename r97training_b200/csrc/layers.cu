// layers.cu -- the elementwise and per-row kernels around the GEMMs and the recurrence of one hybrid
// block, forward and backward, on sm_100a. All HBM-bound: 16-byte vector loads, f32 math, bf16 stores.
//
//   conv prep   causal depthwise conv (width 4) + silu over the q|k|v channels, L2 norm of q and k per
//               head (eps 1e-6)             (reference src/adjoint/host/gdn_prep.cpp:204-365, 367-489)
//   gates       g = chunk-local cumsum of -exp(A_log) softplus(a + dt_bias) (threshold 20), beta = sigmoid(b)
//   swiglu      y = silu(gate) * up over a fused [rows, 2n] row (reference elementwise.cpp:278-312 silu_mul)
//   attention   q/k RMSNorm per head + partial NeoX RoPE into the [B, H, S, D] layout the attention core
//   prep        reads, and the sigmoid output gate (reference src/adjoint/host/qk.cpp, rope.cpp, attention.cpp)
//   embedding   row gather of the tied head weight
//   casts       f32 -> bf16 2-D strided copies (adapter mirrors)
#include "r97b_internal.h"
#include "wmma16.cuh"
#include "fastmath.cuh"

#include <cuda_bf16.h>
#include <math.h>

namespace r97b {
namespace {

__device__ __forceinline__ float sigm(float x) { return sigmoid_ftz(x); }
__device__ __forceinline__ float silu(float x) { return x * sigm(x); }
__device__ __forceinline__ float silu_grad(float x) {
    const float s = sigm(x);
    return s * (1.0f + x * (1.0f - s));
}
__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float (&v)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void ld8f(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

__device__ __forceinline__ float sum32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

constexpr int kW = 4;  // conv width

// ------------------------------------------------------------------------------------------- conv prep

struct ConvArgs {
    const __nv_bfloat16* x;
    int64_t ldx;
    const float* w;  // [conv_dim, 4]
    const int* cu;
    int n_seq, T, Hg, H, conv_dim;
};

__device__ __forceinline__ void ld4(const __nv_bfloat16* p, float (&v)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
    v[0] = f0.x, v[1] = f0.y, v[2] = f1.x, v[3] = f1.y;
}
__device__ __forceinline__ void st4(__nv_bfloat16* p, const float (&v)[4]) {
    uint2 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
    h[0] = __floats2bfloat162_rn(v[0], v[1]);
    h[1] = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(p) = u;
}
// The conv prep, forward and adjoint. A thread owns 4 channels [c, c + 4) of a run of consecutive tokens;
// a warp is one 128-wide head, so a head's L2-norm sums are warp reductions. Tokens go in groups of four:
// the group's rows are loaded together, its four tokens' conv outputs and partial sums formed, and the
// eight warp reductions of a group interleaved, so the shuffles' latency overlaps.
constexpr int kG = 4;
constexpr int kRunF = 32;                // tokens a forward thread emits (8 groups)

// sigmoid by the fast exponential; silu(x) = x s, silu'(x) = s (1 + x (1 - s))
__device__ __forceinline__ float sigm_fast(float x) { return sigmoid_ftz(x); }

struct ConvRun {
    int t_begin, c;
    bool valid;
};

// The thread's channels and token run; whole warps are valid or not (the channel groups are a multiple
// of 32, so a warp never straddles the end).
__device__ __forceinline__ ConvRun conv_run(const ConvArgs& a, int run) {
    const int groups = a.conv_dim / 4;
    const int runs = (a.T + run - 1) / run;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    ConvRun r;
    r.valid = gid < (int64_t)runs * groups;
    const int64_t gi = r.valid ? gid : (int64_t)runs * groups - 1;
    r.t_begin = (int)(gi / groups) * run;
    r.c = (int)(gi % groups) * 4;
    return r;
}

__device__ __forceinline__ void load_w4(const ConvArgs& a, int c, float (&w)[4][kW]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(a.w + (c + i) * kW);
        w[i][0] = v.x, w[i][1] = v.y, w[i][2] = v.z, w[i][3] = v.w;
    }
}

__device__ __forceinline__ void load_x4(const ConvArgs& a, int c, int t, float (&v)[4]) {
    if (t >= 0 && t < a.T) ld4(a.x + (int64_t)t * a.ldx + c, v);
    else v[0] = v[1] = v[2] = v[3] = 0.0f;
}

// Tracks the sequence holding a token as tokens advance: start/end of it.
struct SeqCursor {
    int s, start, end;
    __device__ __forceinline__ void init(const ConvArgs& a, int t) {
        s = 0;
        while (s + 1 < a.n_seq && a.cu[s + 1] <= t) ++s;
        start = a.cu[s];
        end = a.cu[s + 1];
    }
    __device__ __forceinline__ void advance(const ConvArgs& a, int t) {
        while (t >= end && s + 1 < a.n_seq) {
            ++s;
            start = a.cu[s];
            end = a.cu[s + 1];
        }
    }
};

__global__ void __launch_bounds__(256) conv_prep_fwd_kernel(ConvArgs a, __nv_bfloat16* __restrict__ q,
                                                            __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v) {
    const ConvRun cr = conv_run(a, kRunF);
    const int c = cr.c;
    float w[4][kW];
    load_w4(a, c, w);
    const int qk = a.Hg * 128;
    const bool normed = c < 2 * qk;
    __nv_bfloat16* dst;
    int64_t stride;
    if (c < qk) dst = q + c, stride = qk;
    else if (c < 2 * qk) dst = k + (c - qk), stride = qk;
    else dst = v + (c - 2 * qk), stride = (int64_t)a.H * 128;
    float xr[kW - 1 + kG][4];  // rows t0 - 3 .. t0 + 3 of the current group at t0
#pragma unroll
    for (int j = 0; j < kW - 1; ++j) load_x4(a, c, cr.t_begin - (kW - 1) + j, xr[j]);
    SeqCursor sq;
    sq.init(a, cr.t_begin);
#pragma unroll 1
    for (int g0 = 0; g0 < kRunF; g0 += kG) {
        const int tg = cr.t_begin + g0;
#pragma unroll
        for (int j = 0; j < kG; ++j) load_x4(a, c, tg + j, xr[kW - 1 + j]);
        float u[kG][4], ss[kG];
#pragma unroll
        for (int j = 0; j < kG; ++j) {
            sq.advance(a, tg + j);
            ss[j] = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float acc = 0.0f;
#pragma unroll
                for (int tap = 0; tap < kW; ++tap)
                    acc = fmaf(tg + j - (kW - 1) + tap >= sq.start ? xr[j + tap][i] : 0.0f, w[i][tap], acc);
                u[j][i] = acc * sigm_fast(acc);
                ss[j] = fmaf(u[j][i], u[j][i], ss[j]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int j = 0; j < kG; ++j) ss[j] += __shfl_xor_sync(0xFFFFFFFFu, ss[j], o);
#pragma unroll
        for (int j = 0; j < kG; ++j) {
            const int t = tg + j;
            if (normed) {
                const float inv = rsqrt_ftz(ss[j] + 1e-6f);
#pragma unroll
                for (int i = 0; i < 4; ++i) u[j][i] *= inv;
            }
            if (cr.valid && t < a.T) st4(dst + (int64_t)t * stride, u[j]);
        }
#pragma unroll
        for (int j = 0; j < kW - 1; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) xr[j][i] = xr[kG + j][i];
    }
}

// The sequence holding token t: cu[s] <= t < cu[s + 1] (binary search over the n_seq + 1 bounds).
__device__ __forceinline__ void seq_bounds(const ConvArgs& a, int t, int& start, int& end) {
    int lo = 0, hi = a.n_seq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.cu[mid] <= t) lo = mid;
        else hi = mid - 1;
    }
    start = a.cu[lo];
    end = a.cu[lo + 1];
}

// The adjoint by token tiles, persistent and double-buffered. A tile is kConvTT tokens of one 128-channel
// head; a CTA walks tiles blockIdx.x, + gridDim.x, ... (heads fastest, so the CTAs in flight read whole token
// rows), staging the next tile's x rows t0 - 3 .. t0 + kConvTT + 2 and d rows (dq/dk per value head: grp
// slices a row) in shared memory by cp.async while it works on the current one, so HBM streams throughout.
// On a tile a half-warp takes one token row, a lane 8 channels (two groups of 4, 64 apart, so every shared
// access of a half-warp is one contiguous run): phase 1 rebuilds the conv output of rows t0 .. t0 + kConvTT + 2
// and forms dacc (silu's and, for q/k, the L2 norm's backward: two half-warp reductions over the head's row)
// over the row's first d slice; phase 2 emits dx(t) = sum_{s = 0..3, same sequence} dacc(t + s) w[c, 3 - s].
constexpr int kConvRows = 32;                   // dacc rows a tile forms: two per warp, twice
constexpr int kConvTT = kConvRows - (kW - 1);   // tokens a tile emits
constexpr int kConvXRows = kConvRows + kW - 1;  // x rows it reads

struct ConvStage {  // byte offsets within a stage
    int ds, seq, bytes;
};
__host__ __device__ inline ConvStage conv_stage(int grp) {
    ConvStage st;
    st.ds = kConvXRows * 256;                              // x: [kConvXRows][128] bf16
    st.seq = st.ds + kConvRows * grp * 128 * 4;            // d: [kConvRows][grp * 128] f32
    st.bytes = (st.seq + 2 * kConvRows * 4 + 15) & ~15;  // sequence start / end of each row's token
    return st;
}

__device__ __forceinline__ void cp_async8(void* dst, const void* src, bool pred) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(s_addr(dst)), "l"(src), "r"(pred ? 8 : 0)
                 : "memory");
}

struct ConvBwdArgs {
    const float* dq;
    const float* dk;
    const float* dv;
    int grp, n_tiles;
    __nv_bfloat16* dx;
    int64_t lddx;
};

// Stage a tile: every thread issues its share of the 8-byte x and 16-byte d copies (zeros past the tokens),
// and threads 0 .. kConvRows - 1 write their row's sequence bounds.
__device__ __forceinline__ void conv_bwd_issue(const ConvArgs& a, const ConvBwdArgs& b, const ConvStage& sl,
                                               unsigned char* stage, int tile) {
    const int heads = a.conv_dim >> 7, head = tile % heads, t0 = (tile / heads) * kConvTT;
    const int cbase = head * 128, qk = a.Hg * 128;
    const __nv_bfloat16* xsrc = a.x + cbase + (threadIdx.x & 31) * 4;
#pragma unroll
    for (int k = 0; k < (kConvXRows * 32 + 255) / 256; ++k) {
        const int r = (threadIdx.x >> 5) + 8 * k, tt = t0 - (kW - 1) + r;
        const bool on = tt >= 0 && tt < a.T;
        if (r < kConvXRows)
            cp_async8(stage + r * 256 + (threadIdx.x & 31) * 8, xsrc + (int64_t)(on ? tt : 0) * a.ldx, on);
    }
    const float* src;
    int64_t stride;
    int nsum;
    if (cbase < 2 * qk) {
        const int cc = cbase < qk ? cbase : cbase - qk;
        stride = (int64_t)a.Hg * b.grp * 128;
        nsum = b.grp;
        src = (cbase < qk ? b.dq : b.dk) + (int64_t)(cc >> 7) * b.grp * 128;
    } else {
        stride = (int64_t)a.H * 128;
        nsum = 1;
        src = b.dv + (cbase - 2 * qk);
    }
    float* ds = reinterpret_cast<float*>(stage + sl.ds) + (threadIdx.x & 31) * 4;
    src += (threadIdx.x & 31) * 4;
    const int dw = b.grp * 128;
    for (int k = threadIdx.x >> 5; k < kConvRows * nsum; k += 8) {
        const int r = k & (kConvRows - 1), e = k / kConvRows, t = t0 + r;
        const bool on = t < a.T;
        cp_async16(ds + r * dw + e * 128, src + (int64_t)(on ? t : 0) * stride + e * 128, on);
    }
    if (threadIdx.x < kConvRows) {
        const int t = t0 + threadIdx.x;
        int start = 0, end = 0;
        if (t < a.T) seq_bounds(a, t, start, end);
        int* seq = reinterpret_cast<int*>(stage + sl.seq);
        seq[threadIdx.x] = start;
        seq[kConvRows + threadIdx.x] = end;
    }
}

__device__ __forceinline__ void unpack4(uint2 u, float* v) {
    const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    v[0] = f0.x, v[1] = f0.y, v[2] = f1.x, v[3] = f1.y;
}

template <bool NORMED>
__device__ __forceinline__ void conv_bwd_tile(const ConvArgs& a, const ConvBwdArgs& b, const ConvStage& sl,
                                              unsigned char* stage, int head, int t0) {
    const int warp = threadIdx.x >> 5, half = (threadIdx.x >> 4) & 1, hl = threadIdx.x & 15;
    const int c = head * 128 + hl * 4;  // channels c .. c + 3 and c + 64 .. c + 67
    const int dw = b.grp * 128, nsum = NORMED ? b.grp : 1;
    const uint2* xs = reinterpret_cast<const uint2*>(stage);
    float* ds = reinterpret_cast<float*>(stage + sl.ds) + hl * 4;
    const int* seq = reinterpret_cast<const int*>(stage + sl.seq);
    float w[8][kW];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(a.w + (c + (i >> 2) * 64 + (i & 3)) * kW);
        w[i][0] = v.x, w[i][1] = v.y, w[i][2] = v.z, w[i][3] = v.w;
    }
    // phase 1: dacc over each row's first slice
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int r = j * 16 + warp * 2 + half, t = t0 + r;
        uint2 u[kW][2];
#pragma unroll
        for (int tap = 0; tap < kW; ++tap) {
            u[tap][0] = xs[(r + tap) * 32 + hl];
            u[tap][1] = xs[(r + tap) * 32 + 16 + hl];
        }
        const int lim = seq[r] - (t - (kW - 1));  // taps below lim lie before the sequence's start
        if (lim > 0) {
#pragma unroll
            for (int tap = 0; tap < kW; ++tap)
                if (tap < lim) u[tap][0] = u[tap][1] = make_uint2(0u, 0u);
        }
        float d[8];
        {
            const float4 d0 = *reinterpret_cast<const float4*>(ds + r * dw);
            const float4 d1 = *reinterpret_cast<const float4*>(ds + r * dw + 64);
            d[0] = d0.x, d[1] = d0.y, d[2] = d0.z, d[3] = d0.w, d[4] = d1.x, d[5] = d1.y, d[6] = d1.z, d[7] = d1.w;
        }
        for (int e = 1; e < nsum; ++e) {
            const float4 d0 = *reinterpret_cast<const float4*>(ds + r * dw + e * 128);
            const float4 d1 = *reinterpret_cast<const float4*>(ds + r * dw + e * 128 + 64);
            d[0] += d0.x, d[1] += d0.y, d[2] += d0.z, d[3] += d0.w;
            d[4] += d1.x, d[5] += d1.y, d[6] += d1.z, d[7] += d1.w;
        }
        float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int tap = 0; tap < kW; ++tap) {
            float xv[8];
            unpack4(u[tap][0], xv);
            unpack4(u[tap][1], xv + 4);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = fmaf(xv[i], w[i][tap], acc[i]);
        }
        float sg[8], o[8], ss = 0.0f, dot = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            sg[i] = sigm_fast(acc[i]);
            if (NORMED) {
                const float uu = acc[i] * sg[i];
                ss = fmaf(uu, uu, ss);
                dot = fmaf(uu, d[i], dot);
            }
        }
        if (NORMED) {
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) {
                ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
                dot += __shfl_xor_sync(0xFFFFFFFFu, dot, off);
            }
            const float inv = rsqrt_ftz(ss + 1e-6f), k3 = inv * inv * inv * dot;
#pragma unroll
            for (int i = 0; i < 8; ++i) d[i] = inv * d[i] - k3 * (acc[i] * sg[i]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = t < a.T ? d[i] * (sg[i] * (1.0f + acc[i] * (1.0f - sg[i]))) : 0.0f;
        *reinterpret_cast<float4*>(ds + r * dw) = make_float4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<float4*>(ds + r * dw + 64) = make_float4(o[4], o[5], o[6], o[7]);
    }
    __syncthreads();
    // phase 2: the transposed conv
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int r = j * 16 + warp * 2 + half, t = t0 + r;
        if (r >= kConvTT || t >= a.T) continue;
        const int end = seq[kConvRows + r];
        float o[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int s2 = 0; s2 < kW; ++s2) {
            if (t + s2 < end) {
                const float4 g0 = *reinterpret_cast<const float4*>(ds + (r + s2) * dw);
                const float4 g1 = *reinterpret_cast<const float4*>(ds + (r + s2) * dw + 64);
                const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = fmaf(g[i], w[i][kW - 1 - s2], o[i]);
            }
        }
        __nv_bfloat16* dst = b.dx + (int64_t)t * b.lddx + c;
        st4(dst, *reinterpret_cast<const float(*)[4]>(o));
        st4(dst + 64, *reinterpret_cast<const float(*)[4]>(o + 4));
    }
}

__global__ void __launch_bounds__(256, 2) conv_prep_bwd_kernel(ConvArgs a, ConvBwdArgs b) {
    extern __shared__ __align__(16) unsigned char conv_smem[];
    const ConvStage sl = conv_stage(b.grp);
    const int heads = a.conv_dim >> 7;
    int tile = blockIdx.x;
    if (tile < b.n_tiles) conv_bwd_issue(a, b, sl, conv_smem, tile);
    cp_async_commit();
    for (int it = 0; tile < b.n_tiles; ++it, tile += gridDim.x) {
        if (tile + (int)gridDim.x < b.n_tiles)
            conv_bwd_issue(a, b, sl, conv_smem + ((it + 1) & 1) * sl.bytes, tile + gridDim.x);
        cp_async_commit();
        cp_async_wait_but_one();
        __syncthreads();
        unsigned char* stage = conv_smem + (it & 1) * sl.bytes;
        const int head = tile % heads, t0 = (tile / heads) * kConvTT;
        if (head < 2 * a.Hg) conv_bwd_tile<true>(a, b, sl, stage, head, t0);
        else conv_bwd_tile<false>(a, b, sl, stage, head, t0);
        __syncthreads();  // the stage is refilled next iteration but one
    }
    cp_async_wait_all();
}

// ------------------------------------------------------------------------------------------- gates

// A block per (chunk, 32 heads): thread (h, y) owns tokens [8 y, 8 y + 8) of the chunk for head h; its
// 8-token sums are combined across y through shared memory (a within-chunk scan over 8 partial sums).
constexpr int kGateTok = 8;   // tokens a thread owns
constexpr int kGateGroups = 8; // threads a head (covers the chunk's 64 tokens)

// beta = sigmoid(b); g = within-chunk running sum of the decay increment decay * softplus(a + dt_bias)
__global__ void __launch_bounds__(256) gates_fwd_kernel(const __nv_bfloat16* __restrict__ ba, int64_t ldba,
                                                        const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                                        const int* __restrict__ tok0, const int* __restrict__ len,
                                                        int n_chunks, int H, float* __restrict__ g,
                                                        float* __restrict__ beta) {
    __shared__ float part[kGateGroups][32];
    const int c = blockIdx.x, hl = threadIdx.x & 31, y = threadIdx.x >> 5;
    const int h = blockIdx.y * 32 + hl;
    const bool on = h < H;
    const int n = len[c];
    const int64_t t0 = tok0[c];
    const float decay = on ? -expf(a_log[h]) : 0.0f;
    const float bias = on ? dt_bias[h] : 0.0f;
    float inc[kGateTok], run = 0.0f;
#pragma unroll
    for (int i = 0; i < kGateTok; ++i) {
        const int k = y * kGateTok + i;
        inc[i] = 0.0f;
        if (on && k < n) {
            const int64_t t = t0 + k;
            inc[i] = decay * softplus(__bfloat162float(ba[t * ldba + H + h]) + bias);
            beta[t * H + h] = sigm(__bfloat162float(ba[t * ldba + h]));
        }
        run += inc[i];
    }
    part[y][hl] = run;
    __syncthreads();
    float base = 0.0f;
    for (int j = 0; j < y; ++j) base += part[j][hl];
    run = base;
#pragma unroll
    for (int i = 0; i < kGateTok; ++i) {
        const int k = y * kGateTok + i;
        run += inc[i];
        if (on && k < n) g[(t0 + k) * H + h] = run;
    }
}

// d(a) = decay * sigmoid(a + dt_bias) * sum_{j >= i in the chunk} dg_j ; d(b) = dbeta * s (1 - s)
__global__ void __launch_bounds__(256) gates_bwd_kernel(const __nv_bfloat16* __restrict__ ba, int64_t ldba,
                                                        const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                                        const int* __restrict__ tok0, const int* __restrict__ len,
                                                        int n_chunks, int H, const float* __restrict__ dg,
                                                        const float* __restrict__ dbeta, __nv_bfloat16* __restrict__ dba,
                                                        int64_t lddba) {
    __shared__ float part[kGateGroups][32];
    const int c = blockIdx.x, hl = threadIdx.x & 31, y = threadIdx.x >> 5;
    const int h = blockIdx.y * 32 + hl;
    const bool on = h < H;
    const int n = len[c];
    const int64_t t0 = tok0[c];
    const float decay = on ? -expf(a_log[h]) : 0.0f;
    const float bias = on ? dt_bias[h] : 0.0f;
    float d[kGateTok], tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kGateTok; ++i) {
        const int k = y * kGateTok + i;
        d[i] = (on && k < n) ? dg[(t0 + k) * H + h] : 0.0f;
        tot += d[i];
    }
    part[y][hl] = tot;
    __syncthreads();
    float tail = 0.0f;  // the sum over the later tokens' groups
    for (int j = y + 1; j < kGateGroups; ++j) tail += part[j][hl];
#pragma unroll
    for (int i = kGateTok - 1; i >= 0; --i) {
        const int k = y * kGateTok + i;
        tail += d[i];
        if (on && k < n) {
            const int64_t t = t0 + k;
            const float av = __bfloat162float(ba[t * ldba + H + h]) + bias;
            const float sp = av > 20.0f ? 1.0f : sigm(av);
            dba[t * lddba + H + h] = __float2bfloat16_rn(tail * decay * sp);
            const float sg = sigm(__bfloat162float(ba[t * ldba + h]));
            dba[t * lddba + h] = __float2bfloat16_rn(dbeta[t * H + h] * sg * (1.0f - sg));
        }
    }
}

// ------------------------------------------------------------------------------------------- swiglu

__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, int64_t ldgu, int64_t rows,
                                                         int n, __nv_bfloat16* __restrict__ y, int64_t ldy) {
    const int groups = n / 8;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * groups) return;
    const int64_t r = gid / groups;
    const int c = (int)(gid % groups) * 8;
    float gv[8], uv[8];
    ld8(gu + r * ldgu + c, gv);
    ld8(gu + r * ldgu + n + c, uv);
#pragma unroll
    for (int i = 0; i < 8; ++i) gv[i] = silu(gv[i]) * uv[i];
    st8(y + r * ldy + c, gv);
}

__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, int64_t ldgu, int64_t rows,
                                                         int n, const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                                                         __nv_bfloat16* __restrict__ dgu, int64_t lddgu) {
    const int groups = n / 8;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * groups) return;
    const int64_t r = gid / groups;
    const int c = (int)(gid % groups) * 8;
    float gv[8], uv[8], d[8], og[8], ou[8];
    ld8(gu + r * ldgu + c, gv);
    ld8(gu + r * ldgu + n + c, uv);
    ld8(dy + r * lddy + c, d);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        og[i] = d[i] * uv[i] * silu_grad(gv[i]);
        ou[i] = d[i] * silu(gv[i]);
    }
    st8(dgu + r * lddgu + c, og);
    st8(dgu + r * lddgu + n + c, ou);
}

// ------------------------------------------------------------------------------------------- attention prep

// One warp per (token, head) row of D = 32 NV (128 or 256): RMSNorm (eps) with gain w, then NeoX RoPE on the
// first `rot` dims (lanes 0..rot/NV-1), into out[b, head, s, :] with b, s from the token's sequence. Each
// lane holds NV consecutive values of the row.
struct QkArgs {
    const __nv_bfloat16* x;  // rows of `row_stride`, head h at h * head_stride
    int64_t row_stride;
    int head_stride;
    int heads;
    const float* w;          // [D]
    const float* cosb;       // [S, rot/2]
    const float* sinb;
    int rot;
    int T, S;                // tokens, sequence length (fixed-length batch)
    float eps;
};

// q = row / d, r = row % d in 32-bit arithmetic when row fits (a 64-bit division is a long subroutine).
__device__ __forceinline__ void split_row(int64_t row, int d, int& q, int& r) {
    if (row <= 0xFFFFFFFFll) {
        const uint32_t qq = (uint32_t)row / (uint32_t)d;
        q = (int)qq;
        r = (int)((uint32_t)row - qq * (uint32_t)d);
    } else {
        q = (int)(row / d);
        r = (int)(row % d);
    }
}

// NV consecutive bf16 values (NV = 8: one 16-byte load; NV = 4: one 8-byte load) and f32 gains.
template <int NV>
__device__ __forceinline__ void ldv(const __nv_bfloat16* p, float (&v)[NV]) {
    if constexpr (NV == 8) {
        ld8(p, v);
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
        const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
        v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
    }
}
template <int NV>
__device__ __forceinline__ void stv(__nv_bfloat16* p, const float (&v)[NV]) {
    if constexpr (NV == 8) {
        st8(p, v);
    } else {
        uint2 u;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
        h[0] = __floats2bfloat162_rn(v[0], v[1]);
        h[1] = __floats2bfloat162_rn(v[2], v[3]);
        *reinterpret_cast<uint2*>(p) = u;
    }
}
template <int NV>
__device__ __forceinline__ void ldvf(const float* p, float (&v)[NV]) {
    if constexpr (NV == 8) {
        ld8f(p, v);
    } else {
        const float4 a = *reinterpret_cast<const float4*>(p);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
    }
}

template <int NV>
__global__ void __launch_bounds__(256) qk_norm_rope_fwd_kernel(QkArgs a, __nv_bfloat16* __restrict__ out) {
    constexpr int D = 32 * NV;
    const int lane = threadIdx.x & 31;
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= (int64_t)a.T * a.heads) return;
    int t, h, b, s;
    split_row(row, a.heads, t, h);
    split_row(t, a.S, b, s);
    float v[NV], w[NV];
    ldv<NV>(a.x + (int64_t)t * a.row_stride + h * a.head_stride + lane * NV, v);
    ldvf<NV>(a.w + lane * NV, w);
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) ss = fmaf(v[i], v[i], ss);
    ss = sum32(ss);
    const float r = rsqrtf(ss / (float)D + a.eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] *= r * w[i];
    const int half = a.rot / 2;          // rotary pairs (i, i + half)
    const int pl = half / NV;            // lanes holding the first half
    float o[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) o[i] = __shfl_xor_sync(0xFFFFFFFFu, v[i], pl);  // every lane joins
    if (lane < 2 * pl) {
        const bool first = lane < pl;
        const int j0 = (first ? lane : lane - pl) * NV;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float cs = a.cosb[s * half + j0 + i], sn = a.sinb[s * half + j0 + i];
            v[i] = first ? v[i] * cs - o[i] * sn : v[i] * cs + o[i] * sn;
        }
    }
    stv<NV>(out + (((int64_t)b * a.heads + h) * a.S + s) * D + lane * NV, v);
}

// The adjoint: inverse rotation of dout, then the RMSNorm adjoint against the saved pre-norm row;
// dx into rows of `dx_stride` (the projection's cotangent buffer).
template <int NV>
__global__ void __launch_bounds__(256) qk_norm_rope_bwd_kernel(QkArgs a, const __nv_bfloat16* __restrict__ dout,
                                                               __nv_bfloat16* __restrict__ dx, int64_t dx_stride) {
    constexpr int D = 32 * NV;
    const int lane = threadIdx.x & 31;
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= (int64_t)a.T * a.heads) return;
    int t, h, b, s;
    split_row(row, a.heads, t, h);
    split_row(t, a.S, b, s);
    float d[NV], x[NV], w[NV];
    ldv<NV>(dout + (((int64_t)b * a.heads + h) * a.S + s) * D + lane * NV, d);
    ldv<NV>(a.x + (int64_t)t * a.row_stride + h * a.head_stride + lane * NV, x);
    ldvf<NV>(a.w + lane * NV, w);
    const int half = a.rot / 2, pl = half / NV;
    float o[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) o[i] = __shfl_xor_sync(0xFFFFFFFFu, d[i], pl);
    if (lane < 2 * pl) {
        const bool first = lane < pl;
        const int j0 = (first ? lane : lane - pl) * NV;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float cs = a.cosb[s * half + j0 + i], sn = a.sinb[s * half + j0 + i];
            // y1 = x1 c - x2 s, y2 = x2 c + x1 s  =>  dx1 = dy1 c + dy2 s, dx2 = dy2 c - dy1 s
            d[i] = first ? d[i] * cs + o[i] * sn : d[i] * cs - o[i] * sn;
        }
    }
    float ss = 0.0f, tt = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        ss = fmaf(x[i], x[i], ss);
        tt = fmaf(d[i] * x[i], w[i], tt);
    }
    ss = sum32(ss);
    tt = sum32(tt);
    const float r = rsqrtf(ss / (float)D + a.eps);
    const float kk = r * r * r * tt / (float)D;
#pragma unroll
    for (int i = 0; i < NV; ++i) d[i] = r * w[i] * d[i] - kk * x[i];
    stv<NV>(dx + (int64_t)t * dx_stride + h * a.head_stride + lane * NV, d);
}

// [T, heads, D] rows (row stride) -> [B, heads, S, D] and back
template <int NV>
__global__ void __launch_bounds__(256) to_bhsd_kernel(const __nv_bfloat16* __restrict__ x, int64_t row_stride,
                                                      int head_stride, int heads, int T, int S,
                                                      __nv_bfloat16* __restrict__ out, int reverse) {
    constexpr int D = 32 * NV;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)T * heads * 32) return;
    const int lane = (int)(gid & 31);
    const int64_t row = gid >> 5;
    int t, h, b, s;
    split_row(row, heads, t, h);
    split_row(t, S, b, s);
    const int64_t at_bhsd = (((int64_t)b * heads + h) * S + s) * D + lane * NV;
    const int64_t at_row = (int64_t)t * row_stride + (int64_t)h * head_stride + lane * NV;
    float v[NV];
    if (reverse) {
        ldv<NV>(out + at_bhsd, v);
        stv<NV>(const_cast<__nv_bfloat16*>(x) + at_row, v);
    } else {
        ldv<NV>(x + at_row, v);
        stv<NV>(out + at_bhsd, v);
    }
}

// y[t, h*D + d] = attn[b, h, s, d] * sigmoid(gate[t, h * gate_hs + d]) ; gate rows of `gate_stride`
template <int NV>
__global__ void __launch_bounds__(256) gate_mul_fwd_kernel(const __nv_bfloat16* __restrict__ attn,
                                                           const __nv_bfloat16* __restrict__ gate, int64_t gate_stride,
                                                           int gate_hs, int heads, int T, int S,
                                                           __nv_bfloat16* __restrict__ y) {
    constexpr int D = 32 * NV;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)T * heads * 32) return;
    const int lane = (int)(gid & 31);
    const int64_t row = gid >> 5;
    int t, h, b, s;
    split_row(row, heads, t, h);
    split_row(t, S, b, s);
    float av[NV], gv[NV];
    ldv<NV>(attn + (((int64_t)b * heads + h) * S + s) * D + lane * NV, av);
    ldv<NV>(gate + (int64_t)t * gate_stride + (int64_t)h * gate_hs + lane * NV, gv);
#pragma unroll
    for (int i = 0; i < NV; ++i) av[i] *= sigm(gv[i]);
    stv<NV>(y + ((int64_t)t * heads + h) * D + lane * NV, av);
}

template <int NV>
__global__ void __launch_bounds__(256) gate_mul_bwd_kernel(const __nv_bfloat16* __restrict__ attn,
                                                           const __nv_bfloat16* __restrict__ gate, int64_t gate_stride,
                                                           int gate_hs, int heads, int T, int S,
                                                           const __nv_bfloat16* __restrict__ dy,
                                                           __nv_bfloat16* __restrict__ dattn,
                                                           __nv_bfloat16* __restrict__ dgate, int64_t dgate_stride) {
    constexpr int D = 32 * NV;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (int64_t)T * heads * 32) return;
    const int lane = (int)(gid & 31);
    const int64_t row = gid >> 5;
    int t, h, b, s;
    split_row(row, heads, t, h);
    split_row(t, S, b, s);
    const int64_t at = (((int64_t)b * heads + h) * S + s) * D + lane * NV;
    float av[NV], gv[NV], d[NV], da[NV], dg[NV];
    ldv<NV>(attn + at, av);
    ldv<NV>(gate + (int64_t)t * gate_stride + (int64_t)h * gate_hs + lane * NV, gv);
    ldv<NV>(dy + ((int64_t)t * heads + h) * D + lane * NV, d);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const float sg = sigm(gv[i]);
        da[i] = d[i] * sg;
        dg[i] = d[i] * av[i] * sg * (1.0f - sg);
    }
    stv<NV>(dattn + at, da);
    stv<NV>(dgate + (int64_t)t * dgate_stride + (int64_t)h * gate_hs + lane * NV, dg);
}

// ------------------------------------------------------------------------------------------- misc

__global__ void __launch_bounds__(256) embed_kernel(const __nv_bfloat16* __restrict__ table, int64_t ld, int64_t vocab,
                                                    const int32_t* __restrict__ ids, int64_t T, int n,
                                                    __nv_bfloat16* __restrict__ out) {
    const int groups = n / 8;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= T * groups) return;
    const int64_t t = gid / groups;
    const int c = (int)(gid % groups) * 8;
    const int id = ids[t];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (id >= 0 && id < vocab) v = *reinterpret_cast<const uint4*>(table + (int64_t)id * ld + c);
    *reinterpret_cast<uint4*>(out + t * n + c) = v;
}

__global__ void cast_2d_kernel(const float* __restrict__ src, int64_t ld_src, __nv_bfloat16* __restrict__ dst,
                               int64_t ld_dst, int64_t rows, int64_t cols) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * cols) return;
    const int64_t r = gid / cols, c = gid % cols;
    dst[r * ld_dst + c] = __float2bfloat16_rn(src[r * ld_src + c]);
}

// Many casts in one launch: thread u converts the 8 elements of unit u (units counted across the table's
// segments, each segment's rows of `cols` elements in 8-element units); the segment is found by binary
// search on the units before it.
__global__ void cast_segments_kernel(const R97bCastSeg* __restrict__ segs, int nseg, int64_t units) {
    const int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= units) return;
    int lo = 0, hi = nseg - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (segs[mid].unit0 <= u) lo = mid;
        else hi = mid - 1;
    }
    const R97bCastSeg sg = segs[lo];
    const int64_t per_row = sg.cols >> 3;
    const int64_t k = u - sg.unit0;
    const int64_t r = k / per_row, c = (k - r * per_row) * 8;
    const float4 a = *reinterpret_cast<const float4*>(sg.src + r * sg.ld_src + c);
    const float4 b = *reinterpret_cast<const float4*>(sg.src + r * sg.ld_src + c + 4);
    uint4 o;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
    h[0] = __floats2bfloat162_rn(a.x, a.y);
    h[1] = __floats2bfloat162_rn(a.z, a.w);
    h[2] = __floats2bfloat162_rn(b.x, b.y);
    h[3] = __floats2bfloat162_rn(b.z, b.w);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(sg.dst) + r * sg.ld_dst + c) = o;
}

unsigned blocks_for(int64_t threads) { return (unsigned)((threads + 255) / 256); }
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace r97b

using namespace r97b;

extern "C" int r97b_conv_prep_fwd(const uint16_t* x, int64_t ldx, const float* conv_w, const int32_t* cu, int32_t n_seq,
                                  int64_t T, int32_t Hg, int32_t H, uint16_t* q, uint16_t* k, uint16_t* v,
                                  void* stream) {
    if (!x || !conv_w || !cu || !q || !k || !v || T <= 0 || Hg <= 0 || H <= 0 || (ldx % 8) || !al16(x)) return R97B_EINVAL;
    ConvArgs a{reinterpret_cast<const __nv_bfloat16*>(x), ldx, conv_w, cu, n_seq, (int)T, Hg, H, (2 * Hg + H) * 128};
    conv_prep_fwd_kernel<<<blocks_for(((T + kRunF - 1) / kRunF) * (a.conv_dim / 4)), 256, 0, as_stream(stream)>>>(
        a, reinterpret_cast<__nv_bfloat16*>(q), reinterpret_cast<__nv_bfloat16*>(k), reinterpret_cast<__nv_bfloat16*>(v));
    return launch_status();
}

extern "C" int r97b_conv_prep_bwd(const uint16_t* x, int64_t ldx, const float* conv_w, const int32_t* cu,
                                  int32_t n_seq, int64_t T, int32_t Hg, int32_t H, const float* dq, const float* dk,
                                  const float* dv, int32_t dqk_heads, uint16_t* dx, int64_t lddx, void* stream) {
    if (!x || !conv_w || !cu || !dq || !dk || !dv || !dx || T <= 0 || (ldx % 4) || (lddx % 4)) return R97B_EINVAL;
    if (Hg <= 0 || H <= 0 || dqk_heads < Hg || dqk_heads % Hg) return R97B_EINVAL;
    ConvArgs a{reinterpret_cast<const __nv_bfloat16*>(x), ldx, conv_w, cu, n_seq, (int)T, Hg, H, (2 * Hg + H) * 128};
    if (n_seq <= 0) return R97B_EINVAL;
    if ((reinterpret_cast<uintptr_t>(dq) | reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv)) & 15)
        return R97B_EINVAL;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dx)) & 7) return R97B_EINVAL;
    ConvBwdArgs b{dq, dk, dv, dqk_heads / Hg, 0, reinterpret_cast<__nv_bfloat16*>(dx), lddx};
    const int64_t tiles = ((T + kConvTT - 1) / kConvTT) * (a.conv_dim / 128);
    if (tiles > INT32_MAX) return R97B_EINVAL;
    b.n_tiles = (int)tiles;
    const int smem = 2 * conv_stage(b.grp).bytes;
    if (smem > 227 * 1024) return R97B_EINVAL;
    int per_sm = 0;
    if (!smem_opt_in(conv_prep_bwd_kernel, smem) ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, conv_prep_bwd_kernel, 256, smem) != cudaSuccess ||
        per_sm < 1)
        return R97B_ELAUNCH;
    const unsigned grid = (unsigned)std::min<int64_t>(b.n_tiles, (int64_t)r97b::num_sms() * per_sm);
    conv_prep_bwd_kernel<<<grid, 256, smem, as_stream(stream)>>>(a, b);
    return launch_status();
}

extern "C" int r97b_gates_fwd(const uint16_t* ba, int64_t ldba, const float* a_log, const float* dt_bias,
                              const int32_t* chunk_tok0, const int32_t* chunk_len, int32_t n_chunks, int32_t H, float* g,
                              float* beta, void* stream) {
    if (!ba || !a_log || !dt_bias || !chunk_tok0 || !chunk_len || !g || !beta || H <= 0) return R97B_EINVAL;
    if (n_chunks <= 0) return R97B_OK;
    gates_fwd_kernel<<<dim3((unsigned)n_chunks, (unsigned)((H + 31) / 32)), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const __nv_bfloat16*>(ba), ldba, a_log, dt_bias, chunk_tok0, chunk_len, n_chunks, H, g, beta);
    return launch_status();
}

extern "C" int r97b_gates_bwd(const uint16_t* ba, int64_t ldba, const float* a_log, const float* dt_bias,
                              const int32_t* chunk_tok0, const int32_t* chunk_len, int32_t n_chunks, int32_t H,
                              const float* dg, const float* dbeta, uint16_t* dba, int64_t lddba, void* stream) {
    if (!ba || !a_log || !dt_bias || !chunk_tok0 || !chunk_len || !dg || !dbeta || !dba || H <= 0) return R97B_EINVAL;
    if (n_chunks <= 0) return R97B_OK;
    gates_bwd_kernel<<<dim3((unsigned)n_chunks, (unsigned)((H + 31) / 32)), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const __nv_bfloat16*>(ba), ldba, a_log, dt_bias, chunk_tok0, chunk_len, n_chunks, H, dg, dbeta,
        reinterpret_cast<__nv_bfloat16*>(dba), lddba);
    return launch_status();
}

extern "C" int r97b_swiglu_fwd(const uint16_t* gu, int64_t ldgu, int64_t rows, int64_t n, uint16_t* y, int64_t ldy,
                               void* stream) {
    if (!gu || !y || rows <= 0 || n <= 0 || n % 8 || ldgu % 8 || ldy % 8 || !al16(gu) || !al16(y)) return R97B_EINVAL;
    swiglu_fwd_kernel<<<blocks_for(rows * (n / 8)), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const __nv_bfloat16*>(gu), ldgu, rows, (int)n, reinterpret_cast<__nv_bfloat16*>(y), ldy);
    return launch_status();
}

extern "C" int r97b_swiglu_bwd(const uint16_t* gu, int64_t ldgu, int64_t rows, int64_t n, const uint16_t* dy,
                               int64_t lddy, uint16_t* dgu, int64_t lddgu, void* stream) {
    if (!gu || !dy || !dgu || rows <= 0 || n <= 0 || n % 8 || ldgu % 8 || lddy % 8 || lddgu % 8) return R97B_EINVAL;
    swiglu_bwd_kernel<<<blocks_for(rows * (n / 8)), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const __nv_bfloat16*>(gu), ldgu, rows, (int)n, reinterpret_cast<const __nv_bfloat16*>(dy), lddy,
        reinterpret_cast<__nv_bfloat16*>(dgu), lddgu);
    return launch_status();
}

namespace {
// head_dim 128 or 256; the rotated width a whole number of lanes whose count, and its pairing partner, a
// power of two (rot / 2 / (head_dim / 32) in {1, 2, 4, 8, 16})
bool qk_shape_ok(int32_t head_dim, int32_t rot) {
    if (head_dim != 128 && head_dim != 256) return false;
    const int nv = head_dim / 32;
    if (rot <= 0 || rot > head_dim || rot % (2 * nv)) return false;
    const int pl = rot / 2 / nv;
    return (pl & (pl - 1)) == 0 && pl <= 16;
}
}  // namespace

extern "C" int r97b_qk_norm_rope_fwd(const uint16_t* x, int64_t row_stride, int32_t head_stride, int32_t heads,
                                     int32_t head_dim, const float* w, const float* cos_tab, const float* sin_tab,
                                     int32_t rot, int64_t T, int32_t S, float eps, uint16_t* out, void* stream) {
    if (!x || !w || !cos_tab || !sin_tab || !out || T <= 0 || S <= 0 || T % S || !qk_shape_ok(head_dim, rot) ||
        head_stride % 8 || row_stride % 8)
        return R97B_EINVAL;
    QkArgs a{reinterpret_cast<const __nv_bfloat16*>(x), row_stride, head_stride, heads, w, cos_tab, sin_tab, rot,
             (int)T, S, eps};
    if (head_dim == 256)
        qk_norm_rope_fwd_kernel<8><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(
            a, reinterpret_cast<__nv_bfloat16*>(out));
    else
        qk_norm_rope_fwd_kernel<4><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(
            a, reinterpret_cast<__nv_bfloat16*>(out));
    return launch_status();
}

extern "C" int r97b_qk_norm_rope_bwd(const uint16_t* x, int64_t row_stride, int32_t head_stride, int32_t heads,
                                     int32_t head_dim, const float* w, const float* cos_tab, const float* sin_tab,
                                     int32_t rot, int64_t T, int32_t S, float eps, const uint16_t* dout, uint16_t* dx,
                                     int64_t dx_stride, void* stream) {
    if (!x || !w || !cos_tab || !sin_tab || !dout || !dx || T <= 0 || S <= 0 || T % S ||
        !qk_shape_ok(head_dim, rot) || head_stride % 8 || row_stride % 8 || dx_stride % 8)
        return R97B_EINVAL;
    QkArgs a{reinterpret_cast<const __nv_bfloat16*>(x), row_stride, head_stride, heads, w, cos_tab, sin_tab, rot,
             (int)T, S, eps};
    if (head_dim == 256)
        qk_norm_rope_bwd_kernel<8><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(
            a, reinterpret_cast<const __nv_bfloat16*>(dout), reinterpret_cast<__nv_bfloat16*>(dx), dx_stride);
    else
        qk_norm_rope_bwd_kernel<4><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(
            a, reinterpret_cast<const __nv_bfloat16*>(dout), reinterpret_cast<__nv_bfloat16*>(dx), dx_stride);
    return launch_status();
}

extern "C" int r97b_to_bhsd(const uint16_t* x, int64_t row_stride, int32_t head_stride, int32_t heads,
                            int32_t head_dim, int64_t T, int32_t S, uint16_t* out, int32_t reverse, void* stream) {
    if (!x || !out || T <= 0 || S <= 0 || T % S || head_stride % 8 || row_stride % 8 ||
        (head_dim != 128 && head_dim != 256))
        return R97B_EINVAL;
    const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x);
    auto* op = reinterpret_cast<__nv_bfloat16*>(out);
    if (head_dim == 256)
        to_bhsd_kernel<8><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(xp, row_stride, head_stride, heads,
                                                                                   (int)T, S, op, reverse);
    else
        to_bhsd_kernel<4><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(xp, row_stride, head_stride, heads,
                                                                                   (int)T, S, op, reverse);
    return launch_status();
}

extern "C" int r97b_gate_mul_fwd(const uint16_t* attn, const uint16_t* gate, int64_t gate_stride, int32_t gate_hs,
                                 int32_t heads, int32_t head_dim, int64_t T, int32_t S, uint16_t* y, void* stream) {
    if (!attn || !gate || !y || T <= 0 || S <= 0 || T % S || (head_dim != 128 && head_dim != 256) ||
        gate_stride % 8 || gate_hs % 8)
        return R97B_EINVAL;
    const auto* ap = reinterpret_cast<const __nv_bfloat16*>(attn);
    const auto* gp = reinterpret_cast<const __nv_bfloat16*>(gate);
    auto* yp = reinterpret_cast<__nv_bfloat16*>(y);
    if (head_dim == 256)
        gate_mul_fwd_kernel<8><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(ap, gp, gate_stride, gate_hs,
                                                                                        heads, (int)T, S, yp);
    else
        gate_mul_fwd_kernel<4><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(ap, gp, gate_stride, gate_hs,
                                                                                        heads, (int)T, S, yp);
    return launch_status();
}

extern "C" int r97b_gate_mul_bwd(const uint16_t* attn, const uint16_t* gate, int64_t gate_stride, int32_t gate_hs,
                                 int32_t heads, int32_t head_dim, int64_t T, int32_t S, const uint16_t* dy,
                                 uint16_t* dattn, uint16_t* dgate, int64_t dgate_stride, void* stream) {
    if (!attn || !gate || !dy || !dattn || !dgate || T <= 0 || S <= 0 || T % S ||
        (head_dim != 128 && head_dim != 256) || gate_stride % 8 || gate_hs % 8 || dgate_stride % 8)
        return R97B_EINVAL;
    const auto* ap = reinterpret_cast<const __nv_bfloat16*>(attn);
    const auto* gp = reinterpret_cast<const __nv_bfloat16*>(gate);
    const auto* dp = reinterpret_cast<const __nv_bfloat16*>(dy);
    auto* dap = reinterpret_cast<__nv_bfloat16*>(dattn);
    auto* dgp = reinterpret_cast<__nv_bfloat16*>(dgate);
    if (head_dim == 256)
        gate_mul_bwd_kernel<8><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(
            ap, gp, gate_stride, gate_hs, heads, (int)T, S, dp, dap, dgp, dgate_stride);
    else
        gate_mul_bwd_kernel<4><<<blocks_for(T * heads * 32), 256, 0, as_stream(stream)>>>(
            ap, gp, gate_stride, gate_hs, heads, (int)T, S, dp, dap, dgp, dgate_stride);
    return launch_status();
}

extern "C" int r97b_embed(const uint16_t* table, int64_t ld, int64_t vocab, const int32_t* ids, int64_t T, int64_t n,
                          uint16_t* out, void* stream) {
    if (!table || !ids || !out || T <= 0 || n % 8 || ld % 8) return R97B_EINVAL;
    embed_kernel<<<blocks_for(T * (n / 8)), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const __nv_bfloat16*>(table), ld, vocab, ids, T, (int)n, reinterpret_cast<__nv_bfloat16*>(out));
    return launch_status();
}

extern "C" int r97b_cast_f32_bf16(const float* src, int64_t ld_src, uint16_t* dst, int64_t ld_dst, int64_t rows,
                                  int64_t cols, void* stream) {
    if (!src || !dst || rows <= 0 || cols <= 0) return R97B_EINVAL;
    cast_2d_kernel<<<blocks_for(rows * cols), 256, 0, as_stream(stream)>>>(src, ld_src,
                                                                         reinterpret_cast<__nv_bfloat16*>(dst), ld_dst,
                                                                         rows, cols);
    return launch_status();
}

extern "C" int r97b_cast_segments(const R97bCastSeg* segs, int32_t nseg, int64_t units, void* stream) {
    if (!segs || nseg <= 0 || units <= 0) return R97B_EINVAL;
    cast_segments_kernel<<<blocks_for(units), 256, 0, as_stream(stream)>>>(segs, nseg, units);
    return launch_status();
}
