// gdn.cu -- the chunked GatedDeltaNet recurrence, forward and backward, on sm_100a.
//
// It computes the reference's two ops as one path (reference src/adjoint/host/gdn_kkt.cpp and
// gdn_scan.cpp; docs/adjoints/gdn-math.md s2.2, s3, s4):
//   gdn_kkt_solve : A = (I + M)^-1, M[i,l] = beta_i (k_i . k_l) e^{g_i - g_l} (l < i), per chunk of 64
//   gdn_chunk_scan: W = beta (v - e^g k S), V' = A W, o = scale (e^g q S + causal(q k^T e^{g_i-g_j}) V'),
//                   S_next = e^{g_L} S + sum_j e^{g_L - g_j} k_j (x) V'_j
// with the state held as S[d][e] (key lane d, value lane e; the reference's transposed St) in f32 and
// g the within-chunk cumulative log decay. Rewriting V' = u - w S with u = A diag(beta) v and
// w = A diag(beta e^g) k moves every intra-chunk product into chunk-parallel kernels and leaves a short
// sequential pass whose value lanes are independent:
//
//   F1 gdn_fwd_prep  (chunk, head)        M, A by forward substitution, w, u
//   F2 gdn_fwd_state (seq, head, V/32)    S_c entering each chunk, V'_c = u_c - w_c S_c, S_{c+1}
//   F3 gdn_fwd_out   (chunk, head)        P = causal(q k^T e^{g_i-g_j}), o = scale (e^g q S_c + P V'_c)
//   B1 gdn_bwd_state (seq, head, V/32)    reverse pass: dV' = scale P^T dO + K~ dS_next,
//                                          dS = scale Q~^T dO + e^{g_L} dS_next - w^T dV'
//   B2a gdn_bwd_a    (chunk, head)        the terms that read the states: dQ~ = scale dO S^T, dw = -dV' S^T,
//                                          dK~ = V' dS_next^T, and dg_L's e^{g_L} <S, dS_next>
//   B2b gdn_bwd_b    (chunk, head)        the intra-chunk terms: dP, dA = dw kb^T + dV' vb^T, A^T dw, A^T dV',
//                                          and the solve's adjoint dM = -A^T dA A^T (the kkt adjoint)
//
// Sequences are ragged (cu_seqlens); a sequence's last chunk may be short, and its padded rows are zero
// so they add nothing. Head dims K = V = 128 and the chunk of 64 are fixed here.
#include "blockmm.cuh"
#include "r97b_internal.h"

#include <cuda_bf16.h>
#include <math.h>

namespace r97b {
namespace {

constexpr int D = 128;       // key / value head dim
constexpr int L = 64;        // chunk
constexpr int P129 = D + 1;  // f32 pitch of a [*, 128] tile
constexpr int P65 = L + 1;   // f32 pitch of a [64, 64] tile
constexpr int P33 = 33;      // f32 pitch of a [*, 32] value slice
constexpr int VS = 32;       // value lanes per sequential CTA

struct Dims {
    int n_seq, H, Hg, grp, n_chunks;
    float scale;
    const int* tok0;
    const int* len;
    const int* seq_c0;
};

__device__ __forceinline__ float bf(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// rows [0, 64) x 128 of a token-major bf16 tensor [T, heads, 128] for one head; zero past `n` rows
__device__ __forceinline__ void load_rows_bf16(float* dst, const __nv_bfloat16* src, int64_t tok0, int n, int heads,
                                               int head, float scale = 1.0f) {
    for (int idx = threadIdx.x; idx < L * D; idx += blockDim.x) {
        const int i = idx >> 7, d = idx & 127;
        dst[i * P129 + d] = i < n ? scale * bf(src + ((tok0 + i) * heads + head) * D + d) : 0.0f;
    }
}

__device__ __forceinline__ void load_rows_f32(float* dst, const float* src, int64_t tok0, int n, int heads, int head,
                                              float scale = 1.0f) {
    for (int idx = threadIdx.x; idx < L * D; idx += blockDim.x) {
        const int i = idx >> 7, d = idx & 127;
        dst[i * P129 + d] = i < n ? scale * src[((tok0 + i) * heads + head) * D + d] : 0.0f;
    }
}

// the value slice [e0, e0 + 32) of rows [0, 64) of a [T, H, 128] tensor
template <typename T>
__device__ __forceinline__ void load_slice(float* dst, const T* src, int64_t tok0, int n, int H, int h, int e0,
                                           float scale = 1.0f) {
    for (int idx = threadIdx.x; idx < L * VS; idx += blockDim.x) {
        const int i = idx >> 5, e = idx & 31;
        dst[i * P33 + e] = i < n ? scale * ld_f32(src + ((tok0 + i) * H + h) * D + e0 + e) : 0.0f;
    }
}

__device__ __forceinline__ void load_gb(float* gs, float* bs, const float* g, const float* beta, int64_t tok0, int n,
                                        int H, int h) {
    for (int i = threadIdx.x; i < L; i += blockDim.x) {
        gs[i] = i < n ? g[(tok0 + i) * H + h] : 0.0f;
        if (bs) bs[i] = i < n ? beta[(tok0 + i) * H + h] : 0.0f;
    }
}

// sum over the 16 threads of one row group (lanes sharing ty: a half warp)
__device__ __forceinline__ float row16_sum(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// ============================================================================================ forward

// F1: per (chunk, value head): A = (I + M)^-1, w = A diag(beta e^g) k, u = A diag(beta) v.
__global__ void __launch_bounds__(256) gdn_fwd_prep(Dims dm, const __nv_bfloat16* __restrict__ q_unused,
                                                    const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                                                    const float* __restrict__ g, const float* __restrict__ beta,
                                                    float* __restrict__ A, float* __restrict__ w, float* __restrict__ u) {
    extern __shared__ float sm[];
    float* ks = sm;                  // [64][129]
    float* vs = ks + L * P129;       // [64][129]
    float* Ms = vs + L * P129;       // [64][65]
    float* As = Ms + L * P65;        // [64][65]
    float* red = As + L * P65;       // [4][64]
    float* gs = red + 4 * L;         // [64]
    float* bs = gs + L;              // [64]
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    load_rows_bf16(ks, k, tok0, n, dm.Hg, hk);
    load_rows_bf16(vs, v, tok0, n, dm.H, h);
    load_gb(gs, bs, g, beta, tok0, n, dm.H, h);
    __syncthreads();
    {
        float acc[4][4];
        zero_acc<64, 64>(acc);
        bmm<64, 64, 128, false, true>(acc, ks, P129, ks, P129);
        const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = ty + 16 * i, l = tx + 16 * j;
                Ms[r * P65 + l] = l < r ? bs[r] * acc[i][j] * expf(gs[r] - gs[l]) : 0.0f;
            }
    }
    __syncthreads();
    // forward substitution, one row at a time: A[i][j] = delta_ij - sum_{l<i} M[i][l] A[l][j]
    {
        const int j = threadIdx.x & 63, part = threadIdx.x >> 6;
        for (int i = 0; i < L; ++i) {
            float s = 0.0f;
            const int l0 = part * 16;
#pragma unroll
            for (int l = l0; l < l0 + 16; ++l)
                if (l < i) s = fmaf(Ms[i * P65 + l], As[l * P65 + j], s);
            red[part * L + j] = s;
            __syncthreads();
            if (part == 0) {
                const float t = red[j] + red[L + j] + red[2 * L + j] + red[3 * L + j];
                As[i * P65 + j] = j < i ? -t : (j == i ? 1.0f : 0.0f);
            }
            __syncthreads();
        }
    }
    for (int idx = threadIdx.x; idx < L * L; idx += blockDim.x) {
        const int i = idx >> 6, j = idx & 63;
        if (i < n) A[((tok0 + i) * dm.H + h) * L + j] = As[i * P65 + j];
    }
    // kb = diag(beta e^g) k, vb = diag(beta) v, in place
    for (int idx = threadIdx.x; idx < L * D; idx += blockDim.x) {
        const int i = idx >> 7, d = idx & 127;
        ks[i * P129 + d] *= bs[i] * expf(gs[i]);
        vs[i * P129 + d] *= bs[i];
    }
    __syncthreads();
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    float acc[4][8];
    zero_acc<64, 128>(acc);
    bmm<64, 128, 64, false, false>(acc, As, P65, ks, P129);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = ty + 16 * i;
            if (r < n) w[((tok0 + r) * dm.H + h) * D + tx + 16 * j] = acc[i][j];
        }
    zero_acc<64, 128>(acc);
    bmm<64, 128, 64, false, false>(acc, As, P65, vs, P129);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = ty + 16 * i;
            if (r < n) u[((tok0 + r) * dm.H + h) * D + tx + 16 * j] = acc[i][j];
        }
}

// F2: per (sequence, value head, 32 value lanes): the state pass over the sequence's chunks.
__global__ void __launch_bounds__(256) gdn_fwd_state(Dims dm, const __nv_bfloat16* __restrict__ k,
                                                     const float* __restrict__ g, const float* __restrict__ w,
                                                     const float* __restrict__ u, const float* __restrict__ h0,
                                                     float* __restrict__ S_all, float* __restrict__ Vp,
                                                     float* __restrict__ ht) {
    extern __shared__ float sm[];
    float* Ss = sm;                  // [128][33]
    float* ws = Ss + D * P33;        // [64][129]
    float* ks = ws + L * P129;       // [64][129]
    float* us = ks + L * P129;       // [64][33]
    float* gs = us + L * P33;        // [64]
    const int seq = blockIdx.x, h = blockIdx.y, e0 = blockIdx.z * VS, hk = h / dm.grp;
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    for (int idx = threadIdx.x; idx < D * VS; idx += blockDim.x) {
        const int d = idx >> 5, e = idx & 31;
        Ss[d * P33 + e] = h0 ? h0[(((int64_t)seq * dm.H + h) * D + e0 + e) * D + d] : 0.0f;
    }
    const int c0 = dm.seq_c0[seq], c1 = dm.seq_c0[seq + 1];
    for (int c = c0; c < c1; ++c) {
        const int64_t tok0 = dm.tok0[c];
        const int n = dm.len[c];
        __syncthreads();
        float* Sg = S_all + ((int64_t)c * dm.H + h) * D * D;
        for (int idx = threadIdx.x; idx < D * VS; idx += blockDim.x) {
            const int d = idx >> 5, e = idx & 31;
            Sg[d * D + e0 + e] = Ss[d * P33 + e];
        }
        load_rows_f32(ws, w, tok0, n, dm.H, h);
        load_rows_bf16(ks, k, tok0, n, dm.Hg, hk);
        load_slice(us, u, tok0, n, dm.H, h, e0);
        load_gb(gs, nullptr, g, nullptr, tok0, n, dm.H, h);
        __syncthreads();
        {
            float acc[4][2];
            zero_acc<64, 32>(acc);
            bmm<64, 32, 128, false, false>(acc, ws, P129, Ss, P33);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int r = ty + 16 * i, e = tx + 16 * j;
                    const float vp = us[r * P33 + e] - acc[i][j];
                    us[r * P33 + e] = vp;
                    if (r < n) Vp[((tok0 + r) * dm.H + h) * D + e0 + e] = vp;
                }
        }
        const float gl = gs[n - 1];
        for (int idx = threadIdx.x; idx < L * D; idx += blockDim.x) {
            const int i = idx >> 7, d = idx & 127;
            ks[i * P129 + d] *= i < n ? expf(gl - gs[i]) : 0.0f;
        }
        __syncthreads();
        {
            float acc[8][2];
            zero_acc<128, 32>(acc);
            bmm<128, 32, 64, true, false>(acc, ks, P129, us, P33);
            const float el = expf(gl);
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int d = ty + 16 * i, e = tx + 16 * j;
                    Ss[d * P33 + e] = el * Ss[d * P33 + e] + acc[i][j];
                }
        }
    }
    __syncthreads();
    if (ht)
        for (int idx = threadIdx.x; idx < D * VS; idx += blockDim.x) {
            const int d = idx >> 5, e = idx & 31;
            ht[(((int64_t)seq * dm.H + h) * D + e0 + e) * D + d] = Ss[d * P33 + e];
        }
}

// F3: per (chunk, value head): P and the output rows.
__global__ void __launch_bounds__(256) gdn_fwd_out(Dims dm, const __nv_bfloat16* __restrict__ q,
                                                   const __nv_bfloat16* __restrict__ k, const float* __restrict__ g,
                                                   const float* __restrict__ S_all, const float* __restrict__ Vp,
                                                   float* __restrict__ P_all, __nv_bfloat16* __restrict__ o) {
    extern __shared__ float sm[];
    float* qs = sm;                  // [64][129]
    float* ks = qs + L * P129;       // [64][129]  k, then V'
    float* Ps = ks + L * P129;       // [64][65]
    float* Ss = Ps + L * P65;        // [128][129]
    float* gs = Ss + D * P129;       // [64]
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    load_rows_bf16(qs, q, tok0, n, dm.Hg, hk);
    load_rows_bf16(ks, k, tok0, n, dm.Hg, hk);
    load_gb(gs, nullptr, g, nullptr, tok0, n, dm.H, h);
    const float* Sg = S_all + ((int64_t)c * dm.H + h) * D * D;
    for (int idx = threadIdx.x; idx < D * D; idx += blockDim.x) Ss[(idx >> 7) * P129 + (idx & 127)] = Sg[idx];
    __syncthreads();
    {
        float acc[4][4];
        zero_acc<64, 64>(acc);
        bmm<64, 64, 128, false, true>(acc, qs, P129, ks, P129);
        float* Pg = P_all + ((int64_t)c * dm.H + h) * L * L;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = ty + 16 * i, l = tx + 16 * j;
                const float p = (l <= r && r < n) ? acc[i][j] * expf(gs[r] - gs[l]) : 0.0f;
                Ps[r * P65 + l] = p;
                Pg[r * L + l] = p;
            }
    }
    __syncthreads();
    load_rows_f32(ks, Vp, tok0, n, dm.H, h);
    for (int idx = threadIdx.x; idx < L * D; idx += blockDim.x) {
        const int i = idx >> 7, d = idx & 127;
        qs[i * P129 + d] *= expf(gs[i]);
    }
    __syncthreads();
    float acc[4][8];
    zero_acc<64, 128>(acc);
    bmm<64, 128, 128, false, false>(acc, qs, P129, Ss, P129);
    bmm<64, 128, 64, false, false>(acc, Ps, P65, ks, P129);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = ty + 16 * i;
            if (r < n) o[((tok0 + r) * dm.H + h) * D + tx + 16 * j] = __float2bfloat16_rn(dm.scale * acc[i][j]);
        }
}

// ============================================================================================ backward

// B1: per (sequence, value head, 32 value lanes): the reverse state pass.
__global__ void __launch_bounds__(256) gdn_bwd_state(Dims dm, const __nv_bfloat16* __restrict__ q,
                                                     const __nv_bfloat16* __restrict__ k, const float* __restrict__ g,
                                                     const float* __restrict__ w, const float* __restrict__ P_all,
                                                     const __nv_bfloat16* __restrict__ dO, const float* __restrict__ dht,
                                                     float* __restrict__ dS_all, float* __restrict__ dVp,
                                                     float* __restrict__ dh0) {
    extern __shared__ float sm[];
    float* dSs = sm;                 // [128][33]
    float* Ps = dSs + D * P33;       // [64][65]
    float* Kt = Ps + L * P65;        // [64][129]
    float* Qt = Kt + L * P129;       // [64][129]
    float* ws = Qt + L * P129;       // [64][129]
    float* dOs = ws + L * P129;      // [64][33]
    float* dVs = dOs + L * P33;      // [64][33]
    float* gs = dVs + L * P33;       // [64]
    const int seq = blockIdx.x, h = blockIdx.y, e0 = blockIdx.z * VS, hk = h / dm.grp;
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    for (int idx = threadIdx.x; idx < D * VS; idx += blockDim.x) {
        const int d = idx >> 5, e = idx & 31;
        dSs[d * P33 + e] = dht ? dht[(((int64_t)seq * dm.H + h) * D + e0 + e) * D + d] : 0.0f;
    }
    const int c0 = dm.seq_c0[seq], c1 = dm.seq_c0[seq + 1];
    for (int c = c1 - 1; c >= c0; --c) {
        const int64_t tok0 = dm.tok0[c];
        const int n = dm.len[c];
        __syncthreads();
        float* dSg = dS_all + ((int64_t)c * dm.H + h) * D * D;
        for (int idx = threadIdx.x; idx < D * VS; idx += blockDim.x) {
            const int d = idx >> 5, e = idx & 31;
            dSg[d * D + e0 + e] = dSs[d * P33 + e];
        }
        load_gb(gs, nullptr, g, nullptr, tok0, n, dm.H, h);
        const float* Pg = P_all + ((int64_t)c * dm.H + h) * L * L;
        for (int idx = threadIdx.x; idx < L * L; idx += blockDim.x) Ps[(idx >> 6) * P65 + (idx & 63)] = Pg[idx];
        load_rows_bf16(Kt, k, tok0, n, dm.Hg, hk);
        load_rows_bf16(Qt, q, tok0, n, dm.Hg, hk);
        load_rows_f32(ws, w, tok0, n, dm.H, h);
        load_slice(dOs, dO, tok0, n, dm.H, h, e0, dm.scale);
        __syncthreads();
        const float gl = gs[n - 1];
        for (int idx = threadIdx.x; idx < L * D; idx += blockDim.x) {
            const int i = idx >> 7, d = idx & 127;
            Kt[i * P129 + d] *= i < n ? expf(gl - gs[i]) : 0.0f;
            Qt[i * P129 + d] *= expf(gs[i]);
        }
        __syncthreads();
        {
            float acc[4][2];
            zero_acc<64, 32>(acc);
            bmm<64, 32, 64, true, false>(acc, Ps, P65, dOs, P33);
            bmm<64, 32, 128, false, false>(acc, Kt, P129, dSs, P33);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int r = ty + 16 * i, e = tx + 16 * j;
                    const float dv = r < n ? acc[i][j] : 0.0f;
                    dVs[r * P33 + e] = dv;
                    if (r < n) dVp[((tok0 + r) * dm.H + h) * D + e0 + e] = dv;
                }
        }
        __syncthreads();
        {
            float acc[8][2], wt[8][2];
            zero_acc<128, 32>(acc);
            zero_acc<128, 32>(wt);
            bmm<128, 32, 64, true, false>(acc, Qt, P129, dOs, P33);
            bmm<128, 32, 64, true, false>(wt, ws, P129, dVs, P33);
            const float el = expf(gl);
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int d = ty + 16 * i, e = tx + 16 * j;
                    dSs[d * P33 + e] = acc[i][j] + el * dSs[d * P33 + e] - wt[i][j];
                }
        }
    }
    __syncthreads();
    if (dh0)
        for (int idx = threadIdx.x; idx < D * VS; idx += blockDim.x) {
            const int d = idx >> 5, e = idx & 31;
            dh0[(((int64_t)seq * dm.H + h) * D + e0 + e) * D + d] = dSs[d * P33 + e];
        }
}

// B2a: per (chunk, value head): the state-reading terms.
__global__ void __launch_bounds__(256) gdn_bwd_a(Dims dm, const __nv_bfloat16* __restrict__ q,
                                                 const __nv_bfloat16* __restrict__ k, const float* __restrict__ g,
                                                 const float* __restrict__ S_all, const float* __restrict__ Vp,
                                                 const __nv_bfloat16* __restrict__ dO, const float* __restrict__ dS_all,
                                                 const float* __restrict__ dVp, float* __restrict__ dw,
                                                 float* __restrict__ pdq, float* __restrict__ pdk,
                                                 float* __restrict__ pdg) {
    extern __shared__ float sm[];
    float* Ss = sm;                  // [128][129]  S, then dS_next
    float* X1 = Ss + D * P129;       // [64][129]   scale dO, then V'
    float* X2 = X1 + L * P129;       // [64][129]   q, then k
    float* X3 = X2 + L * P129;       // [64][129]   dV'
    float* gs = X3 + L * P129;       // [64]
    float* dgs = gs + L;             // [64]
    float* red = dgs + L;            // [8]
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    const float* Sg = S_all + ((int64_t)c * dm.H + h) * D * D;
    for (int idx = threadIdx.x; idx < D * D; idx += blockDim.x) Ss[(idx >> 7) * P129 + (idx & 127)] = Sg[idx];
    load_rows_bf16(X1, dO, tok0, n, dm.H, h, dm.scale);
    load_rows_bf16(X2, q, tok0, n, dm.Hg, hk);
    load_rows_f32(X3, dVp, tok0, n, dm.H, h);
    load_gb(gs, nullptr, g, nullptr, tok0, n, dm.H, h);
    for (int i = threadIdx.x; i < L; i += blockDim.x) dgs[i] = 0.0f;
    __syncthreads();
    float dq[4][8];
    {
        // dQ~ = (scale dO) S^T ; dq = e^g dQ~ ; dg_i += e^{g_i} q_i . dQ~_i
        zero_acc<64, 128>(dq);
        bmm<64, 128, 128, false, true>(dq, X1, P129, Ss, P129);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 16 * i;
            const float eg = expf(gs[r]);
            float part = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                dq[i][j] *= eg;
                part = fmaf(X2[r * P129 + tx + 16 * j], dq[i][j], part);
            }
            part = row16_sum(part);
            if (tx == 0) dgs[r] += part;
        }
    }
    {
        // dw = -dV' S^T
        float acc[4][8];
        zero_acc<64, 128>(acc);
        bmm<64, 128, 128, false, true>(acc, X3, P129, Ss, P129);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int r = ty + 16 * i;
                if (r < n) dw[((tok0 + r) * dm.H + h) * D + tx + 16 * j] = -acc[i][j];
            }
    }
    __syncthreads();
    // <S, dS_next>, replacing S by dS_next in place
    const float* dSg = dS_all + ((int64_t)c * dm.H + h) * D * D;
    float sdot = 0.0f;
    for (int idx = threadIdx.x; idx < D * D; idx += blockDim.x) {
        float* p = Ss + (idx >> 7) * P129 + (idx & 127);
        const float ds = dSg[idx];
        sdot = fmaf(*p, ds, sdot);
        *p = ds;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sdot += __shfl_xor_sync(0xFFFFFFFFu, sdot, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sdot;
    load_rows_f32(X1, Vp, tok0, n, dm.H, h);
    load_rows_bf16(X2, k, tok0, n, dm.Hg, hk);
    __syncthreads();
    const float gl = gs[n - 1];
    float dk[4][8];
    float tsum = 0.0f;
    {
        // dK~ = V' dS_next^T ; dk_j = e^{gL-gj} dK~_j ; dg_j -= K~_j . dK~_j ; dg_L += sum
        zero_acc<64, 128>(dk);
        bmm<64, 128, 128, false, true>(dk, X1, P129, Ss, P129);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 16 * i;
            const float f = r < n ? expf(gl - gs[r]) : 0.0f;
            float part = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                dk[i][j] *= f;
                part = fmaf(X2[r * P129 + tx + 16 * j], dk[i][j], part);
            }
            part = row16_sum(part);
            if (tx == 0) {
                dgs[r] -= part;
                tsum += part;
            }
        }
    }
    // tsum lives in the tx == 0 threads; gather it with the <S, dS_next> partials
    __shared__ float tred[16];
    if (tx == 0) tred[ty] = tsum;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f, t = 0.0f;
        for (int i = 0; i < 8; ++i) s += red[i];
        for (int i = 0; i < 16; ++i) t += tred[i];
        dgs[n - 1] += expf(gl) * s + t;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = ty + 16 * i;
            if (r < n) {
                const int64_t at = ((tok0 + r) * dm.H + h) * D + tx + 16 * j;
                pdq[at] = dq[i][j];
                pdk[at] = dk[i][j];
            }
        }
    for (int i = threadIdx.x; i < n; i += blockDim.x) pdg[(tok0 + i) * dm.H + h] = dgs[i];
}

// B2b: per (chunk, value head): the intra-chunk terms and the solve's adjoint; adds B2a's partials.
__global__ void __launch_bounds__(256) gdn_bwd_b(Dims dm, const __nv_bfloat16* __restrict__ q,
                                                 const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                                                 const float* __restrict__ g, const float* __restrict__ beta,
                                                 const float* __restrict__ A, const float* __restrict__ Vp,
                                                 const __nv_bfloat16* __restrict__ dO, const float* __restrict__ dVp,
                                                 const float* __restrict__ dw, const float* __restrict__ pdq,
                                                 const float* __restrict__ pdk, const float* __restrict__ pdg,
                                                 float* __restrict__ dq_out, float* __restrict__ dk_out,
                                                 float* __restrict__ dv_out, float* __restrict__ dbeta_out,
                                                 float* __restrict__ dg_out) {
    extern __shared__ float sm[];
    float* X1 = sm;                  // q, then v
    float* X2 = X1 + L * P129;       // k
    float* X3 = X2 + L * P129;       // scale dO, then dw, then Y = dA A^T (pitch 65)
    float* X4 = X3 + L * P129;       // V', then dV'
    float* T1 = X4 + L * P129;       // P^ (gated q k^T), then A
    float* T2 = T1 + L * P65;        // K^ = (k k^T) e^{g_i-g_l}, strict lower
    float* T3 = T2 + L * P65;        // gated dP, then dA, then E
    float* gs = T3 + L * P65;
    float* bs = gs + L;
    float* dgs = bs + L;
    float* dbs = dgs + L;
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
    load_rows_bf16(X1, q, tok0, n, dm.Hg, hk);
    load_rows_bf16(X2, k, tok0, n, dm.Hg, hk);
    load_rows_bf16(X3, dO, tok0, n, dm.H, h, dm.scale);
    load_rows_f32(X4, Vp, tok0, n, dm.H, h);
    load_gb(gs, bs, g, beta, tok0, n, dm.H, h);
    for (int i = threadIdx.x; i < L; i += blockDim.x) {
        dgs[i] = 0.0f;
        dbs[i] = 0.0f;
    }
    __syncthreads();
    {
        float acc[4][4];
        zero_acc<64, 64>(acc);
        bmm<64, 64, 128, false, true>(acc, X1, P129, X2, P129);  // q k^T
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = ty + 16 * i, l = tx + 16 * j;
                T1[r * P65 + l] = (l <= r && r < n) ? acc[i][j] * expf(gs[r] - gs[l]) : 0.0f;
            }
        zero_acc<64, 64>(acc);
        bmm<64, 64, 128, false, true>(acc, X2, P129, X2, P129);  // k k^T
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = ty + 16 * i, l = tx + 16 * j;
                T2[r * P65 + l] = (l < r && r < n) ? acc[i][j] * expf(gs[r] - gs[l]) : 0.0f;
            }
        // dP = (scale dO) V'^T, causal; D = dP * P^ -> dg ; gated dP -> T3
        zero_acc<64, 64>(acc);
        bmm<64, 64, 128, false, true>(acc, X3, P129, X4, P129);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 16 * i;
            float rowD = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int l = tx + 16 * j;
                const bool on = l <= r && r < n;
                const float dp = on ? acc[i][j] : 0.0f;
                const float dd = dp * T1[r * P65 + l];
                rowD += dd;
                if (on) atomicAdd(&dgs[l], -dd);
                T3[r * P65 + l] = on ? dp * expf(gs[r] - gs[l]) : 0.0f;
            }
            rowD = row16_sum(rowD);
            if (tx == 0) atomicAdd(&dgs[r], rowD);
        }
    }
    __syncthreads();
    float dqa[4][8], dka[4][8];
    zero_acc<64, 128>(dqa);
    zero_acc<64, 128>(dka);
    bmm<64, 128, 64, false, false>(dqa, T3, P65, X2, P129);  // dq += gated dP k
    bmm<64, 128, 64, true, false>(dka, T3, P65, X1, P129);   // dk += gated dP^T q
    __syncthreads();
    // v, dw, dV', A
    for (int idx = threadIdx.x; idx < L * D; idx += blockDim.x) {
        const int i = idx >> 7, d = idx & 127;
        const int64_t at = ((tok0 + i) * dm.H + h) * D + d;
        X1[i * P129 + d] = i < n ? __bfloat162float(v[at]) : 0.0f;
        X3[i * P129 + d] = i < n ? dw[at] : 0.0f;
        X4[i * P129 + d] = i < n ? dVp[at] : 0.0f;
    }
    for (int idx = threadIdx.x; idx < L * L; idx += blockDim.x) {
        const int i = idx >> 6, j = idx & 63;
        T1[i * P65 + j] = i < n ? A[((tok0 + i) * dm.H + h) * L + j] : 0.0f;
    }
    __syncthreads();
    {
        // dA = dw kb^T + dV' vb^T, strict lower ; kb_j = beta_j e^{g_j} k_j, vb_j = beta_j v_j
        float a1[4][4], a2[4][4];
        zero_acc<64, 64>(a1);
        zero_acc<64, 64>(a2);
        bmm<64, 64, 128, false, true>(a1, X3, P129, X2, P129);
        bmm<64, 64, 128, false, true>(a2, X4, P129, X1, P129);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = ty + 16 * i, l = tx + 16 * j;
                T3[r * P65 + l] = l < r ? bs[l] * (expf(gs[l]) * a1[i][j] + a2[i][j]) : 0.0f;
            }
    }
    {
        // dkb = A^T dw -> dk, dbeta, dg
        float acc[4][8];
        zero_acc<64, 128>(acc);
        bmm<64, 128, 64, true, false>(acc, T1, P65, X3, P129);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 16 * i;
            const float eg = expf(gs[r]), be = bs[r] * eg;
            float part = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                part = fmaf(X2[r * P129 + tx + 16 * j], acc[i][j], part);
                dka[i][j] = fmaf(be, acc[i][j], dka[i][j]);
            }
            part = row16_sum(part);
            if (tx == 0) {
                dbs[r] += eg * part;
                dgs[r] += be * part;
            }
        }
        // dvb = A^T dV' -> dv, dbeta
        zero_acc<64, 128>(acc);
        bmm<64, 128, 64, true, false>(acc, T1, P65, X4, P129);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 16 * i;
            float part = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                part = fmaf(X1[r * P129 + tx + 16 * j], acc[i][j], part);
                if (r < n) dv_out[((tok0 + r) * dm.H + h) * D + tx + 16 * j] = bs[r] * acc[i][j];
            }
            part = row16_sum(part);
            if (tx == 0) dbs[r] += part;
        }
    }
    __syncthreads();
    {
        // Y = dA A^T into X3 (pitch 65); dM = -A^T Y, strict lower
        float acc[4][4];
        zero_acc<64, 64>(acc);
        bmm<64, 64, 64, false, true>(acc, T3, P65, T1, P65);
        __syncthreads();
        store_acc<64, 64>(acc, X3, P65);
        __syncthreads();
        zero_acc<64, 64>(acc);
        bmm<64, 64, 64, true, false>(acc, T1, P65, X3, P65);
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 16 * i;
            float rowB = 0.0f, rowG = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int l = tx + 16 * j;
                const bool on = l < r && r < n;
                const float dm_ = on ? -acc[i][j] : 0.0f;
                const float kh = T2[r * P65 + l];
                rowB = fmaf(dm_, kh, rowB);
                const float gg = dm_ * bs[r] * kh;
                rowG += gg;
                if (on) atomicAdd(&dgs[l], -gg);
                T3[r * P65 + l] = on ? dm_ * bs[r] * expf(gs[r] - gs[l]) : 0.0f;
            }
            rowB = row16_sum(rowB);
            rowG = row16_sum(rowG);
            if (tx == 0) {
                dbs[r] += rowB;
                atomicAdd(&dgs[r], rowG);  // other threads add column terms to the same entries
            }
        }
    }
    __syncthreads();
    bmm<64, 128, 64, false, false>(dka, T3, P65, X2, P129);  // dk_i += sum_l E_il k_l
    bmm<64, 128, 64, true, false>(dka, T3, P65, X2, P129);   // dk_l += sum_i E_il k_i
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = ty + 16 * i;
            if (r < n) {
                const int64_t at = ((tok0 + r) * dm.H + h) * D + tx + 16 * j;
                dq_out[at] = dqa[i][j] + pdq[at];
                dk_out[at] = dka[i][j] + pdk[at];
            }
        }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int64_t at = (tok0 + i) * dm.H + h;
        dg_out[at] = dgs[i] + pdg[at];
        dbeta_out[at] = dbs[i];
    }
}

// dst[t, hk, :] = sum over the value heads hk * grp .. of src[t, h, :]
__global__ void gdn_sum_heads_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t T, int H, int Hg) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= T * Hg * D) return;
    const int d = idx % D;
    const int hk = (idx / D) % Hg;
    const int64_t t = idx / ((int64_t)D * Hg);
    const int grp = H / Hg;
    float s = 0.0f;
    for (int j = 0; j < grp; ++j) s += src[(t * H + hk * grp + j) * D + d];
    dst[idx] = s;
}

constexpr size_t kSmemPrep = (2 * L * P129 + 2 * L * P65 + 4 * L + 2 * L) * 4;
constexpr size_t kSmemState = (D * P33 + 2 * L * P129 + L * P33 + L) * 4;
constexpr size_t kSmemOut = (2 * L * P129 + L * P65 + D * P129 + L) * 4;
constexpr size_t kSmemBState = (D * P33 + L * P65 + 3 * L * P129 + 2 * L * P33 + L) * 4;
constexpr size_t kSmemBA = (D * P129 + 3 * L * P129 + 2 * L + 8) * 4;
constexpr size_t kSmemBB = (4 * L * P129 + 3 * L * P65 + 4 * L) * 4;

bool g_attr = false;

void set_attrs() {
    if (g_attr) return;
    cudaFuncSetAttribute(gdn_fwd_prep, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemPrep);
    cudaFuncSetAttribute(gdn_fwd_state, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemState);
    cudaFuncSetAttribute(gdn_fwd_out, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOut);
    cudaFuncSetAttribute(gdn_bwd_state, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBState);
    cudaFuncSetAttribute(gdn_bwd_a, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBA);
    cudaFuncSetAttribute(gdn_bwd_b, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBB);
    g_attr = true;
}

bool dims_ok(const R97bGdnDims& d) {
    return d.n_seq > 0 && d.H > 0 && d.Hg > 0 && d.H % d.Hg == 0 && d.n_chunks >= 0 && d.T >= 0 && d.chunk_tok0 &&
           d.chunk_len && d.seq_chunk0 && d.head_k == D && d.head_v == D && d.chunk == L;
}

Dims to_dims(const R97bGdnDims& d) {
    return Dims{d.n_seq, d.H, d.Hg, d.H / d.Hg, d.n_chunks, d.scale, d.chunk_tok0, d.chunk_len, d.seq_chunk0};
}

}  // namespace
}  // namespace r97b

using namespace r97b;

extern "C" int32_t r97b_gdn_chunk_table(const int32_t* cu_host, int32_t n_seq, int32_t chunk, int32_t* tok0_host,
                                        int32_t* len_host, int32_t* seq_chunk0_host) {
    if (!cu_host || n_seq <= 0 || chunk <= 0) return -1;
    int32_t c = 0;
    for (int32_t s = 0; s < n_seq; ++s) {
        if (seq_chunk0_host) seq_chunk0_host[s] = c;
        const int32_t bos = cu_host[s], len = cu_host[s + 1] - cu_host[s];
        if (len < 0) return -1;
        for (int32_t c0 = 0; c0 < len; c0 += chunk, ++c) {
            if (tok0_host) tok0_host[c] = bos + c0;
            if (len_host) len_host[c] = len - c0 < chunk ? len - c0 : chunk;
        }
    }
    if (seq_chunk0_host) seq_chunk0_host[n_seq] = c;
    return c;
}

extern "C" int r97b_gdn_fwd(const R97bGdnDims* dims, const R97bGdnFwd* a, void* stream) {
    if (!dims || !a || !dims_ok(*dims)) return R97B_EINVAL;
    if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->A || !a->w || !a->u || !a->S || !a->Vp || !a->P || !a->o)
        return R97B_EINVAL;
    set_attrs();
    const Dims dm = to_dims(*dims);
    cudaStream_t s = as_stream(stream);
    const auto* q = reinterpret_cast<const __nv_bfloat16*>(a->q);
    const auto* k = reinterpret_cast<const __nv_bfloat16*>(a->k);
    const auto* v = reinterpret_cast<const __nv_bfloat16*>(a->v);
    if (dm.n_chunks > 0) {
        gdn_fwd_prep<<<dim3(dm.n_chunks, dm.H), 256, kSmemPrep, s>>>(dm, q, k, v, a->g, a->beta, a->A, a->w, a->u);
    }
    gdn_fwd_state<<<dim3(dm.n_seq, dm.H, D / VS), 256, kSmemState, s>>>(dm, k, a->g, a->w, a->u, a->h0, a->S, a->Vp,
                                                                       a->ht);
    if (dm.n_chunks > 0)
        gdn_fwd_out<<<dim3(dm.n_chunks, dm.H), 256, kSmemOut, s>>>(dm, q, k, a->g, a->S, a->Vp, a->P,
                                                                   reinterpret_cast<__nv_bfloat16*>(a->o));
    return launch_status(dm.n_chunks > 0 ? 3 : 1);
}

extern "C" int r97b_gdn_bwd(const R97bGdnDims* dims, const R97bGdnBwd* a, void* stream) {
    if (!dims || !a || !dims_ok(*dims)) return R97B_EINVAL;
    if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->A || !a->w || !a->S || !a->Vp || !a->P || !a->dO ||
        !a->dS || !a->dVp || !a->dw || !a->pdq || !a->pdk || !a->pdg || !a->dq || !a->dk || !a->dv || !a->dbeta ||
        !a->dg)
        return R97B_EINVAL;
    set_attrs();
    const Dims dm = to_dims(*dims);
    cudaStream_t s = as_stream(stream);
    const auto* q = reinterpret_cast<const __nv_bfloat16*>(a->q);
    const auto* k = reinterpret_cast<const __nv_bfloat16*>(a->k);
    const auto* v = reinterpret_cast<const __nv_bfloat16*>(a->v);
    const auto* dO = reinterpret_cast<const __nv_bfloat16*>(a->dO);
    gdn_bwd_state<<<dim3(dm.n_seq, dm.H, D / VS), 256, kSmemBState, s>>>(dm, q, k, a->g, a->w, a->P, dO, a->dht,
                                                                        a->dS, a->dVp, a->dh0);
    if (dm.n_chunks > 0) {
        gdn_bwd_a<<<dim3(dm.n_chunks, dm.H), 256, kSmemBA, s>>>(dm, q, k, a->g, a->S, a->Vp, dO, a->dS, a->dVp, a->dw,
                                                                a->pdq, a->pdk, a->pdg);
        gdn_bwd_b<<<dim3(dm.n_chunks, dm.H), 256, kSmemBB, s>>>(dm, q, k, v, a->g, a->beta, a->A, a->Vp, dO, a->dVp,
                                                                a->dw, a->pdq, a->pdk, a->pdg, a->dq, a->dk, a->dv,
                                                                a->dbeta, a->dg);
    }
    return launch_status(dm.n_chunks > 0 ? 3 : 1);
}

extern "C" int r97b_gdn_sum_heads(const float* src, float* dst, int64_t T, int32_t H, int32_t Hg, void* stream) {
    if (!src || !dst || T < 0 || H <= 0 || Hg <= 0 || H % Hg) return R97B_EINVAL;
    const int64_t total = T * Hg * 128;
    if (total == 0) return R97B_OK;
    gdn_sum_heads_kernel<<<(unsigned)((total + 255) / 256), 256, 0, as_stream(stream)>>>(src, dst, T, H, Hg);
    return launch_status();
}
