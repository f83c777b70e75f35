// gdn.cu -- the chunked GatedDeltaNet recurrence, forward and backward, on sm_100a tensor cores.
//
// It computes the reference's two ops as one path (reference src/adjoint/host/gdn_kkt.cpp and
// gdn_scan.cpp; docs/adjoints/gdn-math.md s2.2, s3, s4):
//   gdn_kkt_solve : A = (I + M)^-1, M[i,l] = beta_i (k_i . k_l) e^{g_i - g_l} (l < i), per chunk of 64
//   gdn_chunk_scan: W = beta (v - e^g k S), V' = A W, o = scale (e^g q S + causal(q k^T e^{g_i-g_j}) V'),
//                   S_next = e^{g_L} S + sum_j e^{g_L - g_j} k_j (x) V'_j
// with the state held as S[d][e] (key lane d, value lane e; the reference's transposed St) in f32 and
// g the within-chunk cumulative log decay. Writing V' = u - w S with u = A diag(beta) v and
// w = A diag(beta e^g) k moves every intra-chunk product into chunk-parallel kernels and leaves a short
// sequential pass whose value lanes are independent:
//
//   F1 gdn_fwd_prep  (chunk, head)        M, A by forward substitution, w, u
//   F2 gdn_fwd_state (seq, head, V/64)    S_c entering each chunk, V'_c = u_c - w_c S_c, S_{c+1}
//   F3 gdn_fwd_out   (chunk, head)        P = causal(q k^T e^{g_i-g_j}), o = scale (e^g q S_c + P V'_c)
//   B1 gdn_bwd_state (seq, head, V/64)    reverse pass: dV' = scale P^T dO + K~ dS_next,
//                                          dS = scale Q~^T dO + e^{g_L} dS_next - w^T dV'
//   B2a gdn_bwd_a    (chunk, head)        the terms that read the states: dQ~ = scale dO S^T, dw = -dV' S^T,
//                                          dK~ = V' dS_next^T, and dg_L's e^{g_L} <S, dS_next>
//   B2b gdn_bwd_b    (chunk, head)        the intra-chunk terms: dP, dA = dw kb^T + dV' vb^T, A^T dw, A^T dV',
//                                          and the solve's adjoint dM = -A^T dA A^T (the kkt adjoint)
//
// Every product runs on the tensor cores (wmma16.cuh: mma.sync m16n8k16, bf16 in, f32 accumulate).
// q, k, v and dO are bf16 already and enter exactly; an f32 operand (a state, A, P, V', w, dV', ...) is
// split into bf16 hi + lo tiles and its product takes two or three passes, which keeps ~16 bits of the
// operand. The sequential passes keep their state in the f32 MMA accumulators. Only the 64-step forward
// substitution of the solve runs on CUDA cores.
//
// Sequences are ragged (cu_seqlens); a sequence's last chunk may be short, and its padded rows are zero
// so they add nothing. Head dims K = V = 128 and the chunk of 64 are fixed here.
#include "r97b_internal.h"
#include "fastmath.cuh"
#include "wmma16.cuh"

#include <cuda_bf16.h>
#include <math.h>

namespace r97b {
namespace {
// e^x for the decay factors: one ex2 of x log2 e (flush-to-zero). The arguments are within-chunk cumulative
// log decays or differences of them, at most 0 for a decaying gate, so the result lies in (0, 1]; the
// approximation's relative error (2 ulp, plus |x| times the rounding of x log2 e) stays below that of the
// ~16-bit split operands the products carry it into.
__device__ __forceinline__ float gexp(float x) { return ex2_ftz(x * 1.4426950408889634f); }
}  // namespace
namespace {

using bf16 = __nv_bfloat16;

constexpr int D = 128;   // key / value head dim
constexpr int L = 64;    // chunk
constexpr int F65 = 65;  // f32 pitch of a [64, 64] tile

struct Dims {
    int n_seq, H, Hg, grp, n_chunks, flags;
    int64_t T;
    float scale;
    const int* tok0;
    const int* len;
    const int* seq_c0;
};

// ------------------------------------------------------------------------------------------ staging

__device__ __forceinline__ void put_split(bf16* hi, bf16* lo, int64_t at, float x) {
    bf16 h, l;
    split_bf16(x, h, l);
    hi[at] = h;
    lo[at] = l;
}

// ---- asynchronous staging (cp.async): every f32 intermediate the kernels hand each other (V', S, dV', dS,
// dw, w, P) is kept as a bf16 (hi, lo) pair -- hi plane then lo plane, in the bytes of its f32 buffer --
// so a consumer copies it into its split tiles without converting. Rows past a chunk's end land as zeros.

// The (hi, lo) planes of an f32 buffer of `count` values.
struct Pair {
    bf16* hi;
    bf16* lo;
};
__device__ __forceinline__ Pair pair_of(const float* buf, int64_t count) {
    bf16* h = const_cast<bf16*>(reinterpret_cast<const bf16*>(buf));
    return Pair{h, h + count};
}

// rows [0, 64) of one head of a token-major [T, heads, 128] bf16 tensor -> a [64][kP128] tile
__device__ __forceinline__ void async_rows(bf16* dst, const bf16* src, int64_t tok0, int n, int heads, int head) {
    for (int idx = threadIdx.x; idx < L * 16; idx += blockDim.x) {
        const int i = idx >> 4, x = (idx & 15) * 8;
        const bool on = i < n;
        cp_async16(dst + i * kP128 + x, src + ((on ? tok0 + i : tok0) * heads + head) * D + x, on);
    }
}

// the same rows of a pair buffer -> hi and lo tiles
__device__ __forceinline__ void async_rows_pair(bf16* dh, bf16* dl, Pair src, int64_t tok0, int n, int heads,
                                                int head) {
    async_rows(dh, src.hi, tok0, n, heads, head);
    async_rows(dl, src.lo, tok0, n, heads, head);
}

// one (chunk, head)'s [128][128] block of a pair buffer [chunks, H, 128, 128] -> [128][kP128] tiles
__device__ __forceinline__ void async_block_pair(bf16* dh, bf16* dl, Pair src, int64_t block) {
    const bf16* h = src.hi + block * D * D;
    const bf16* l = src.lo + block * D * D;
    for (int idx = threadIdx.x; idx < D * 16; idx += blockDim.x) {
        const int r = idx >> 4, x = (idx & 15) * 8;
        cp_async16(dh + r * kP128 + x, h + r * D + x, true);
        cp_async16(dl + r * kP128 + x, l + r * D + x, true);
    }
}

// g (and beta) of the chunk's rows; zero past its end
__device__ __forceinline__ void async_gb(float* gs, float* bs, const float* g, const float* beta, int64_t tok0, int n,
                                         int H, int h) {
    for (int i = threadIdx.x; i < L; i += blockDim.x) {
        const bool on = i < n;
        const int64_t at = (on ? tok0 + i : tok0) * H + h;
        cp_async4(gs + i, g + at, on);
        if (bs) cp_async4(bs + i, beta + at, on);
    }
}

// sum over the 4 lanes of an accumulator row quad (lanes sharing g = lane / 4)
__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
    v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
    return v;
}

// Adds the column sums of a warp's 16 x 32 accumulator tile -- cs[j][b] holds this lane's partial for
// column n0 + 8j + 2t + b (t = lane % 4) over its two rows -- into dst[col]: a reduction over the eight
// lanes sharing t, then one shared-memory atomic per column instead of one per element.
__device__ __forceinline__ void colsum_add(float (&cs)[4][2], int n0, float* dst) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            float v = cs[j][b];
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 8);
            v += __shfl_xor_sync(0xFFFFFFFFu, v, 16);
            if (lane < 4) atomicAdd(&dst[n0 + 8 * j + 2 * lane + b], v);
        }
}

// two- / three-pass products of split operands
template <int WM, int WN, int K, bool AT, bool BT>
__device__ __forceinline__ void mma_split_a(float (&acc)[WM / 16][WN / 8][4], const bf16* Ah, const bf16* Al, int pa,
                                            const bf16* B, int pb, int m0, int n0) {
    warp_mma<WM, WN, K, AT, BT>(acc, Ah, pa, B, pb, m0, n0);
    warp_mma<WM, WN, K, AT, BT>(acc, Al, pa, B, pb, m0, n0);
}
template <int WM, int WN, int K, bool AT, bool BT>
__device__ __forceinline__ void mma_split_b(float (&acc)[WM / 16][WN / 8][4], const bf16* A, int pa, const bf16* Bh,
                                            const bf16* Bl, int pb, int m0, int n0) {
    warp_mma<WM, WN, K, AT, BT>(acc, A, pa, Bh, pb, m0, n0);
    warp_mma<WM, WN, K, AT, BT>(acc, A, pa, Bl, pb, m0, n0);
}
template <int WM, int WN, int K, bool AT, bool BT>
__device__ __forceinline__ void mma_split_ab(float (&acc)[WM / 16][WN / 8][4], const bf16* Ah, const bf16* Al, int pa,
                                             const bf16* Bh, const bf16* Bl, int pb, int m0, int n0) {
    warp_mma<WM, WN, K, AT, BT>(acc, Ah, pa, Bh, pb, m0, n0);
    warp_mma<WM, WN, K, AT, BT>(acc, Al, pa, Bh, pb, m0, n0);
    warp_mma<WM, WN, K, AT, BT>(acc, Ah, pa, Bl, pb, m0, n0);
}

// ============================================================================================ forward

// ------------------------------------------------------------------------------ the chunk's solve

// dst[i][j] = sign * sum_l X[i][l] Y[l][j] for N x N blocks (pitches px, py, pd), by the whole CTA: a thread
// a 2 x 2 tile of dst, so each shared load feeds two multiply-adds (the product is shared-load bound).
template <int N>
__device__ __forceinline__ void block_product(const float* X, int px, const float* Y, int py, float* dst, int pd,
                                              float sign) {
    constexpr int T = N / 2;  // tiles a side
    for (int e = threadIdx.x; e < T * T; e += blockDim.x) {
        const int i = (e / T) * 2, j = (e % T) * 2;
        float a00 = 0.0f, a01 = 0.0f, a10 = 0.0f, a11 = 0.0f;
#pragma unroll 8
        for (int l = 0; l < N; ++l) {
            const float x0 = X[i * px + l], x1 = X[(i + 1) * px + l];
            const float y0 = Y[l * py + j], y1 = Y[l * py + j + 1];
            a00 = fmaf(x0, y0, a00);
            a01 = fmaf(x0, y1, a01);
            a10 = fmaf(x1, y0, a10);
            a11 = fmaf(x1, y1, a11);
        }
        dst[i * pd + j] = sign * a00;
        dst[i * pd + j + 1] = sign * a01;
        dst[(i + 1) * pd + j] = sign * a10;
        dst[(i + 1) * pd + j + 1] = sign * a11;
    }
}

// As = (I + Ms)^-1 for a strictly lower-triangular 64x64 Ms (pitch F65); `scratch` holds 2 x 32 x 33 f32.
// Every thread of the 256-thread CTA calls it; it ends with the CTA synchronised.
__device__ __forceinline__ void invert_unit_lower(const float* Ms, float* As, float* scratch) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < 4) {
        // diagonal block b: lane j < 16 holds column j in registers; rows in order, no barrier needed
        const int b0 = warp * 16;
        if (lane < 16) {
            const int j = lane;
            float a[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float acc = 0.0f;
#pragma unroll
                for (int l = 0; l < i; ++l) acc = fmaf(Ms[(b0 + i) * F65 + b0 + l], a[l], acc);
                a[i] = i == j ? 1.0f : (j < i ? -acc : 0.0f);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) As[(b0 + i) * F65 + b0 + j] = a[i];
        }
    } else {
        // the strictly upper blocks are zero
        for (int e = threadIdx.x - 128; e < 64 * 64; e += 128) {
            const int i = e >> 6, j = e & 63;
            if ((j >> 4) > (i >> 4)) As[i * F65 + j] = 0.0f;
        }
    }
    __syncthreads();
    // 16 -> 32: blocks (1,0) and (3,2) (pair p: rows r0 = 16 or 48, columns c0 = 0 or 32);
    // T = M21 A11 into scratch, then X21 = -A22 T
    // (2 x 2 output tiles a thread, as block_product: each shared load feeds two multiply-adds)
    if (threadIdx.x < 128) {
        const int e = threadIdx.x, p = e >> 6, i = ((e >> 3) & 7) * 2, j = (e & 7) * 2;
        const int r0 = p ? 48 : 16, c0 = p ? 32 : 0;
        float a00 = 0.0f, a01 = 0.0f, a10 = 0.0f, a11 = 0.0f;
#pragma unroll 8
        for (int l = 0; l < 16; ++l) {
            const float x0 = Ms[(r0 + i) * F65 + c0 + l], x1 = Ms[(r0 + i + 1) * F65 + c0 + l];
            const float y0 = As[(c0 + l) * F65 + c0 + j], y1 = As[(c0 + l) * F65 + c0 + j + 1];
            a00 = fmaf(x0, y0, a00);
            a01 = fmaf(x0, y1, a01);
            a10 = fmaf(x1, y0, a10);
            a11 = fmaf(x1, y1, a11);
        }
        float* t = scratch + p * 16 * 17;
        t[i * 17 + j] = a00;
        t[i * 17 + j + 1] = a01;
        t[(i + 1) * 17 + j] = a10;
        t[(i + 1) * 17 + j + 1] = a11;
    }
    __syncthreads();
    if (threadIdx.x < 128) {
        const int e = threadIdx.x, p = e >> 6, i = ((e >> 3) & 7) * 2, j = (e & 7) * 2;
        const int r0 = p ? 48 : 16, c0 = p ? 32 : 0;
        const float* t = scratch + p * 16 * 17;
        float a00 = 0.0f, a01 = 0.0f, a10 = 0.0f, a11 = 0.0f;
#pragma unroll 8
        for (int l = 0; l < 16; ++l) {
            const float x0 = As[(r0 + i) * F65 + r0 + l], x1 = As[(r0 + i + 1) * F65 + r0 + l];
            const float y0 = t[l * 17 + j], y1 = t[l * 17 + j + 1];
            a00 = fmaf(x0, y0, a00);
            a01 = fmaf(x0, y1, a01);
            a10 = fmaf(x1, y0, a10);
            a11 = fmaf(x1, y1, a11);
        }
        As[(r0 + i) * F65 + c0 + j] = -a00;
        As[(r0 + i) * F65 + c0 + j + 1] = -a01;
        As[(r0 + i + 1) * F65 + c0 + j] = -a10;
        As[(r0 + i + 1) * F65 + c0 + j + 1] = -a11;
    }
    __syncthreads();
    // 32 -> 64: block (1,0) of 32x32 blocks; T = M[32:64][0:32] A[0:32][0:32], X = -A[32:64][32:64] T
    float* t = scratch;  // [32][33]
    block_product<32>(Ms + 32 * F65, F65, As, F65, t, 33, 1.0f);
    __syncthreads();
    block_product<32>(As + 32 * F65 + 32, F65, t, 33, As + 32 * F65, F65, -1.0f);
    __syncthreads();
}

// F1: per (chunk, value head): A = (I + M)^-1, w = (A diag(beta e^g)) k, u = (A diag(beta)) v.
__global__ void __launch_bounds__(256) gdn_fwd_prep(Dims dm, const bf16* __restrict__ k, const bf16* __restrict__ v,
                                                    const float* __restrict__ g, const float* __restrict__ beta,
                                                    float* __restrict__ A, float* __restrict__ w, float* __restrict__ u) {
    extern __shared__ __align__(16) unsigned char smraw[];
    bf16* ks = reinterpret_cast<bf16*>(smraw);          // [64][136]
    bf16* vs = ks + L * kP128;                           // [64][136]
    bf16* a1h = vs + L * kP128;                          // [64][72]  A diag(beta e^g), hi/lo
    bf16* a1l = a1h + L * kP64;
    bf16* a2h = a1l + L * kP64;                          // A diag(beta), hi/lo
    bf16* a2l = a2h + L * kP64;
    float* Ms = reinterpret_cast<float*>(a2l + L * kP64);  // [64][65]
    float* As = Ms + L * F65;                              // [64][65]
    float* red = As + L * F65;                             // [4][64]
    float* gs = red + 4 * L;
    float* bs = gs + L;
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int warp = threadIdx.x >> 5;
    const bool given = (dm.flags & R97B_GDN_A_GIVEN) != 0;
    async_rows(ks, k, tok0, n, dm.Hg, hk);
    async_rows(vs, v, tok0, n, dm.H, h);
    async_gb(gs, bs, g, beta, tok0, n, dm.H, h);
    cp_async_commit();
    if (given) {  // the caller's solve: its lower triangle, diagonal included, for the chunk's rows
        const int j = threadIdx.x & 63, i0 = threadIdx.x >> 6;  // 256 threads: rows i0, i0 + 4, ...
        float av[L / 4];
#pragma unroll
        for (int q = 0; q < L / 4; ++q) {  // every load issued before the first store
            const int i = i0 + 4 * q;
            av[q] = (i < n && j <= i) ? A[((tok0 + i) * dm.H + h) * L + j] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < L / 4; ++q) As[(i0 + 4 * q) * F65 + j] = av[q];
    }
    cp_async_wait_all();
    __syncthreads();
    if (!given) {
        // M = strict lower of beta_i (k_i . k_l) e^{g_i - g_l}
        float acc[1][4][4];
        acc_zero<16, 32>(acc);
        const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 32;
        warp_mma<16, 32, 128, false, false>(acc, ks, kP128, ks, kP128, m0, n0);
        acc_for<16, 32>(acc, m0, n0, [&](int r, int l, float& x) {
            // only the chunk's own rows: a padded row's g is 0, and e^{0 - g_l} can overflow to inf, whose
            // 0 * inf the blocked inverse would carry into every row
            Ms[r * F65 + l] = (l < r && r < n) ? bs[r] * x * gexp(gs[r] - gs[l]) : 0.0f;
        });
        __syncthreads();
        // A = (I + M)^-1 by blocks: the four 16x16 diagonal blocks by forward substitution (a warp each),
        // then 16 -> 32 -> 64 with X21 = -A22 (M21 A11) (the inverse of a block lower-triangular matrix)
        invert_unit_lower(Ms, As, reinterpret_cast<float*>(a1h));
    }
    {
        const int j = threadIdx.x & 63;  // a thread keeps its column (the stride is a multiple of 64)
        const float e = bs[j] * gexp(gs[j]), bj = bs[j];
        for (int i = threadIdx.x >> 6; i < L; i += blockDim.x >> 6) {
            const float a = As[i * F65 + j];
            if (i < n && !given) A[((tok0 + i) * dm.H + h) * L + j] = a;
            put_split(a1h, a1l, i * kP64 + j, a * e);
            put_split(a2h, a2l, i * kP64 + j, a * bj);
        }
    }
    __syncthreads();
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 64;
    float acc[1][8][4];
    acc_zero<16, 64>(acc);
    mma_split_a<16, 64, 64, false, true>(acc, a1h, a1l, kP64, ks, kP128, m0, n0);
    bf16* w_hi = reinterpret_cast<bf16*>(w);             // w is kept as a bf16 (hi, lo) pair in the
    bf16* w_lo = w_hi + (int64_t)dm.T * dm.H * D;         // bytes of an f32 [T, H, 128] buffer
    acc_pairs<16, 64>(m0, n0, [&](int r, int d, int i, int j, int hh) {
        if (r < n) put_split2(w_hi, w_lo, ((tok0 + r) * dm.H + h) * D + d, acc[i][j][2 * hh], acc[i][j][2 * hh + 1]);
    });
    acc_zero<16, 64>(acc);
    mma_split_a<16, 64, 64, false, true>(acc, a2h, a2l, kP64, vs, kP128, m0, n0);
    acc_pairs<16, 64>(m0, n0, [&](int r, int d, int i, int j, int hh) {
        if (r < n)
            *reinterpret_cast<float2*>(u + ((tok0 + r) * dm.H + h) * D + d) =
                make_float2(acc[i][j][2 * hh], acc[i][j][2 * hh + 1]);
    });
}

// F2: per (sequence, value head, 64 value lanes): the state pass over the sequence's chunks. The state
// slice S[128][64] lives in the f32 accumulators of its own product (S += k^T V''); each chunk's operands
// (w as a bf16 hi/lo pair, k, the u slice, g) stream into a double-buffered stage with cp.async while the
// previous chunk computes.
constexpr int VS2 = 64;   // value lanes per forward-state CTA
constexpr int P64 = 72;   // bf16 pitch of a [*, 64] tile (== kP64)
constexpr int U68 = 68;   // f32 pitch of the u slice

struct F2Stage {
    bf16 wh[L * kP128], wl[L * kP128], ks[L * kP128];
    float us[L * U68];
    float gs[L];
};

__device__ __forceinline__ void f2_issue(F2Stage& st, const Dims& dm, const bf16* w_hi, const bf16* w_lo,
                                         const bf16* k, const float* u, const float* g, int c, int h, int hk, int e0) {
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    for (int idx = threadIdx.x; idx < L * 16; idx += blockDim.x) {
        const int i = idx >> 4, q = (idx & 15) * 8;
        const bool on = i < n;
        const int64_t row = on ? tok0 + i : tok0;
        cp_async16(&st.wh[i * kP128 + q], w_hi + (row * dm.H + h) * D + q, on);
        cp_async16(&st.wl[i * kP128 + q], w_lo + (row * dm.H + h) * D + q, on);
        cp_async16(&st.ks[i * kP128 + q], k + (row * dm.Hg + hk) * D + q, on);
        cp_async16(&st.us[i * U68 + (q >> 1)], u + (row * dm.H + h) * D + e0 + (q >> 1), on);
    }
    for (int i = threadIdx.x; i < L; i += blockDim.x) {
        const bool on = i < n;
        cp_async4(&st.gs[i], g + ((on ? tok0 + i : tok0) * dm.H + h), on);
    }
    cp_async_commit();
}

__global__ void __launch_bounds__(256) gdn_fwd_state(Dims dm, const bf16* __restrict__ k, const float* __restrict__ g,
                                                     const float* __restrict__ w, const float* __restrict__ u,
                                                     const float* __restrict__ h0, float* __restrict__ S_all,
                                                     float* __restrict__ Vp, float* __restrict__ ht) {
    extern __shared__ __align__(16) unsigned char smraw[];
    F2Stage* stage = reinterpret_cast<F2Stage*>(smraw);           // [2]
    bf16* sh = reinterpret_cast<bf16*>(smraw + 2 * sizeof(F2Stage));  // S hi/lo [128][72]
    bf16* sl = sh + D * P64;
    bf16* vh = sl + D * P64;                                       // V'' = e^{gL-g} V' hi/lo [64][72]
    bf16* vl = vh + L * P64;
    const bf16* w_hi = reinterpret_cast<const bf16*>(w);
    const bf16* w_lo = w_hi + dm.T * dm.H * D;
    const int seq = blockIdx.x, h = blockIdx.y, e0 = blockIdx.z * VS2, hk = h / dm.grp;
    const int warp = threadIdx.x >> 5;
    const int sm0 = (warp & 3) * 32, sn0 = (warp >> 2) * 32;  // this warp's S tile (32 x 32)
    const int vm0 = (warp & 3) * 16, vn0 = (warp >> 2) * 32;  // this warp's V' tile (16 x 32)
    const int c0 = dm.seq_c0[seq], c1 = dm.seq_c0[seq + 1];
    if (c0 < c1) f2_issue(stage[0], dm, w_hi, w_lo, k, u, g, c0, h, hk, e0);
    float S[2][4][4];
    acc_for<32, 32>(S, sm0, sn0, [&](int d, int e, float& x) {
        x = h0 ? h0[(((int64_t)seq * dm.H + h) * D + e0 + e) * D + d] : 0.0f;
    });
    acc_pairs<32, 32>(sm0, sn0, [&](int d, int e, int i, int j, int hh) {
        put_split2(sh, sl, d * P64 + e, S[i][j][2 * hh], S[i][j][2 * hh + 1]);
    });
    const Pair Sp = pair_of(S_all, (int64_t)dm.n_chunks * dm.H * D * D);
    const Pair Vpp = pair_of(Vp, dm.T * dm.H * D);
    for (int c = c0; c < c1; ++c) {
        F2Stage& st = stage[(c - c0) & 1];
        const int64_t tok0 = dm.tok0[c];
        const int n = dm.len[c];
        const int64_t sb = ((int64_t)c * dm.H + h) * D * D;
        acc_pairs<32, 32>(sm0, sn0, [&](int d, int e, int i, int j, int hh) {
            put_split2(Sp.hi, Sp.lo, sb + d * D + e0 + e, S[i][j][2 * hh], S[i][j][2 * hh + 1]);
        });
        cp_async_wait_all();
        __syncthreads();  // stage c landed; S split written; every warp is past chunk c-1's products
        if (c + 1 < c1) f2_issue(stage[(c + 1 - c0) & 1], dm, w_hi, w_lo, k, u, g, c + 1, h, hk, e0);
        const float gl = st.gs[n - 1];
        {
            float acc[1][4][4];
            acc_zero<16, 32>(acc);
            mma_split_ab<16, 32, 128, false, true>(acc, st.wh, st.wl, kP128, sh, sl, P64, vm0, vn0);
            acc_pairs<16, 32>(vm0, vn0, [&](int i, int e, int a, int b, int hh) {
                const float v0 = st.us[i * U68 + e] - acc[a][b][2 * hh];
                const float v1 = st.us[i * U68 + e + 1] - acc[a][b][2 * hh + 1];
                const float sc = i < n ? gexp(gl - st.gs[i]) : 0.0f;
                if (i < n) put_split2(Vpp.hi, Vpp.lo, ((tok0 + i) * dm.H + h) * D + e0 + e, v0, v1);
                put_split2(vh, vl, i * P64 + e, v0 * sc, v1 * sc);
            });
        }
        __syncthreads();
        const float el = gexp(gl);
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b)
#pragma unroll
                for (int e = 0; e < 4; ++e) S[a][b][e] *= el;
        mma_split_b<32, 32, 64, true, true>(S, st.ks, kP128, vh, vl, P64, sm0, sn0);
        // the next chunk's S operand (sh/sl were last read before the sync above)
        acc_pairs<32, 32>(sm0, sn0, [&](int d, int e, int i, int j, int hh) {
            put_split2(sh, sl, d * P64 + e, S[i][j][2 * hh], S[i][j][2 * hh + 1]);
        });
    }
    if (ht)
        acc_for<32, 32>(S, sm0, sn0, [&](int d, int e, float& x) {
            ht[(((int64_t)seq * dm.H + h) * D + e0 + e) * D + d] = x;
        });
}

// F3: per (chunk, value head): P and the output rows.
__global__ void __launch_bounds__(256) gdn_fwd_out(Dims dm, const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                   const float* __restrict__ g, const float* __restrict__ S_all,
                                                   const float* __restrict__ Vp, float* __restrict__ P_all,
                                                   bf16* __restrict__ o) {
    extern __shared__ __align__(16) unsigned char smraw[];
    bf16* qs = reinterpret_cast<bf16*>(smraw);   // [64][136]
    bf16* ks = qs + L * kP128;                   // [64][136]
    bf16* vh = ks + L * kP128;                   // V' hi/lo [64][136]
    bf16* vl = vh + L * kP128;
    bf16* sh = vl + L * kP128;                   // S hi/lo [128][136]
    bf16* sl = sh + D * kP128;
    bf16* ph = sl + D * kP128;                   // P hi/lo [64][72]
    bf16* pl = ph + L * kP64;
    float* gs = reinterpret_cast<float*>(pl + L * kP64);
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int warp = threadIdx.x >> 5;
    async_rows(qs, q, tok0, n, dm.Hg, hk);
    async_rows(ks, k, tok0, n, dm.Hg, hk);
    async_rows_pair(vh, vl, pair_of(Vp, dm.T * dm.H * D), tok0, n, dm.H, h);
    async_block_pair(sh, sl, pair_of(S_all, (int64_t)dm.n_chunks * dm.H * D * D), (int64_t)c * dm.H + h);
    async_gb(gs, nullptr, g, nullptr, tok0, n, dm.H, h);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    {
        float acc[1][4][4];
        acc_zero<16, 32>(acc);
        const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 32;
        warp_mma<16, 32, 128, false, false>(acc, qs, kP128, ks, kP128, m0, n0);
        // P is kept as a bf16 (hi, lo) pair in the bytes of an f32 [chunks, H, 64, 64] buffer
        bf16* P_hi = reinterpret_cast<bf16*>(P_all);
        bf16* P_lo = P_hi + (int64_t)dm.n_chunks * dm.H * L * L;
        const int64_t pbase = ((int64_t)c * dm.H + h) * L * L;
        acc_pairs<16, 32>(m0, n0, [&](int r, int l, int i, int j, int hh) {
            const float p0 = (l <= r && r < n) ? acc[i][j][2 * hh] * gexp(gs[r] - gs[l]) : 0.0f;
            const float p1 = (l + 1 <= r && r < n) ? acc[i][j][2 * hh + 1] * gexp(gs[r] - gs[l + 1]) : 0.0f;
            put_split2(P_hi, P_lo, pbase + r * L + l, p0, p1);
            put_split2(ph, pl, r * kP64 + l, p0, p1);
        });
    }
    __syncthreads();
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 64;
    float qsacc[1][8][4], pvacc[1][8][4];
    acc_zero<16, 64>(qsacc);
    acc_zero<16, 64>(pvacc);
    mma_split_b<16, 64, 128, false, true>(qsacc, qs, kP128, sh, sl, kP128, m0, n0);
    mma_split_ab<16, 64, 64, false, true>(pvacc, ph, pl, kP64, vh, vl, kP128, m0, n0);
    const int lane = threadIdx.x & 31, gq = lane >> 2;
    const float eg0 = gexp(gs[m0 + gq]), eg1 = gexp(gs[m0 + gq + 8]);
    acc_pairs<16, 64>(m0, n0, [&](int r, int e, int i, int j, int hh) {  // two columns a 4-byte store
        const float eg = hh ? eg1 : eg0;
        const float y0 = dm.scale * (qsacc[i][j][2 * hh] * eg + pvacc[i][j][2 * hh]);
        const float y1 = dm.scale * (qsacc[i][j][2 * hh + 1] * eg + pvacc[i][j][2 * hh + 1]);
        if (r < n)
            *reinterpret_cast<__nv_bfloat162*>(o + ((tok0 + r) * dm.H + h) * D + e) = __floats2bfloat162_rn(y0, y1);
    });
}

// ============================================================================================ backward

// B1: per (sequence, value head, 64 value lanes): the reverse state pass; dS lives in the accumulators.
// Each chunk's operands stream in with cp.async: the ones read late in a chunk (w as a bf16 hi/lo pair, q)
// are double-buffered and fetched a whole chunk ahead; the ones only the dV' products read (P as a pair,
// k, the dO slice, g) have one buffer, refilled for the next chunk as soon as those products are done.
constexpr int VSB = 64;  // value lanes per backward-state CTA

struct B1Late {
    bf16 wh[L * kP128], wl[L * kP128], qs[L * kP128];
};
struct B1Early {
    bf16 ph[L * kP64], pl[L * kP64];
    bf16 ks[L * kP128];
    bf16 dos[L * kP64];
    float gs[L];
};

__device__ __forceinline__ void b1_issue_late(B1Late& st, const Dims& dm, const bf16* q, const bf16* w_hi,
                                              const bf16* w_lo, int c, int h, int hk) {
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    for (int idx = threadIdx.x; idx < L * 16; idx += blockDim.x) {
        const int i = idx >> 4, x = (idx & 15) * 8;
        const bool on = i < n;
        const int64_t row = on ? tok0 + i : tok0;
        cp_async16(&st.wh[i * kP128 + x], w_hi + (row * dm.H + h) * D + x, on);
        cp_async16(&st.wl[i * kP128 + x], w_lo + (row * dm.H + h) * D + x, on);
        cp_async16(&st.qs[i * kP128 + x], q + (row * dm.Hg + hk) * D + x, on);
    }
    cp_async_commit();
}

__device__ __forceinline__ void b1_issue_early(B1Early& st, const Dims& dm, const bf16* k, const bf16* P_hi,
                                               const bf16* P_lo, const bf16* dO, const float* g, int c, int h,
                                               int hk, int e0) {
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int64_t pbase = ((int64_t)c * dm.H + h) * L * L;
    for (int idx = threadIdx.x; idx < L * 16; idx += blockDim.x) {
        const int i = idx >> 4, x = (idx & 15) * 8;
        const bool on = i < n;
        const int64_t row = on ? tok0 + i : tok0;
        cp_async16(&st.ks[i * kP128 + x], k + (row * dm.Hg + hk) * D + x, on);
        if (x < L) {
            cp_async16(&st.ph[i * kP64 + x], P_hi + pbase + i * L + x, true);
            cp_async16(&st.pl[i * kP64 + x], P_lo + pbase + i * L + x, true);
            cp_async16(&st.dos[i * kP64 + x], dO + (row * dm.H + h) * D + e0 + x, on);
        }
    }
    for (int i = threadIdx.x; i < L; i += blockDim.x) {
        const bool on = i < n;
        cp_async4(&st.gs[i], g + ((on ? tok0 + i : tok0) * dm.H + h), on);
    }
    cp_async_commit();
}

__global__ void __launch_bounds__(256) gdn_bwd_state(Dims dm, const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                     const float* __restrict__ g, const float* __restrict__ w,
                                                     const float* __restrict__ P_all, const bf16* __restrict__ dO,
                                                     const float* __restrict__ dht, float* __restrict__ dS_all,
                                                     float* __restrict__ dVp, float* __restrict__ dh0) {
    extern __shared__ __align__(16) unsigned char smraw[];
    B1Late* late = reinterpret_cast<B1Late*>(smraw);                          // [2]
    B1Early* early = reinterpret_cast<B1Early*>(smraw + 2 * sizeof(B1Late));  // [1]
    bf16* dsh = reinterpret_cast<bf16*>(smraw + 2 * sizeof(B1Late) + sizeof(B1Early));  // dS hi/lo [128][72]
    bf16* dsl = dsh + D * kP64;
    bf16* egh = dsl + D * kP64;  // e^g dO hi/lo [64][72]
    bf16* egl = egh + L * kP64;
    bf16* dvh = egl + L * kP64;  // dV' hi/lo [64][72]
    bf16* dvl = dvh + L * kP64;
    const bf16* w_hi = reinterpret_cast<const bf16*>(w);
    const bf16* w_lo = w_hi + dm.T * dm.H * D;
    const bf16* P_hi = reinterpret_cast<const bf16*>(P_all);
    const bf16* P_lo = P_hi + (int64_t)dm.n_chunks * dm.H * L * L;
    const int seq = blockIdx.x, h = blockIdx.y, e0 = blockIdx.z * VSB, hk = h / dm.grp;
    const int warp = threadIdx.x >> 5;
    const int sm0 = (warp & 3) * 32, sn0 = (warp >> 2) * 32;  // this warp's dS tile (32 x 32)
    const int vm0 = (warp & 3) * 16, vn0 = (warp >> 2) * 32;  // this warp's dV' tile (16 x 32)
    const Pair dSp = pair_of(dS_all, (int64_t)dm.n_chunks * dm.H * D * D);
    const Pair dVpp = pair_of(dVp, dm.T * dm.H * D);
    const int c0 = dm.seq_c0[seq], c1 = dm.seq_c0[seq + 1];
    if (c0 < c1) {
        b1_issue_late(late[0], dm, q, w_hi, w_lo, c1 - 1, h, hk);
        b1_issue_early(*early, dm, k, P_hi, P_lo, dO, g, c1 - 1, h, hk, e0);
    }
    float dS[2][4][4];
    acc_for<32, 32>(dS, sm0, sn0, [&](int d, int e, float& x) {
        x = dht ? dht[(((int64_t)seq * dm.H + h) * D + e0 + e) * D + d] : 0.0f;
    });
    for (int c = c1 - 1; c >= c0; --c) {
        B1Late& lt = late[(c1 - 1 - c) & 1];
        B1Early& et = *early;
        const int64_t tok0 = dm.tok0[c];
        const int n = dm.len[c];
        const int64_t sb = ((int64_t)c * dm.H + h) * D * D;
        // dsh/dsl were last read by the previous chunk's dV' products, before its middle barrier
        acc_pairs<32, 32>(sm0, sn0, [&](int d, int e, int i, int j, int hh) {
            const float x0 = dS[i][j][2 * hh], x1 = dS[i][j][2 * hh + 1];
            put_split2(dSp.hi, dSp.lo, sb + d * D + e0 + e, x0, x1);
            put_split2(dsh, dsl, d * kP64 + e, x0, x1);
        });
        cp_async_wait_all();
        __syncthreads();  // chunk c's operands landed; dS split written; chunk c+1's products are done
        if (c > c0) b1_issue_late(late[(c1 - c) & 1], dm, q, w_hi, w_lo, c - 1, h, hk);
        const float gl = et.gs[n - 1];
        for (int idx = threadIdx.x; idx < L * VSB / 2; idx += blockDim.x) {
            const int i = idx >> 5, e = (idx & 31) * 2;
            const float eg = gexp(et.gs[i]);
            const float2 d2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(et.dos + i * kP64 + e));
            put_split2(egh, egl, i * kP64 + e, d2.x * eg, d2.y * eg);
        }
        {
            // dV' = scale P^T dO + e^{gL - g} (k dS)
            float a1[1][4][4], a2[1][4][4];
            acc_zero<16, 32>(a1);
            acc_zero<16, 32>(a2);
            mma_split_a<16, 32, 64, true, true>(a1, et.ph, et.pl, kP64, et.dos, kP64, vm0, vn0);
            mma_split_b<16, 32, 128, false, true>(a2, et.ks, kP128, dsh, dsl, kP64, vm0, vn0);
            const int ja = vm0 + ((threadIdx.x & 31) >> 2), jb = ja + 8;  // this lane's two rows
            const float sca = ja < n ? gexp(gl - et.gs[ja]) : 0.0f, scb = jb < n ? gexp(gl - et.gs[jb]) : 0.0f;
            acc_pairs<16, 32>(vm0, vn0, [&](int j, int e, int a, int b, int hh) {
                const float sc = hh ? scb : sca;
                const float d0 = j < n ? dm.scale * a1[a][b][2 * hh] + sc * a2[a][b][2 * hh] : 0.0f;
                const float d1 = j < n ? dm.scale * a1[a][b][2 * hh + 1] + sc * a2[a][b][2 * hh + 1] : 0.0f;
                if (j < n) put_split2(dVpp.hi, dVpp.lo, ((tok0 + j) * dm.H + h) * D + e0 + e, d0, d1);
                put_split2(dvh, dvl, j * kP64 + e, d0, d1);
            });
        }
        __syncthreads();  // dV' written; chunk c's P, k, dO and g are no longer read
        if (c > c0) b1_issue_early(*early, dm, k, P_hi, P_lo, dO, g, c - 1, h, hk, e0);
        // dS = e^{gL} dS + scale q^T (e^g dO) - w^T dV'
        const float el = gexp(gl);
        float t1[2][4][4], t2[2][4][4];
        acc_zero<32, 32>(t1);
        acc_zero<32, 32>(t2);
        mma_split_b<32, 32, 64, true, true>(t1, lt.qs, kP128, egh, egl, kP64, sm0, sn0);
        mma_split_ab<32, 32, 64, true, true>(t2, lt.wh, lt.wl, kP128, dvh, dvl, kP64, sm0, sn0);
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b)
#pragma unroll
                for (int e = 0; e < 4; ++e) dS[a][b][e] = el * dS[a][b][e] + dm.scale * t1[a][b][e] - t2[a][b][e];
    }
    if (dh0)
        acc_for<32, 32>(dS, sm0, sn0, [&](int d, int e, float& x) {
            dh0[(((int64_t)seq * dm.H + h) * D + e0 + e) * D + d] = x;
        });
}

// B2a: per (chunk, value head): the state-reading terms, written as partials of dq, dk, dg (pdq, pdk, pdg:
// the launcher passes the outputs themselves, which B2b then adds to). Its operands arrive in three
// cp.async groups: what dQ~ and dw read (S, dO, q, dV', g), then dS_next, then (into the tiles dQ~ and dw
// free) V' and k.
__global__ void __launch_bounds__(256) gdn_bwd_a(Dims dm, const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                 const float* __restrict__ g, const float* __restrict__ S_all,
                                                 const float* __restrict__ Vp, const bf16* __restrict__ dO,
                                                 const float* __restrict__ dS_all, const float* __restrict__ dVp,
                                                 float* __restrict__ dw, float* __restrict__ pdq, float* __restrict__ pdk,
                                                 float* __restrict__ pdg) {
    extern __shared__ __align__(16) unsigned char smraw[];
    bf16* sh = reinterpret_cast<bf16*>(smraw);   // S hi/lo [128][136]
    bf16* sl = sh + D * kP128;
    bf16* th = sl + D * kP128;                   // dS_next hi/lo [128][136]
    bf16* tl = th + D * kP128;
    bf16* xs = tl + D * kP128;                   // dO [64][136], then k
    bf16* qs = xs + L * kP128;                   // q [64][136]
    bf16* yh = qs + L * kP128;                   // dV' hi/lo [64][136], then V' hi/lo
    bf16* yl = yh + L * kP128;
    float* gs = reinterpret_cast<float*>(yl + L * kP128);
    float* dgs = gs + L;
    float* red = dgs + L;  // [8]
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 64;
    const int64_t nb = (int64_t)dm.n_chunks * dm.H * D * D, nt = dm.T * dm.H * D;
    const int64_t blk = (int64_t)c * dm.H + h;
    async_block_pair(sh, sl, pair_of(S_all, nb), blk);
    async_rows(xs, dO, tok0, n, dm.H, h);
    async_rows(qs, q, tok0, n, dm.Hg, hk);
    async_rows_pair(yh, yl, pair_of(dVp, nt), tok0, n, dm.H, h);
    async_gb(gs, nullptr, g, nullptr, tok0, n, dm.H, h);
    cp_async_commit();
    async_block_pair(th, tl, pair_of(dS_all, nb), blk);
    cp_async_commit();
    for (int i = threadIdx.x; i < L; i += blockDim.x) dgs[i] = 0.0f;
    cp_async_wait_but_one();
    __syncthreads();
    float dq[1][8][4];
    {
        // dQ~ = scale dO S^T ; dq = e^g dQ~ ; dg_i += e^{g_i} q_i . dQ~_i
        acc_zero<16, 64>(dq);
        mma_split_b<16, 64, 128, false, false>(dq, xs, kP128, sh, sl, kP128, m0, n0);
        float p0 = 0.0f, p1 = 0.0f;
        const int gq = lane >> 2;  // this lane's two rows: m0 + gq and m0 + gq + 8
        const float f0 = dm.scale * gexp(gs[m0 + gq]), f1 = dm.scale * gexp(gs[m0 + gq + 8]);
        acc_walk<16, 64>(m0, n0, [&](int r, int d, int i, int j, int q) {
            float& x = dq[i][j][q];
            x *= (q >> 1) ? f1 : f0;
            const float t = __bfloat162float(qs[r * kP128 + d]) * x;
            if (q >> 1) p1 += t; else p0 += t;
        });
        p0 = quad_sum(p0);
        p1 = quad_sum(p1);
        if ((lane & 3) == 0) {
            atomicAdd(&dgs[m0 + (lane >> 2)], p0);
            atomicAdd(&dgs[m0 + (lane >> 2) + 8], p1);
        }
    }
    {
        // dw = -dV' S^T
        const Pair dwp = pair_of(dw, nt);
        float acc[1][8][4];
        acc_zero<16, 64>(acc);
        mma_split_ab<16, 64, 128, false, false>(acc, yh, yl, kP128, sh, sl, kP128, m0, n0);
        acc_pairs<16, 64>(m0, n0, [&](int r, int d, int i, int j, int hh) {
            if (r < n) put_split2(dwp.hi, dwp.lo, ((tok0 + r) * dm.H + h) * D + d, -acc[i][j][2 * hh], -acc[i][j][2 * hh + 1]);
        });
    }
    __syncthreads();  // dO and dV' are no longer read
    async_rows_pair(yh, yl, pair_of(Vp, nt), tok0, n, dm.H, h);
    async_rows(xs, k, tok0, n, dm.Hg, hk);
    cp_async_commit();
    cp_async_wait_but_one();  // dS_next landed
    __syncthreads();
    // <S, dS_next> from the pairs, while V' and k land
    float sdot = 0.0f;
    for (int idx = threadIdx.x; idx < D * D / 2; idx += blockDim.x) {
        const int r = (idx * 2) >> 7, cc = (idx * 2) & 127;
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sh + r * kP128 + cc));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sl + r * kP128 + cc));
        const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(th + r * kP128 + cc));
        const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(tl + r * kP128 + cc));
        sdot += (a.x + b.x) * (x.x + y.x) + (a.y + b.y) * (x.y + y.y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sdot += __shfl_xor_sync(0xFFFFFFFFu, sdot, o);
    if (lane == 0) red[warp] = sdot;
    cp_async_wait_all();
    __syncthreads();
    const float gl = gs[n - 1];
    float dk[1][8][4];
    {
        // dK~ = V' dS_next^T ; dk_j = e^{gL-gj} dK~_j ; dg_j -= K~_j . dK~_j ; dg_L += their sum
        acc_zero<16, 64>(dk);
        mma_split_ab<16, 64, 128, false, false>(dk, yh, yl, kP128, th, tl, kP128, m0, n0);
        float p0 = 0.0f, p1 = 0.0f;
        const int gq = lane >> 2, ra = m0 + gq, rb = ra + 8;
        const float f0 = ra < n ? gexp(gl - gs[ra]) : 0.0f, f1 = rb < n ? gexp(gl - gs[rb]) : 0.0f;
        acc_walk<16, 64>(m0, n0, [&](int r, int d, int i, int j, int q) {
            float& x = dk[i][j][q];
            x *= (q >> 1) ? f1 : f0;
            const float t = __bfloat162float(xs[r * kP128 + d]) * x;
            if (q >> 1) p1 += t; else p0 += t;
        });
        p0 = quad_sum(p0);
        p1 = quad_sum(p1);
        if ((lane & 3) == 0) {
            atomicAdd(&dgs[m0 + (lane >> 2)], -p0);
            atomicAdd(&dgs[m0 + (lane >> 2) + 8], -p1);
            atomicAdd(&dgs[n - 1], p0 + p1);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int i = 0; i < 8; ++i) s += red[i];
        dgs[n - 1] += gexp(gl) * s;
    }
    __syncthreads();
    acc_pairs<16, 64>(m0, n0, [&](int r, int d, int i, int j, int hh) {  // two columns an 8-byte store
        if (r < n) {
            const int64_t at = ((tok0 + r) * dm.H + h) * D + d;
            *reinterpret_cast<float2*>(pdq + at) = make_float2(dq[i][j][2 * hh], dq[i][j][2 * hh + 1]);
            *reinterpret_cast<float2*>(pdk + at) = make_float2(dk[i][j][2 * hh], dk[i][j][2 * hh + 1]);
        }
    });
    for (int i = threadIdx.x; i < n; i += blockDim.x) pdg[(tok0 + i) * dm.H + h] = dgs[i];
}

// The solve's adjoint for one (chunk, head), shared by B2b and B3 (reference gdn_kkt.cpp:272-352): with
// dA in th/tl (its strict lower triangle is what counts), Y = dA A^T, dM = -A^T Y on the strict lower
// block, then dbeta_i += sum_l dM_il C_il, dg_i += sum_l dM_il M_il, dg_l -= the same, and
// dk += E k + E^T k with E_il = dM_il beta_i e^{g_i - g_l}. C = (k k^T) e^{g_i - g_l} (strict lower, Cs).
// th/tl are overwritten with E; yh/yl are scratch. Every thread of the CTA calls it.
__device__ __forceinline__ void kkt_adjoint(const bf16* ah, const bf16* al, bf16* th, bf16* tl, bf16* yh, bf16* yl,
                                            const bf16* ks, const float* Cs, const float* gs, const float* bs,
                                            float* dgs, float* dbs, int n, float (&dka)[1][8][4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pm0 = (warp & 3) * 16, pn0 = (warp >> 2) * 32;
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 64;
    {
        float acc[1][4][4];
        acc_zero<16, 32>(acc);
        mma_split_ab<16, 32, 64, false, false>(acc, th, tl, kP64, ah, al, kP64, pm0, pn0);
        acc_for<16, 32>(acc, pm0, pn0, [&](int r, int l, float& x) { put_split(yh, yl, r * kP64 + l, x); });
        __syncthreads();
        acc_zero<16, 32>(acc);
        mma_split_ab<16, 32, 64, true, true>(acc, ah, al, kP64, yh, yl, kP64, pm0, pn0);
        __syncthreads();  // every warp has read dA (th/tl) before E overwrites it
        float b0 = 0.0f, b1 = 0.0f, g0 = 0.0f, g1 = 0.0f;
        float cs[4][2] = {};
        acc_walk<16, 32>(pm0, pn0, [&](int r, int l, int i, int j, int q) {
            const bool on = l < r && r < n;
            const float dm_ = on ? -acc[i][j][q] : 0.0f;
            const float kh = Cs[r * F65 + l];
            const float gg = dm_ * bs[r] * kh;
            if (q >> 1) { b1 += dm_ * kh; g1 += gg; } else { b0 += dm_ * kh; g0 += gg; }
            cs[j][q & 1] -= gg;  // zero off the strict lower block
            put_split(th, tl, r * kP64 + l, on ? dm_ * bs[r] * gexp(gs[r] - gs[l]) : 0.0f);
        });
        colsum_add(cs, pn0, dgs);
        b0 = quad_sum(b0);
        b1 = quad_sum(b1);
        g0 = quad_sum(g0);
        g1 = quad_sum(g1);
        if ((lane & 3) == 0) {
            atomicAdd(&dbs[pm0 + (lane >> 2)], b0);
            atomicAdd(&dgs[pm0 + (lane >> 2)], g0);
            atomicAdd(&dbs[pm0 + (lane >> 2) + 8], b1);
            atomicAdd(&dgs[pm0 + (lane >> 2) + 8], g1);
        }
    }
    __syncthreads();
    mma_split_a<16, 64, 64, false, true>(dka, th, tl, kP64, ks, kP128, m0, n0);  // dk_i += sum_l E_il k_l
    mma_split_a<16, 64, 64, true, true>(dka, th, tl, kP64, ks, kP128, m0, n0);   // dk_l += sum_i E_il k_i
}

// B2b: per (chunk, value head): the intra-chunk terms and the solve's adjoint; adds B2a's partials.
__global__ void __launch_bounds__(256) gdn_bwd_b(Dims dm, const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                 const bf16* __restrict__ v, const float* __restrict__ g,
                                                 const float* __restrict__ beta, const float* __restrict__ A,
                                                 const float* __restrict__ Vp, const bf16* __restrict__ dO,
                                                 const float* __restrict__ dVp, const float* __restrict__ dw,
                                                 float* __restrict__ dq_out,
                                                 float* __restrict__ dk_out, float* __restrict__ dv_out,
                                                 float* __restrict__ dbeta_out, float* __restrict__ dg_out,
                                                 float* __restrict__ dA_out) {
    extern __shared__ __align__(16) unsigned char smraw[];
    bf16* ks = reinterpret_cast<bf16*>(smraw);   // k [64][136]
    bf16* qv = ks + L * kP128;                   // q, then v [64][136]
    bf16* dos = qv + L * kP128;                  // dO [64][136]
    bf16* xh = dos + L * kP128;                  // V' hi/lo, then dw hi/lo [64][136]
    bf16* xl = xh + L * kP128;
    bf16* dvh = xl + L * kP128;                  // dV' hi/lo [64][136]
    bf16* dvl = dvh + L * kP128;
    bf16* ah = dvl + L * kP128;                  // A hi/lo [64][72]
    bf16* al = ah + L * kP64;
    bf16* th = al + L * kP64;                    // gated dP, then dA, then E (hi/lo) [64][72]
    bf16* tl = th + L * kP64;
    bf16* yh = tl + L * kP64;                    // Y = dA A^T hi/lo [64][72]
    bf16* yl = yh + L * kP64;
    float* Cs = reinterpret_cast<float*>(yl + L * kP64);  // (k k^T) e^{g_i-g_l}, strict lower [64][65]
    float* gs = Cs + L * F65;
    float* bs = gs + L;
    float* dgs = bs + L;
    float* dbs = dgs + L;
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pm0 = (warp & 3) * 16, pn0 = (warp >> 2) * 32;   // [64 x 64] warp tile
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 64;     // [64 x 128] warp tile
    const bool split = (dm.flags & R97B_GDN_SPLIT_KKT) != 0;
    const int64_t nt = dm.T * dm.H * D;
    async_rows(ks, k, tok0, n, dm.Hg, hk);
    async_rows(qv, q, tok0, n, dm.Hg, hk);
    async_rows(dos, dO, tok0, n, dm.H, h);
    async_rows_pair(xh, xl, pair_of(Vp, nt), tok0, n, dm.H, h);
    async_rows_pair(dvh, dvl, pair_of(dVp, nt), tok0, n, dm.H, h);
    async_gb(gs, bs, g, beta, tok0, n, dm.H, h);
    cp_async_commit();
    // A (the caller's f32) is split by hand while the copies fly
    {
        // a thread's 16 loads issued together (a loop of load-then-split would wait out each one in turn)
        const int j = threadIdx.x & 63, i0 = threadIdx.x >> 6;  // 256 threads: rows i0, i0 + 4, ...
        float av[L / 4];
#pragma unroll
        for (int q = 0; q < L / 4; ++q) {
            const int i = i0 + 4 * q;
            av[q] = i < n ? A[((tok0 + i) * dm.H + h) * L + j] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < L / 4; ++q) put_split(ah, al, (i0 + 4 * q) * kP64 + j, av[q]);
    }
    for (int i = threadIdx.x; i < L; i += blockDim.x) {
        dgs[i] = 0.0f;
        dbs[i] = 0.0f;
    }
    cp_async_wait_all();
    __syncthreads();
    {
        float qk[1][4][4], kk[1][4][4], dp[1][4][4];
        acc_zero<16, 32>(qk);
        acc_zero<16, 32>(kk);
        acc_zero<16, 32>(dp);
        warp_mma<16, 32, 128, false, false>(qk, qv, kP128, ks, kP128, pm0, pn0);
        warp_mma<16, 32, 128, false, false>(kk, ks, kP128, ks, kP128, pm0, pn0);
        mma_split_b<16, 32, 128, false, false>(dp, dos, kP128, xh, xl, kP128, pm0, pn0);
        float r0 = 0.0f, r1 = 0.0f;
        float cs[4][2] = {};
        acc_walk<16, 32>(pm0, pn0, [&](int r, int l, int i, int j, int q) {
            const bool on = l <= r && r < n;
            // e^{g_r - g_l} only where l <= r: above the diagonal it can overflow (g decreases within a
            // chunk), and 0 * inf would poison the sums
            const float phi = on ? gexp(gs[r] - gs[l]) : 0.0f;
            const float dpv = on ? dm.scale * dp[i][j][q] : 0.0f;
            const float dd = dpv * qk[i][j][q] * phi;
            if (q >> 1) r1 += dd; else r0 += dd;
            cs[j][q & 1] -= dd;  // dd is zero off the lower triangle
            put_split(th, tl, r * kP64 + l, on ? dpv * phi : 0.0f);
            Cs[r * F65 + l] = (l < r && r < n) ? kk[i][j][q] * phi : 0.0f;
        });
        colsum_add(cs, pn0, dgs);
        r0 = quad_sum(r0);
        r1 = quad_sum(r1);
        if ((lane & 3) == 0) {
            atomicAdd(&dgs[pm0 + (lane >> 2)], r0);
            atomicAdd(&dgs[pm0 + (lane >> 2) + 8], r1);
        }
    }
    __syncthreads();
    float dqa[1][8][4], dka[1][8][4];
    acc_zero<16, 64>(dqa);
    acc_zero<16, 64>(dka);
    mma_split_a<16, 64, 64, false, true>(dqa, th, tl, kP64, ks, kP128, m0, n0);  // dq += gated dP k
    mma_split_a<16, 64, 64, true, true>(dka, th, tl, kP64, qv, kP128, m0, n0);   // dk += gated dP^T q
    __syncthreads();  // q and V' are no longer read
    async_rows(qv, v, tok0, n, dm.H, h);
    async_rows_pair(xh, xl, pair_of(dw, nt), tok0, n, dm.H, h);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    {
        // dA = dw kb^T + dV' vb^T, strict lower ; kb_j = beta_j e^{g_j} k_j, vb_j = beta_j v_j
        float a1[1][4][4], a2[1][4][4];
        acc_zero<16, 32>(a1);
        acc_zero<16, 32>(a2);
        mma_split_a<16, 32, 128, false, false>(a1, xh, xl, kP128, ks, kP128, pm0, pn0);
        mma_split_a<16, 32, 128, false, false>(a2, dvh, dvl, kP128, qv, kP128, pm0, pn0);
        float el[4][2], bl[4][2];  // this lane's eight columns l = pn0 + 8 j + 2 (lane % 4) + b
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const int l = pn0 + 8 * j + 2 * (lane & 3) + b;
                el[j][b] = gexp(gs[l]);
                bl[j][b] = bs[l];
            }
        acc_walk<16, 32>(pm0, pn0, [&](int r, int l, int i, int j, int q) {
            const float da = bl[j][q & 1] * (el[j][q & 1] * a1[i][j][q] + a2[i][j][q]);
            if (split) {  // the scan's own cotangent of A, its lower triangle with the diagonal
                if (r < n) dA_out[((tok0 + r) * dm.H + h) * L + l] = l <= r ? da : 0.0f;
            } else {
                put_split(th, tl, r * kP64 + l, l < r ? da : 0.0f);
            }
        });
    }
    {
        // dkb = A^T dw -> dk, dbeta, dg ;  dvb = A^T dV' -> dv, dbeta
        float acc[1][8][4];
        acc_zero<16, 64>(acc);
        mma_split_ab<16, 64, 64, true, true>(acc, ah, al, kP64, xh, xl, kP128, m0, n0);
        float p0 = 0.0f, p1 = 0.0f;
        const int gq = lane >> 2;  // this lane's two rows: m0 + gq and m0 + gq + 8
        const float f0 = bs[m0 + gq] * gexp(gs[m0 + gq]), f1 = bs[m0 + gq + 8] * gexp(gs[m0 + gq + 8]);
        acc_walk<16, 64>(m0, n0, [&](int r, int d, int i, int j, int q) {
            const float x = acc[i][j][q];
            const float t = __bfloat162float(ks[r * kP128 + d]) * x;
            if (q >> 1) p1 += t; else p0 += t;
            dka[i][j][q] += ((q >> 1) ? f1 : f0) * x;
        });
        p0 = quad_sum(p0);
        p1 = quad_sum(p1);
        if ((lane & 3) == 0) {
            const int ra = m0 + (lane >> 2), rb = ra + 8;
            const float ea = gexp(gs[ra]), eb = gexp(gs[rb]);
            atomicAdd(&dbs[ra], ea * p0);
            atomicAdd(&dgs[ra], bs[ra] * ea * p0);
            atomicAdd(&dbs[rb], eb * p1);
            atomicAdd(&dgs[rb], bs[rb] * eb * p1);
        }
        acc_zero<16, 64>(acc);
        mma_split_ab<16, 64, 64, true, true>(acc, ah, al, kP64, dvh, dvl, kP128, m0, n0);
        p0 = p1 = 0.0f;
        acc_pairs<16, 64>(m0, n0, [&](int r, int d, int i, int j, int hh) {  // two columns an 8-byte store
            const float x0 = acc[i][j][2 * hh], x1 = acc[i][j][2 * hh + 1];
            float& p = hh ? p1 : p0;
            const float t0 = __bfloat162float(qv[r * kP128 + d]) * x0;
            p += t0;
            const float t1 = __bfloat162float(qv[r * kP128 + d + 1]) * x1;
            p += t1;
            if (r < n)
                *reinterpret_cast<float2*>(dv_out + ((tok0 + r) * dm.H + h) * D + d) = make_float2(bs[r] * x0, bs[r] * x1);
        });
        p0 = quad_sum(p0);
        p1 = quad_sum(p1);
        if ((lane & 3) == 0) {
            atomicAdd(&dbs[m0 + (lane >> 2)], p0);
            atomicAdd(&dbs[m0 + (lane >> 2) + 8], p1);
        }
    }
    __syncthreads();
    if (!split) kkt_adjoint(ah, al, th, tl, yh, yl, ks, Cs, gs, bs, dgs, dbs, n, dka);
    __syncthreads();
    // B2a left its partials in dq, dk and dg: one reduction each adds this kernel's terms (fire-and-forget,
    // and with a single add per element the sum is the same as loading the partial and storing the total)
    acc_pairs<16, 64>(m0, n0, [&](int r, int d, int i, int j, int hh) {  // two columns an 8-byte reduction
        if (r < n) {
            const int64_t at = ((tok0 + r) * dm.H + h) * D + d;
            atomicAdd(reinterpret_cast<float2*>(dq_out + at), make_float2(dqa[i][j][2 * hh], dqa[i][j][2 * hh + 1]));
            atomicAdd(reinterpret_cast<float2*>(dk_out + at), make_float2(dka[i][j][2 * hh], dka[i][j][2 * hh + 1]));
        }
    });
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int64_t at = (tok0 + i) * dm.H + h;
        atomicAdd(dg_out + at, dgs[i]);
        dbeta_out[at] = dbs[i];
    }
}

// B3: per (chunk, value head): the solve's adjoint alone, for a caller that keeps gdn_kkt_solve and
// gdn_chunk_scan as two ops (the backward's R97B_GDN_SPLIT_KKT mode hands it the scan's dA).
// dk is per value head [T, H, 128]; dbeta and dg [T, H] are written, not added.
__global__ void __launch_bounds__(256) gdn_kkt_bwd(Dims dm, const bf16* __restrict__ k, const float* __restrict__ g,
                                                   const float* __restrict__ beta, const float* __restrict__ A,
                                                   const float* __restrict__ dA, float* __restrict__ dk_out,
                                                   float* __restrict__ dbeta_out, float* __restrict__ dg_out) {
    extern __shared__ __align__(16) unsigned char smraw[];
    bf16* ks = reinterpret_cast<bf16*>(smraw);   // k [64][136]
    bf16* ah = ks + L * kP128;                   // A hi/lo [64][72]
    bf16* al = ah + L * kP64;
    bf16* th = al + L * kP64;                    // dA, then E hi/lo [64][72]
    bf16* tl = th + L * kP64;
    bf16* yh = tl + L * kP64;                    // Y = dA A^T hi/lo [64][72]
    bf16* yl = yh + L * kP64;
    float* Cs = reinterpret_cast<float*>(yl + L * kP64);  // (k k^T) e^{g_i-g_l}, strict lower [64][65]
    float* gs = Cs + L * F65;
    float* bs = gs + L;
    float* dgs = bs + L;
    float* dbs = dgs + L;
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int warp = threadIdx.x >> 5;
    async_rows(ks, k, tok0, n, dm.Hg, hk);
    async_gb(gs, bs, g, beta, tok0, n, dm.H, h);
    cp_async_commit();
    {
        // a thread's loads issued together, as in B2b
        const int j = threadIdx.x & 63, i0 = threadIdx.x >> 6;  // 256 threads: rows i0, i0 + 4, ...
        float av[L / 4], dv[L / 4];
#pragma unroll
        for (int q = 0; q < L / 4; ++q) {
            const int i = i0 + 4 * q;
            const bool on = i < n && j <= i;
            const int64_t at = ((tok0 + i) * dm.H + h) * L + j;
            av[q] = on ? A[at] : 0.0f;
            dv[q] = on ? dA[at] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < L / 4; ++q) {
            put_split(ah, al, (i0 + 4 * q) * kP64 + j, av[q]);
            put_split(th, tl, (i0 + 4 * q) * kP64 + j, dv[q]);
        }
    }
    for (int i = threadIdx.x; i < L; i += blockDim.x) {
        dgs[i] = 0.0f;
        dbs[i] = 0.0f;
    }
    cp_async_wait_all();
    __syncthreads();
    {
        float kk[1][4][4];
        acc_zero<16, 32>(kk);
        const int pm0 = (warp & 3) * 16, pn0 = (warp >> 2) * 32;
        warp_mma<16, 32, 128, false, false>(kk, ks, kP128, ks, kP128, pm0, pn0);
        acc_for<16, 32>(kk, pm0, pn0, [&](int r, int l, float& x) {
            Cs[r * F65 + l] = (l < r && r < n) ? x * gexp(gs[r] - gs[l]) : 0.0f;
        });
    }
    __syncthreads();
    float dka[1][8][4];
    acc_zero<16, 64>(dka);
    kkt_adjoint(ah, al, th, tl, yh, yl, ks, Cs, gs, bs, dgs, dbs, n, dka);
    __syncthreads();
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 64;
    acc_for<16, 64>(dka, m0, n0, [&](int r, int d, float& x) {
        if (r < n) dk_out[((tok0 + r) * dm.H + h) * D + d] = x;
    });
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int64_t at = (tok0 + i) * dm.H + h;
        dg_out[at] = dgs[i];
        dbeta_out[at] = dbs[i];
    }
}

// dst[t, hk, :] = sum over the value heads hk * grp .. of src[t, h, :]
__global__ void gdn_sum_heads_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t T, int H, int Hg) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= T * Hg * (D / 4)) return;
    const int d4 = (int)(idx % (D / 4)) * 4;
    const int hk = (int)((idx / (D / 4)) % Hg);
    const int64_t t = idx / ((int64_t)(D / 4) * Hg);
    const int grp = H / Hg;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < grp; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(src + (t * H + hk * grp + j) * D + d4);
        s.x += v.x, s.y += v.y, s.z += v.z, s.w += v.w;
    }
    *reinterpret_cast<float4*>(dst + (t * Hg + hk) * D + d4) = s;
}

constexpr size_t kSmemPrep = (2 * L * kP128 + 4 * L * kP64) * 2 + (2 * L * F65 + 4 * L + 2 * L) * 4;
constexpr size_t kSmemState = 2 * sizeof(F2Stage) + (2 * D * P64 + 2 * L * P64) * 2;
constexpr size_t kSmemOut = (4 * L * kP128 + 2 * D * kP128 + 2 * L * kP64) * 2 + L * 4;
constexpr size_t kSmemBState = 2 * sizeof(B1Late) + sizeof(B1Early) + (2 * D * kP64 + 4 * L * kP64) * 2;
constexpr size_t kSmemBA = (4 * D * kP128 + 4 * L * kP128) * 2 + (2 * L + 8) * 4;
constexpr size_t kSmemBB = (7 * L * kP128 + 6 * L * kP64) * 2 + (L * F65 + 4 * L) * 4;
constexpr size_t kSmemKB = (L * kP128 + 6 * L * kP64) * 2 + (L * F65 + 4 * L) * 4;

// Each kernel's dynamic shared-memory opt-in on the current device; false when the runtime refuses one.
bool set_attrs() {
    return smem_opt_in(gdn_fwd_prep, (int)kSmemPrep) && smem_opt_in(gdn_fwd_state, (int)kSmemState) &&
           smem_opt_in(gdn_fwd_out, (int)kSmemOut) && smem_opt_in(gdn_bwd_state, (int)kSmemBState) &&
           smem_opt_in(gdn_bwd_a, (int)kSmemBA) && smem_opt_in(gdn_bwd_b, (int)kSmemBB) &&
           smem_opt_in(gdn_kkt_bwd, (int)kSmemKB);
}

bool dims_ok(const R97bGdnDims& d) {
    return d.n_seq > 0 && d.H > 0 && d.Hg > 0 && d.H % d.Hg == 0 && d.n_chunks >= 0 && d.T >= 0 && d.chunk_tok0 &&
           d.chunk_len && d.seq_chunk0 && d.head_k == D && d.head_v == D && d.chunk == L &&
           (d.flags & ~(R97B_GDN_A_GIVEN | R97B_GDN_SPLIT_KKT)) == 0;
}

Dims to_dims(const R97bGdnDims& d) {
    return Dims{d.n_seq, d.H, d.Hg, d.H / d.Hg, d.n_chunks, d.flags, d.T, d.scale, d.chunk_tok0, d.chunk_len, d.seq_chunk0};
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
    // u and o are written two columns at a time
    if ((reinterpret_cast<uintptr_t>(a->u) & 7) || (reinterpret_cast<uintptr_t>(a->o) & 3)) return R97B_EINVAL;
    if (!set_attrs()) return R97B_ELAUNCH;
    const Dims dm = to_dims(*dims);
    cudaStream_t s = as_stream(stream);
    const auto* q = reinterpret_cast<const bf16*>(a->q);
    const auto* k = reinterpret_cast<const bf16*>(a->k);
    const auto* v = reinterpret_cast<const bf16*>(a->v);
    if (dm.n_chunks > 0)
        gdn_fwd_prep<<<dim3(dm.n_chunks, dm.H), 256, kSmemPrep, s>>>(dm, k, v, a->g, a->beta, a->A, a->w, a->u);
    gdn_fwd_state<<<dim3(dm.n_seq, dm.H, D / VS2), 256, kSmemState, s>>>(dm, k, a->g, a->w, a->u, a->h0, a->S, a->Vp,
                                                                       a->ht);
    if (dm.n_chunks > 0)
        gdn_fwd_out<<<dim3(dm.n_chunks, dm.H), 256, kSmemOut, s>>>(dm, q, k, a->g, a->S, a->Vp, a->P,
                                                                   reinterpret_cast<bf16*>(a->o));
    return launch_status(dm.n_chunks > 0 ? 3 : 1);
}

extern "C" int r97b_gdn_bwd(const R97bGdnDims* dims, const R97bGdnBwd* a, void* stream) {
    if (!dims || !a || !dims_ok(*dims)) return R97B_EINVAL;
    if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->A || !a->w || !a->S || !a->Vp || !a->P || !a->dO ||
        !a->dS || !a->dVp || !a->dw || !a->dq || !a->dk || !a->dv || !a->dbeta ||
        !a->dg)
        return R97B_EINVAL;
    // dq, dk, dv are written two columns at a time (8-byte stores and reductions)
    if ((reinterpret_cast<uintptr_t>(a->dq) | reinterpret_cast<uintptr_t>(a->dk) | reinterpret_cast<uintptr_t>(a->dv)) & 7)
        return R97B_EINVAL;
    if ((dims->flags & R97B_GDN_SPLIT_KKT) && !a->dA) return R97B_EINVAL;
    if (!set_attrs()) return R97B_ELAUNCH;
    const Dims dm = to_dims(*dims);
    cudaStream_t s = as_stream(stream);
    const auto* q = reinterpret_cast<const bf16*>(a->q);
    const auto* k = reinterpret_cast<const bf16*>(a->k);
    const auto* v = reinterpret_cast<const bf16*>(a->v);
    const auto* dO = reinterpret_cast<const bf16*>(a->dO);
    gdn_bwd_state<<<dim3(dm.n_seq, dm.H, D / VSB), 256, kSmemBState, s>>>(dm, q, k, a->g, a->w, a->P, dO, a->dht,
                                                                        a->dS, a->dVp, a->dh0);
    if (dm.n_chunks > 0) {
        // B2a writes its partials of dq, dk, dg into the outputs; B2b adds its own terms to them
        gdn_bwd_a<<<dim3(dm.n_chunks, dm.H), 256, kSmemBA, s>>>(dm, q, k, a->g, a->S, a->Vp, dO, a->dS, a->dVp, a->dw,
                                                                a->dq, a->dk, a->dg);
        gdn_bwd_b<<<dim3(dm.n_chunks, dm.H), 256, kSmemBB, s>>>(dm, q, k, v, a->g, a->beta, a->A, a->Vp, dO, a->dVp,
                                                                a->dw, a->dq, a->dk, a->dv, a->dbeta, a->dg, a->dA);
    }
    return launch_status(dm.n_chunks > 0 ? 3 : 1);
}

extern "C" int r97b_gdn_kkt_bwd(const R97bGdnDims* dims, const uint16_t* k, const float* g, const float* beta,
                                const float* A, const float* dA, float* dk, float* dbeta, float* dg, void* stream) {
    if (!dims || !dims_ok(*dims) || !k || !g || !beta || !A || !dA || !dk || !dbeta || !dg) return R97B_EINVAL;
    if (dims->n_chunks == 0) return R97B_OK;
    if (!set_attrs()) return R97B_ELAUNCH;
    const Dims dm = to_dims(*dims);
    gdn_kkt_bwd<<<dim3(dm.n_chunks, dm.H), 256, kSmemKB, as_stream(stream)>>>(
        dm, reinterpret_cast<const bf16*>(k), g, beta, A, dA, dk, dbeta, dg);
    return launch_status();
}

extern "C" int r97b_gdn_sum_heads(const float* src, float* dst, int64_t T, int32_t H, int32_t Hg, void* stream) {
    if (!src || !dst || T < 0 || H <= 0 || Hg <= 0 || H % Hg) return R97B_EINVAL;
    const int64_t total = T * Hg * (128 / 4);
    if (total == 0) return R97B_OK;
    gdn_sum_heads_kernel<<<(unsigned)((total + 255) / 256), 256, 0, as_stream(stream)>>>(src, dst, T, H, Hg);
    return launch_status();
}
