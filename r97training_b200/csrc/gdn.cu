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
// Every product runs on the tensor cores, bf16 in and f32 accumulate. F1, F2, F3, B1 and B2a are tcgen05
// kernels (tc_tile.cuh: swizzled shared-memory tiles, one thread issuing the MMAs, f32 accumulators in
// TMEM; the state passes keep their state in registers laid out as the accumulator); B2b and the
// standalone solve adjoint B3 use warp mma.sync (wmma16.cuh), whose register-resident 64 x 64 products
// measured faster for B2b's chain of small intra-chunk products than a tcgen05 form (668 against 1008 us
// for a config-5 layer). q, k, v and dO are bf16 already and enter exactly; an f32 operand (a state, A, P,
// V', w, dV', ...) is split into bf16 hi + lo tiles and its product takes two or three passes, which keeps
// ~16 bits of the operand. Only the 64-step forward substitution of the solve runs on CUDA cores.
//
// Sequences are ragged (cu_seqlens); a sequence's last chunk may be short, and its padded rows are zero
// so they add nothing. Head dims K = V = 128 and the chunk of 64 are fixed here.
#include "r97b_internal.h"
#include "fastmath.cuh"
#include "wmma16.cuh"
#include "tc_tile.cuh"

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

// F1: per (chunk, value head): A = (I + M)^-1, w = (A diag(beta e^g)) k, u = (A diag(beta)) v, on tcgen05
// for the products: k k^T (M = 128 rows of which the chunk's 64 are read), then w^T = k^T (A diag(beta e^g))^T
// and u^T = v^T (A diag(beta))^T with the 128 lanes as M (the A factors as bf16 (hi, lo) tiles, two passes).
// The solve stays on CUDA cores in f32. TMEM: k k^T at column 0, w^T at 64, u^T at 128.
namespace f1 {
constexpr int kK = 0;
constexpr int kV = kK + tc::kRowTile;
constexpr int kA1h = kV + tc::kRowTile;     // A diag(beta e^g) hi/lo [64][64]; before the solve ends, its scratch
constexpr int kA1l = kA1h + tc::kSqTile;
constexpr int kA2h = kA1l + tc::kSqTile;    // A diag(beta) hi/lo
constexpr int kA2l = kA2h + tc::kSqTile;
constexpr int kMs = kA2l + tc::kSqTile;     // f32 [64][65]
constexpr int kAs = kMs + L * F65 * 4;      // f32 [64][65]
constexpr int kG = kAs + L * F65 * 4;       // g, beta [64] each
constexpr int kBar = kG + 2 * L * 4;
constexpr int kUsed = kBar + 16;
}  // namespace f1

__global__ void __launch_bounds__(256) gdn_fwd_prep(Dims dm, const bf16* __restrict__ k, const bf16* __restrict__ v,
                                                    const float* __restrict__ g, const float* __restrict__ beta,
                                                    float* __restrict__ A, float* __restrict__ w, float* __restrict__ u) {
    using namespace f1;
    extern __shared__ unsigned char smraw[];
    unsigned char* sm = tc::align1024(smraw);
    unsigned char *Ks = sm + kK, *Vs = sm + kV, *A1h = sm + kA1h, *A1l = sm + kA1l, *A2h = sm + kA2h, *A2l = sm + kA2l;
    float* Ms = reinterpret_cast<float*>(sm + kMs);
    float* As = reinterpret_cast<float*>(sm + kAs);
    float* gs = reinterpret_cast<float*>(sm + kG);
    float* bs = gs + L;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kBar);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kBar + 8);
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3, ch = warp >> 2;
    const bool given = (dm.flags & R97B_GDN_A_GIVEN) != 0;
    tc::stage_rows(Ks, k, tok0, n, dm.Hg, hk);
    tc::stage_rows(Vs, v, tok0, n, dm.H, h);
    async_gb(gs, bs, g, beta, tok0, n, dm.H, h);
    cp_async_commit();
    if (given) {  // the caller's solve: its lower triangle, diagonal included, for the chunk's rows
        const int j = threadIdx.x & 63, i0 = threadIdx.x >> 6;  // 256 threads: rows i0, i0 + 4, ...
        float av[L / 4];
#pragma unroll
        for (int s = 0; s < L / 4; ++s) {  // every load issued before the first store
            const int i = i0 + 4 * s;
            av[s] = (i < n && j <= i) ? A[((tok0 + i) * dm.H + h) * L + j] : 0.0f;
        }
#pragma unroll
        for (int s = 0; s < L / 4; ++s) As[(i0 + 4 * s) * F65 + j] = av[s];
    }
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(tslot, 256);
        tmem_relinquish();
    }
    cp_async_wait_all();
    tc::fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tslot;
    const uint32_t tq = tm + ((uint32_t)(32 * qd) << 16) + (uint32_t)(32 * ch);
    constexpr uint32_t id = make_idesc_bf16(128, 64, 0, 0);
    constexpr uint32_t id_a = make_idesc_bf16(128, 64, 1, 0);  // A MN-major
    const uint32_t sk = smem_u32(Ks), sv = smem_u32(Vs);
    uint32_t phase = 0;
    bool ok = true;
    if (!given) {
        // M = strict lower of beta_i (k_i . k_l) e^{g_i - g_l}
        if (threadIdx.x == 0) {
            for (int kk = 0; kk < 8; ++kk)
                umma_f16(tm, tc::kdesc(sk, 64, 0, kk), tc::kdesc(sk, 64, 0, kk), id, kk > 0 ? 1u : 0u);
            umma_commit(bar);
        }
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar, phase, nullptr));
        phase ^= 1u;
        tc_fence_after();
        if (ok && qd < 2) {
            const int r = 32 * qd + lane;
            float x[32];
            tc::tmem_row32(tq, x);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int l = 32 * ch + i;
                // only the chunk's own rows: a padded row's g is 0, and e^{0 - g_l} can overflow to inf, whose
                // 0 * inf the blocked inverse would carry into every row
                Ms[r * F65 + l] = (l < r && r < n) ? bs[r] * x[i] * gexp(gs[r] - gs[l]) : 0.0f;
            }
        }
        __syncthreads();
        // A = (I + M)^-1 by blocks: the four 16x16 diagonal blocks by forward substitution (a warp each),
        // then 16 -> 32 -> 64 with X21 = -A22 (M21 A11) (the inverse of a block lower-triangular matrix)
        invert_unit_lower(Ms, As, reinterpret_cast<float*>(A1h));
    }
    {
        const int j = threadIdx.x & 63;  // a thread keeps its column (the stride is a multiple of 64)
        const float e = bs[j] * gexp(gs[j]), bj = bs[j];
        for (int i = threadIdx.x >> 6; i < L; i += blockDim.x >> 6) {
            const float a = As[i * F65 + j];
            if (i < n && !given) A[((tok0 + i) * dm.H + h) * L + j] = a;
            __nv_bfloat16 hi, lo;
            const uint32_t o = tc::elem_off(64, i, j);
            split_bf16(a * e, hi, lo);
            *reinterpret_cast<__nv_bfloat16*>(A1h + o) = hi;
            *reinterpret_cast<__nv_bfloat16*>(A1l + o) = lo;
            split_bf16(a * bj, hi, lo);
            *reinterpret_cast<__nv_bfloat16*>(A2h + o) = hi;
            *reinterpret_cast<__nv_bfloat16*>(A2l + o) = lo;
        }
    }
    tc::fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0 && ok) {
        const uint32_t a1h = smem_u32(A1h), a1l = smem_u32(A1l), a2h = smem_u32(A2h), a2l = smem_u32(A2l);
        // w^T = k^T a1^T, u^T = v^T a2^T (a1, a2: hi, lo)
        for (int kk = 0; kk < 4; ++kk)
            umma_f16(tm + 64, tc::mdesc(sk, 64, 0, kk), tc::kdesc(a1h, 64, 0, kk), id_a, kk > 0 ? 1u : 0u);
        for (int kk = 0; kk < 4; ++kk) umma_f16(tm + 64, tc::mdesc(sk, 64, 0, kk), tc::kdesc(a1l, 64, 0, kk), id_a, 1u);
        for (int kk = 0; kk < 4; ++kk)
            umma_f16(tm + 128, tc::mdesc(sv, 64, 0, kk), tc::kdesc(a2h, 64, 0, kk), id_a, kk > 0 ? 1u : 0u);
        for (int kk = 0; kk < 4; ++kk) umma_f16(tm + 128, tc::mdesc(sv, 64, 0, kk), tc::kdesc(a2l, 64, 0, kk), id_a, 1u);
        umma_commit(bar);
    }
    ok = __all_sync(0xFFFFFFFFu, ok && mbar_wait(bar, phase, nullptr));
    tc_fence_after();
    if (ok) {
        // lane d = 32 (warp % 4) + lane of the chunk's tokens 32 (warp / 4) ..: w as a (hi, lo) pair in the
        // bytes of an f32 [T, H, 128] buffer, u in f32
        const int d = 32 * qd + lane;
        bf16* w_hi = reinterpret_cast<bf16*>(w);
        bf16* w_lo = w_hi + (int64_t)dm.T * dm.H * D;
        float x[32];
        tc::tmem_row32(tq + 64, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int r = 32 * ch + i;
            if (r < n) put_split(w_hi, w_lo, ((tok0 + r) * dm.H + h) * D + d, x[i]);
        }
        tc::tmem_row32(tq + 128, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int r = 32 * ch + i;
            if (r < n) u[((tok0 + r) * dm.H + h) * D + d] = x[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, 256);
}

// F2: per (sequence, value head, 64 value lanes): the state pass over the sequence's chunks, on tcgen05.
// The state slice S[128 key lanes][64 value lanes] stays in registers in the accumulator's TMEM layout (key
// lane d = 32 (warp % 4) + lane, value lanes 32 (warp / 4) .. + 31), and each chunk takes two products:
// W' = w S (M = the chunk's 64 tokens, the upper half of the 128-row MMA unused; w and S as bf16 (hi, lo)
// tiles, three passes), giving V' = u - W' and V'' = e^{gL - g} V'; then k^T V'' (M = the 128 key lanes,
// two passes), added to e^{gL} S. A chunk's w pair, k, u slice and g stream into a double-buffered stage
// by cp.async while the previous chunk computes. TMEM: W' at column 0, k^T V'' at 64.
namespace f2 {
constexpr int kWh = 0;
constexpr int kWl = kWh + tc::kRowTile;
constexpr int kK = kWl + tc::kRowTile;
constexpr int kU = kK + tc::kRowTile;        // u slice, f32 [64][68]
constexpr int kUP = 68;                       // its pitch: a quarter-warp's 16-byte row reads hit distinct banks
constexpr int kG = kU + L * kUP * 4;
constexpr int kStage = ((kG + L * 4) + 1023) & ~1023;
constexpr int kSh = 2 * kStage;               // S hi/lo [128][64]
constexpr int kSl = kSh + 128 * 64 * 2;
constexpr int kVh = kSl + 128 * 64 * 2;       // V'' hi/lo [64][64]
constexpr int kVl = kVh + tc::kSqTile;
constexpr int kOh = kVl + tc::kSqTile;        // V' hi/lo [64][64], staged for its coalesced copy out
constexpr int kOl = kOh + tc::kSqTile;
constexpr int kBar = kOl + tc::kSqTile;       // mbarrier, abort flag, TMEM slot
constexpr int kUsed = kBar + 16;
}  // namespace f2

__device__ __forceinline__ void f2_issue(unsigned char* st, const Dims& dm, const bf16* w_hi, const bf16* w_lo,
                                         const bf16* k, const float* u, const float* g, int c, int h, int hk, int e0) {
    using namespace f2;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    tc::stage_rows(st + kWh, w_hi, tok0, n, dm.H, h);
    tc::stage_rows(st + kWl, w_lo, tok0, n, dm.H, h);
    tc::stage_rows(st + kK, k, tok0, n, dm.Hg, hk);
    float* us = reinterpret_cast<float*>(st + kU);
    for (int idx = threadIdx.x; idx < L * 16; idx += blockDim.x) {
        const int i = idx >> 4, q = (idx & 15) * 4;
        const bool on = i < n;
        cp_async16(us + i * kUP + q, u + ((on ? tok0 + i : tok0) * dm.H + h) * D + e0 + q, on);
    }
    async_gb(reinterpret_cast<float*>(st + kG), nullptr, g, nullptr, tok0, n, dm.H, h);
    cp_async_commit();
}

__global__ void __launch_bounds__(256) gdn_fwd_state(Dims dm, const bf16* __restrict__ k, const float* __restrict__ g,
                                                     const float* __restrict__ w, const float* __restrict__ u,
                                                     const float* __restrict__ h0, float* __restrict__ S_all,
                                                     float* __restrict__ Vp, float* __restrict__ ht) {
    using namespace f2;
    extern __shared__ unsigned char smraw[];
    unsigned char* sm = tc::align1024(smraw);
    unsigned char *Sh = sm + kSh, *Sl = sm + kSl, *Vh = sm + kVh, *Vl = sm + kVl, *Oh = sm + kOh, *Ol = sm + kOl;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kBar);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + kBar + 8);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kBar + 12);
    const bf16* w_hi = reinterpret_cast<const bf16*>(w);
    const bf16* w_lo = w_hi + dm.T * dm.H * D;
    const int seq = blockIdx.x, h = blockIdx.y, e0 = blockIdx.z * 64, hk = h / dm.grp;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3, ch = warp >> 2;
    const int d = 32 * qd + lane;  // this thread's key lane; its value lanes are e0 + 32 ch .. + 31
    const int c0 = dm.seq_c0[seq], c1 = dm.seq_c0[seq + 1];
    if (c0 < c1) f2_issue(sm, dm, w_hi, w_lo, k, u, g, c0, h, hk, e0);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(tslot, 128);
        tmem_relinquish();
    }
    float S[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
        S[i] = h0 ? h0[(((int64_t)seq * dm.H + h) * D + e0 + 32 * ch + i) * D + d] : 0.0f;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tslot;
    const uint32_t tq = tm + ((uint32_t)(32 * qd) << 16) + (uint32_t)(32 * ch);
    constexpr uint32_t id_b = make_idesc_bf16(128, 64, 0, 1);   // B MN-major
    constexpr uint32_t id_ab = make_idesc_bf16(128, 64, 1, 1);  // A, B MN-major
    const Pair Sp = pair_of(S_all, (int64_t)dm.n_chunks * dm.H * D * D);
    const Pair Vpp = pair_of(Vp, dm.T * dm.H * D);
    uint32_t phase = 0;
    for (int c = c0; c < c1; ++c) {
        unsigned char* st = sm + ((c - c0) & 1) * kStage;
        const int64_t tok0 = dm.tok0[c];
        const int n = dm.len[c];
        // the state entering chunk c: its tiles, then S_all[c] copied out of them
        tc::put_row32(Sh, Sl, 128, d, 32 * ch, S);
        cp_async_wait_all();
        tc::fence_proxy_async();
        tc_fence_before();
        __syncthreads();  // chunk c's stage landed; the S tiles written; chunk c-1's products are done
        tc_fence_after();
        if (*abort_flag) break;
        tc::tile_to_global(Sh, Sl, 128, 128, Sp.hi, Sp.lo, ((int64_t)c * dm.H + h) * D * D + e0, D);
        if (c + 1 < c1) f2_issue(sm + ((c + 1 - c0) & 1) * kStage, dm, w_hi, w_lo, k, u, g, c + 1, h, hk, e0);
        const uint32_t swh = smem_u32(st + kWh), swl = smem_u32(st + kWl), sk = smem_u32(st + kK);
        const uint32_t ssh = smem_u32(Sh), ssl = smem_u32(Sl), svh = smem_u32(Vh), svl = smem_u32(Vl);
        if (threadIdx.x == 0) {
            // W' = w S: hi hi, lo hi, hi lo
            for (int kk = 0; kk < 8; ++kk)
                umma_f16(tm, tc::kdesc(swh, 64, 0, kk), tc::mdesc(ssh, 128, 0, kk), id_b, kk > 0 ? 1u : 0u);
            for (int kk = 0; kk < 8; ++kk) umma_f16(tm, tc::kdesc(swl, 64, 0, kk), tc::mdesc(ssh, 128, 0, kk), id_b, 1u);
            for (int kk = 0; kk < 8; ++kk) umma_f16(tm, tc::kdesc(swh, 64, 0, kk), tc::mdesc(ssl, 128, 0, kk), id_b, 1u);
            umma_commit(bar);
        }
        bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar, phase, abort_flag));
        phase ^= 1u;
        tc_fence_after();
        const float* gs = reinterpret_cast<const float*>(st + kG);
        const float gl = gs[n - 1];
        if (ok && qd < 2) {
            // V' = u - w S for token i = d (lanes 0 .. 63 hold the chunk's rows), value lanes 32 ch ..
            const int i = d;
            float x[32];
            tc::tmem_row32(tq, x);
            const float* ur = reinterpret_cast<const float*>(st + kU) + i * kUP + 32 * ch;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 u4 = *reinterpret_cast<const float4*>(ur + 4 * j);
                x[4 * j] = u4.x - x[4 * j];
                x[4 * j + 1] = u4.y - x[4 * j + 1];
                x[4 * j + 2] = u4.z - x[4 * j + 2];
                x[4 * j + 3] = u4.w - x[4 * j + 3];
            }
            tc::put_row32(Oh, Ol, 64, i, 32 * ch, x);
            const float sc = i < n ? gexp(gl - gs[i]) : 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) x[j] *= sc;
            tc::put_row32(Vh, Vl, 64, i, 32 * ch, x);
        }
        tc::fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        tc::tile_to_global(Oh, Ol, 64, n, Vpp.hi, Vpp.lo, (tok0 * dm.H + h) * D + e0, (int64_t)dm.H * D);
        if (threadIdx.x == 0 && !*abort_flag) {
            // k^T V'' (V'': hi, lo)
            for (int kk = 0; kk < 4; ++kk)
                umma_f16(tm + 64, tc::mdesc(sk, 64, 0, kk), tc::mdesc(svh, 64, 0, kk), id_ab, kk > 0 ? 1u : 0u);
            for (int kk = 0; kk < 4; ++kk) umma_f16(tm + 64, tc::mdesc(sk, 64, 0, kk), tc::mdesc(svl, 64, 0, kk), id_ab, 1u);
            umma_commit(bar);
        }
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar, phase, abort_flag));
        phase ^= 1u;
        tc_fence_after();
        if (ok) {
            const float el = gexp(gl);
            float p[32];
            tc::tmem_row32(tq + 64, p);
#pragma unroll
            for (int j = 0; j < 32; ++j) S[j] = el * S[j] + p[j];
        }
    }
    if (ht)
#pragma unroll
        for (int i = 0; i < 32; ++i) ht[(((int64_t)seq * dm.H + h) * D + e0 + 32 * ch + i) * D + d] = S[i];
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, 128);
}

// F3: per (chunk, value head): P and the output rows, on tcgen05. [q; k] k^T (M = 128, one [128][128] tile
// of q over k) gives q k^T in its first 64 rows; the output is formed transposed, value lanes as M:
// o^T = scale (S^T q^T e^g + V'^T P^T), the two products in separate TMEM blocks because only the first is
// scaled per token. S, V' and P enter as bf16 (hi, lo) tiles: two passes for S^T q^T, three for V'^T P^T.
// TMEM: q k^T at column 0, S^T q^T at 64, V'^T P^T at 128.
namespace f3 {
constexpr int kQK = 0;
constexpr int kSh = kQK + tc::kBlockTile;
constexpr int kSl = kSh + tc::kBlockTile;
constexpr int kVh = kSl + tc::kBlockTile;
constexpr int kVl = kVh + tc::kRowTile;
constexpr int kPh = kVl + tc::kRowTile;
constexpr int kPl = kPh + tc::kSqTile;
constexpr int kG = kPl + tc::kSqTile;
constexpr int kBar = kG + L * 4;
constexpr int kUsed = kBar + 16;
}  // namespace f3

__global__ void __launch_bounds__(256) gdn_fwd_out(Dims dm, const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                   const float* __restrict__ g, const float* __restrict__ S_all,
                                                   const float* __restrict__ Vp, float* __restrict__ P_all,
                                                   bf16* __restrict__ o) {
    using namespace f3;
    extern __shared__ unsigned char smraw[];
    unsigned char* sm = tc::align1024(smraw);
    unsigned char *QK = sm + kQK, *Sh = sm + kSh, *Sl = sm + kSl, *Vh = sm + kVh, *Vl = sm + kVl, *Ph = sm + kPh,
                  *Pl = sm + kPl;
    float* gs = reinterpret_cast<float*>(sm + kG);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kBar);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nb = (int64_t)dm.n_chunks * dm.H * D * D, nt = dm.T * dm.H * D;
    const int64_t blk = (int64_t)c * dm.H + h;
    const Pair Sp = pair_of(S_all, nb), Vpp = pair_of(Vp, nt);
    tc::stage_rows(QK, q, tok0, n, dm.Hg, hk, 128, 0);
    tc::stage_rows(QK, k, tok0, n, dm.Hg, hk, 128, 64);
    async_gb(gs, nullptr, g, nullptr, tok0, n, dm.H, h);
    cp_async_commit();
    tc::stage_block(Sh, Sp.hi + blk * D * D);
    tc::stage_block(Sl, Sp.lo + blk * D * D);
    tc::stage_rows(Vh, Vpp.hi, tok0, n, dm.H, h);
    tc::stage_rows(Vl, Vpp.lo, tok0, n, dm.H, h);
    cp_async_commit();
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(tslot, 256);
        tmem_relinquish();
    }
    cp_async_wait_but_one();
    tc::fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tslot;
    constexpr uint32_t id = make_idesc_bf16(128, 64, 0, 0);
    constexpr uint32_t id_m = make_idesc_bf16(128, 64, 1, 0);
    const uint32_t sQK = smem_u32(QK), sSh = smem_u32(Sh), sSl = smem_u32(Sl), sVh = smem_u32(Vh),
                   sVl = smem_u32(Vl), sPh = smem_u32(Ph), sPl = smem_u32(Pl);
    if (threadIdx.x == 0) {
        for (int kk = 0; kk < 8; ++kk)
            umma_f16(tm, tc::kdesc(sQK, 128, 0, kk), tc::kdesc(sQK, 128, 64, kk), id, kk > 0 ? 1u : 0u);
        umma_commit(bar);
    }
    bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar, 0, nullptr));
    tc_fence_after();
    const int qd = warp & 3, ch = warp >> 2;
    const uint32_t tq = tm + ((uint32_t)(32 * qd) << 16) + (uint32_t)(32 * ch);
    if (ok && qd < 2) {
        // P = causal(q k^T e^{g_r - g_l}), kept as a bf16 (hi, lo) pair in the bytes of an f32
        // [chunks, H, 64, 64] buffer, and as the tiles the P V' product reads
        const int r = 32 * qd + lane;
        float p[32];
        tc::tmem_row32(tq, p);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int l = 32 * ch + i;
            p[i] = (l <= r && r < n) ? p[i] * gexp(gs[r] - gs[l]) : 0.0f;
        }
        tc::put_row32(Ph, Pl, 64, r, 32 * ch, p);
    }
    cp_async_wait_all();
    tc::fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    {
        const Pair Pp = pair_of(P_all, (int64_t)dm.n_chunks * dm.H * L * L);
        tc::tile_to_global(Ph, Pl, 64, 64, Pp.hi, Pp.lo, blk * L * L, L);
    }
    if (threadIdx.x == 0 && ok) {
        // S^T q^T (S: hi, lo) ; V'^T P^T (hi hi, lo hi, hi lo)
        for (int kk = 0; kk < 8; ++kk)
            umma_f16(tm + 64, tc::mdesc(sSh, 128, 0, kk), tc::kdesc(sQK, 128, 0, kk), id_m, kk > 0 ? 1u : 0u);
        for (int kk = 0; kk < 8; ++kk) umma_f16(tm + 64, tc::mdesc(sSl, 128, 0, kk), tc::kdesc(sQK, 128, 0, kk), id_m, 1u);
        for (int kk = 0; kk < 4; ++kk)
            umma_f16(tm + 128, tc::mdesc(sVh, 64, 0, kk), tc::kdesc(sPh, 64, 0, kk), id_m, kk > 0 ? 1u : 0u);
        for (int kk = 0; kk < 4; ++kk) umma_f16(tm + 128, tc::mdesc(sVl, 64, 0, kk), tc::kdesc(sPh, 64, 0, kk), id_m, 1u);
        for (int kk = 0; kk < 4; ++kk) umma_f16(tm + 128, tc::mdesc(sVh, 64, 0, kk), tc::kdesc(sPl, 64, 0, kk), id_m, 1u);
        umma_commit(bar);
    }
    ok = __all_sync(0xFFFFFFFFu, ok && mbar_wait(bar, 1, nullptr));
    tc_fence_after();
    if (ok) {
        // o = scale (e^g q S + P V'): value lane e = 32 (warp % 4) + lane, tokens 32 (warp / 4) ..
        const int e = 32 * qd + lane;
        float a[32], b[32];
        tc::tmem_row32(tq + 64, a);
        tc::tmem_row32(tq + 128, b);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int r = 32 * ch + i;
            if (r < n) o[((tok0 + r) * dm.H + h) * D + e] = __float2bfloat16_rn(dm.scale * (a[i] * gexp(gs[r]) + b[i]));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, 256);
}

// ============================================================================================ backward

// B1: per (sequence, value head, 64 value lanes): the reverse state pass, on tcgen05. dS[128 key lanes]
// [64 value lanes] stays in registers in the accumulator's TMEM layout (as F2's S), and each chunk takes
// two rounds of products: dV' = scale P^T dO + e^{gL - g} (k dS) (M = the chunk's 64 tokens, the upper half
// of the 128-row MMA unused; P and dS as bf16 (hi, lo) tiles, two passes each); then q^T (e^g dO) and
// w^T dV' (M = the 128 key lanes; two and three passes), which update dS = e^{gL} dS + scale q^T (e^g dO)
// - w^T dV'. The operands read late in a chunk (w as a pair, q) are double-buffered and fetched a whole
// chunk ahead; the ones the dV' products read (P as a pair, k, the dO slice, g) have one buffer, refilled
// for the next chunk as soon as those products are done. TMEM: P^T dO 0, k dS 64, q^T (e^g dO) 128,
// w^T dV' 192.
namespace b1 {
constexpr int kLateWh = 0;                        // a late stage: w hi/lo, q [64][128]
constexpr int kLateWl = kLateWh + tc::kRowTile;
constexpr int kLateQ = kLateWl + tc::kRowTile;
constexpr int kLate = kLateQ + tc::kRowTile;
constexpr int kEarly = 2 * kLate;                 // P hi/lo [64][64], k [64][128], dO slice [64][64], g
constexpr int kPh = kEarly;
constexpr int kPl = kPh + tc::kSqTile;
constexpr int kK = kPl + tc::kSqTile;
constexpr int kDO = kK + tc::kRowTile;
constexpr int kG = kDO + tc::kSqTile;
constexpr int kDSh = (kG + L * 4 + 1023) & ~1023; // dS hi/lo [128][64]
constexpr int kDSl = kDSh + 128 * 64 * 2;
constexpr int kEGh = kDSl + 128 * 64 * 2;         // e^g dO hi/lo [64][64]
constexpr int kEGl = kEGh + tc::kSqTile;
constexpr int kDVh = kEGl + tc::kSqTile;          // dV' hi/lo [64][64]
constexpr int kDVl = kDVh + tc::kSqTile;
constexpr int kBar = kDVl + tc::kSqTile;          // mbarrier, abort flag, TMEM slot
constexpr int kUsed = kBar + 16;
}  // namespace b1

__device__ __forceinline__ void b1_issue_late(unsigned char* st, const Dims& dm, const bf16* q, const bf16* w_hi,
                                              const bf16* w_lo, int c, int h, int hk) {
    using namespace b1;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    tc::stage_rows(st + kLateWh, w_hi, tok0, n, dm.H, h);
    tc::stage_rows(st + kLateWl, w_lo, tok0, n, dm.H, h);
    tc::stage_rows(st + kLateQ, q, tok0, n, dm.Hg, hk);
    cp_async_commit();
}

__device__ __forceinline__ void b1_issue_early(unsigned char* sm, const Dims& dm, const bf16* k, const bf16* P_hi,
                                               const bf16* P_lo, const bf16* dO, const float* g, int c, int h,
                                               int hk, int e0) {
    using namespace b1;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int64_t pbase = ((int64_t)c * dm.H + h) * L * L;
    tc::stage_rows(sm + kK, k, tok0, n, dm.Hg, hk);
    for (int idx = threadIdx.x; idx < L * 8; idx += blockDim.x) {
        const int i = idx >> 3, j = idx & 7;
        const bool on = i < n;
        const uint32_t o = tc::chunk_off(64, i, j);
        cp_async16(sm + kPh + o, P_hi + pbase + i * L + j * 8, true);
        cp_async16(sm + kPl + o, P_lo + pbase + i * L + j * 8, true);
        cp_async16(sm + kDO + o, dO + ((on ? tok0 + i : tok0) * dm.H + h) * D + e0 + j * 8, on);
    }
    async_gb(reinterpret_cast<float*>(sm + kG), nullptr, g, nullptr, tok0, n, dm.H, h);
    cp_async_commit();
}

__global__ void __launch_bounds__(256) gdn_bwd_state(Dims dm, const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                     const float* __restrict__ g, const float* __restrict__ w,
                                                     const float* __restrict__ P_all, const bf16* __restrict__ dO,
                                                     const float* __restrict__ dht, float* __restrict__ dS_all,
                                                     float* __restrict__ dVp, float* __restrict__ dh0) {
    using namespace b1;
    extern __shared__ unsigned char smraw[];
    unsigned char* sm = tc::align1024(smraw);
    unsigned char *DSh = sm + kDSh, *DSl = sm + kDSl, *EGh = sm + kEGh, *EGl = sm + kEGl, *DVh = sm + kDVh,
                  *DVl = sm + kDVl;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kBar);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + kBar + 8);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kBar + 12);
    const bf16* w_hi = reinterpret_cast<const bf16*>(w);
    const bf16* w_lo = w_hi + dm.T * dm.H * D;
    const bf16* P_hi = reinterpret_cast<const bf16*>(P_all);
    const bf16* P_lo = P_hi + (int64_t)dm.n_chunks * dm.H * L * L;
    const int seq = blockIdx.x, h = blockIdx.y, e0 = blockIdx.z * 64, hk = h / dm.grp;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, qd = warp & 3, ch = warp >> 2;
    const int d = 32 * qd + lane;  // this thread's key lane; its value lanes are e0 + 32 ch .. + 31
    const Pair dSp = pair_of(dS_all, (int64_t)dm.n_chunks * dm.H * D * D);
    const Pair dVpp = pair_of(dVp, dm.T * dm.H * D);
    const int c0 = dm.seq_c0[seq], c1 = dm.seq_c0[seq + 1];
    if (c0 < c1) {
        b1_issue_late(sm, dm, q, w_hi, w_lo, c1 - 1, h, hk);
        b1_issue_early(sm, dm, k, P_hi, P_lo, dO, g, c1 - 1, h, hk, e0);
    }
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(tslot, 256);
        tmem_relinquish();
    }
    float dS[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
        dS[i] = dht ? dht[(((int64_t)seq * dm.H + h) * D + e0 + 32 * ch + i) * D + d] : 0.0f;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tslot;
    const uint32_t tq = tm + ((uint32_t)(32 * qd) << 16) + (uint32_t)(32 * ch);
    constexpr uint32_t id_b = make_idesc_bf16(128, 64, 0, 1);   // B MN-major
    constexpr uint32_t id_ab = make_idesc_bf16(128, 64, 1, 1);  // A, B MN-major
    const uint32_t sph = smem_u32(sm + kPh), spl = smem_u32(sm + kPl), sk = smem_u32(sm + kK),
                   sdo = smem_u32(sm + kDO), sdsh = smem_u32(DSh), sdsl = smem_u32(DSl), segh = smem_u32(EGh),
                   segl = smem_u32(EGl), sdvh = smem_u32(DVh), sdvl = smem_u32(DVl);
    const float* gs = reinterpret_cast<const float*>(sm + kG);
    uint32_t phase = 0;
    for (int c = c1 - 1; c >= c0; --c) {
        unsigned char* lt = sm + ((c1 - 1 - c) & 1) * kLate;
        const int64_t tok0 = dm.tok0[c];
        const int n = dm.len[c];
        // dS entering (from the right) chunk c: its tiles, then dS_all[c] copied out of them
        tc::put_row32(DSh, DSl, 128, d, 32 * ch, dS);
        cp_async_wait_all();
        tc::fence_proxy_async();
        tc_fence_before();
        __syncthreads();  // chunk c's operands landed; the dS tiles written; chunk c+1's products are done
        tc_fence_after();
        if (*abort_flag) break;
        tc::tile_to_global(DSh, DSl, 128, 128, dSp.hi, dSp.lo, ((int64_t)c * dm.H + h) * D * D + e0, D);
        if (c > c0) b1_issue_late(sm + ((c1 - c) & 1) * kLate, dm, q, w_hi, w_lo, c - 1, h, hk);
        if (threadIdx.x == 0) {
            // P^T dO (P: hi, lo) ; k dS (dS: hi, lo)
            for (int kk = 0; kk < 4; ++kk)
                umma_f16(tm, tc::mdesc(sph, 64, 0, kk), tc::mdesc(sdo, 64, 0, kk), id_ab, kk > 0 ? 1u : 0u);
            for (int kk = 0; kk < 4; ++kk) umma_f16(tm, tc::mdesc(spl, 64, 0, kk), tc::mdesc(sdo, 64, 0, kk), id_ab, 1u);
            for (int kk = 0; kk < 8; ++kk)
                umma_f16(tm + 64, tc::kdesc(sk, 64, 0, kk), tc::mdesc(sdsh, 128, 0, kk), id_b, kk > 0 ? 1u : 0u);
            for (int kk = 0; kk < 8; ++kk) umma_f16(tm + 64, tc::kdesc(sk, 64, 0, kk), tc::mdesc(sdsl, 128, 0, kk), id_b, 1u);
            umma_commit(bar);
        }
        const float gl = gs[n - 1];
        // e^g dO as (hi, lo) tiles for the dS products, while the dV' products run
        for (int idx = threadIdx.x; idx < L * 8; idx += blockDim.x) {
            const int i = idx >> 3, j = idx & 7;
            const float eg = gexp(gs[i]);
            const uint32_t o = tc::chunk_off(64, i, j);
            const uint4 raw = *reinterpret_cast<const uint4*>(sm + kDO + o);
            const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(x2[e]);
                const float a = f.x * eg, b = f.y * eg;
                const __nv_bfloat162 hh = __floats2bfloat162_rn(a, b);
                const float2 hf = __bfloat1622float2(hh);
                const __nv_bfloat162 ll = __floats2bfloat162_rn(a - hf.x, b - hf.y);
                hw[e] = *reinterpret_cast<const uint32_t*>(&hh);
                lw[e] = *reinterpret_cast<const uint32_t*>(&ll);
            }
            *reinterpret_cast<uint4*>(EGh + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(EGl + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar, phase, abort_flag));
        phase ^= 1u;
        tc_fence_after();
        if (ok && qd < 2) {
            // dV' = scale P^T dO + e^{gL - g} (k dS) for token j = d, value lanes 32 ch ..
            const int j = d;
            float a1[32], a2[32];
            tc::tmem_row32(tq, a1);
            tc::tmem_row32(tq + 64, a2);
            const float sc = j < n ? gexp(gl - gs[j]) : 0.0f;
#pragma unroll
            for (int e = 0; e < 32; ++e) a1[e] = j < n ? dm.scale * a1[e] + sc * a2[e] : 0.0f;
            tc::put_row32(DVh, DVl, 64, j, 32 * ch, a1);
        }
        tc::fence_proxy_async();
        tc_fence_before();
        __syncthreads();  // dV' and e^g dO written; chunk c's P, k, dO and g are no longer read
        tc_fence_after();
        tc::tile_to_global(DVh, DVl, 64, n, dVpp.hi, dVpp.lo, (tok0 * dm.H + h) * D + e0, (int64_t)dm.H * D);
        if (threadIdx.x == 0 && !*abort_flag) {
            // q^T (e^g dO) (hi, lo) ; w^T dV' (hi hi, lo hi, hi lo)
            const uint32_t sq = smem_u32(lt + kLateQ), swh = smem_u32(lt + kLateWh), swl = smem_u32(lt + kLateWl);
            for (int kk = 0; kk < 4; ++kk)
                umma_f16(tm + 128, tc::mdesc(sq, 64, 0, kk), tc::mdesc(segh, 64, 0, kk), id_ab, kk > 0 ? 1u : 0u);
            for (int kk = 0; kk < 4; ++kk) umma_f16(tm + 128, tc::mdesc(sq, 64, 0, kk), tc::mdesc(segl, 64, 0, kk), id_ab, 1u);
            for (int kk = 0; kk < 4; ++kk)
                umma_f16(tm + 192, tc::mdesc(swh, 64, 0, kk), tc::mdesc(sdvh, 64, 0, kk), id_ab, kk > 0 ? 1u : 0u);
            for (int kk = 0; kk < 4; ++kk) umma_f16(tm + 192, tc::mdesc(swl, 64, 0, kk), tc::mdesc(sdvh, 64, 0, kk), id_ab, 1u);
            for (int kk = 0; kk < 4; ++kk) umma_f16(tm + 192, tc::mdesc(swh, 64, 0, kk), tc::mdesc(sdvl, 64, 0, kk), id_ab, 1u);
            umma_commit(bar);
        }
        if (c > c0) b1_issue_early(sm, dm, k, P_hi, P_lo, dO, g, c - 1, h, hk, e0);
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar, phase, abort_flag));
        phase ^= 1u;
        tc_fence_after();
        if (ok) {
            const float el = gexp(gl);
            float t1[32], t2[32];
            tc::tmem_row32(tq + 128, t1);
            tc::tmem_row32(tq + 192, t2);
#pragma unroll
            for (int e = 0; e < 32; ++e) dS[e] = el * dS[e] + dm.scale * t1[e] - t2[e];
        }
    }
    if (dh0)
#pragma unroll
        for (int i = 0; i < 32; ++i) dh0[(((int64_t)seq * dm.H + h) * D + e0 + 32 * ch + i) * D + d] = dS[i];
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, 256);
}

// B2a: per (chunk, value head): the state-reading terms, written as partials of dq, dk, dg (pdq, pdk, pdg:
// the launcher passes the outputs themselves, which B2b then adds to). On tcgen05, transposed so the 128
// key lanes are the MMA's M (every TMEM lane busy, and a token column of the accumulator stores as one
// coalesced row): Q~^T = S dO^T, W^T = S dV'^T and K~^T = dS_next V'^T, [128 x 64] each, f32 in TMEM
// columns 0, 64 and 128. The f32 states and V', dV' enter as their stored bf16 (hi, lo) planes, so the
// products take two or three passes (hi hi, lo hi, hi lo), as the mma.sync forms did. Operands arrive in
// three cp.async groups: S, dO, q, dV', g; then dS_next; then (into the tiles dO and dV' held, once the
// first products have read them) V' and k.
constexpr int kBaTmemCols = 256;

__global__ void __launch_bounds__(256) gdn_bwd_a(Dims dm, const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                 const float* __restrict__ g, const float* __restrict__ S_all,
                                                 const float* __restrict__ Vp, const bf16* __restrict__ dO,
                                                 const float* __restrict__ dS_all, const float* __restrict__ dVp,
                                                 float* __restrict__ dw, float* __restrict__ pdq, float* __restrict__ pdk,
                                                 float* __restrict__ pdg) {
    extern __shared__ unsigned char smraw[];
    unsigned char* sm = tc::align1024(smraw);
    unsigned char* Sh = sm;                              // S hi/lo [128][128]
    unsigned char* Sl = Sh + tc::kBlockTile;
    unsigned char* Th = Sl + tc::kBlockTile;             // dS_next hi/lo [128][128]
    unsigned char* Tl = Th + tc::kBlockTile;
    unsigned char* Xs = Tl + tc::kBlockTile;             // dO [64][128], then k
    unsigned char* Yh = Xs + tc::kRowTile;               // dV' hi/lo [64][128], then V' hi/lo
    unsigned char* Yl = Yh + tc::kRowTile;
    unsigned char* Qs = Yl + tc::kRowTile;               // q [64][128]
    float* gs = reinterpret_cast<float*>(Qs + tc::kRowTile);
    float* dgs = gs + L;
    float* red = dgs + L;                                // [8]
    uint64_t* bar = reinterpret_cast<uint64_t*>(red + 8);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
    const int c = blockIdx.x, h = blockIdx.y, hk = h / dm.grp;
    const int64_t tok0 = dm.tok0[c];
    const int n = dm.len[c];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nb = (int64_t)dm.n_chunks * dm.H * D * D, nt = dm.T * dm.H * D;
    const int64_t blk = (int64_t)c * dm.H + h;
    const Pair Sp = pair_of(S_all, nb), Tp = pair_of(dS_all, nb), dVpp = pair_of(dVp, nt), Vpp = pair_of(Vp, nt);
    tc::stage_block(Sh, Sp.hi + blk * D * D);
    tc::stage_block(Sl, Sp.lo + blk * D * D);
    tc::stage_rows(Xs, dO, tok0, n, dm.H, h);
    tc::stage_rows(Qs, q, tok0, n, dm.Hg, hk);
    tc::stage_rows(Yh, dVpp.hi, tok0, n, dm.H, h);
    tc::stage_rows(Yl, dVpp.lo, tok0, n, dm.H, h);
    async_gb(gs, nullptr, g, nullptr, tok0, n, dm.H, h);
    cp_async_commit();
    tc::stage_block(Th, Tp.hi + blk * D * D);
    tc::stage_block(Tl, Tp.lo + blk * D * D);
    cp_async_commit();
    if (threadIdx.x < L) dgs[threadIdx.x] = 0.0f;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (warp == 0) {
        tmem_alloc(tslot, kBaTmemCols);
        tmem_relinquish();
    }
    cp_async_wait_but_one();
    tc::fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tslot;
    constexpr uint32_t idesc = make_idesc_bf16(128, 64, 0, 0);
    if (threadIdx.x == 0) {
        const uint32_t sh = smem_u32(Sh), sl = smem_u32(Sl), xs = smem_u32(Xs), yh = smem_u32(Yh), yl = smem_u32(Yl);
        // Q~^T = S dO^T (S: hi, lo)
        for (int kk = 0; kk < 8; ++kk)
            umma_f16(tm, tc::kdesc(sh, 128, 0, kk), tc::kdesc(xs, 64, 0, kk), idesc, kk > 0 ? 1u : 0u);
        for (int kk = 0; kk < 8; ++kk) umma_f16(tm, tc::kdesc(sl, 128, 0, kk), tc::kdesc(xs, 64, 0, kk), idesc, 1u);
        // W^T = S dV'^T (hi hi, lo hi, hi lo)
        for (int kk = 0; kk < 8; ++kk)
            umma_f16(tm + 64, tc::kdesc(sh, 128, 0, kk), tc::kdesc(yh, 64, 0, kk), idesc, kk > 0 ? 1u : 0u);
        for (int kk = 0; kk < 8; ++kk) umma_f16(tm + 64, tc::kdesc(sl, 128, 0, kk), tc::kdesc(yh, 64, 0, kk), idesc, 1u);
        for (int kk = 0; kk < 8; ++kk) umma_f16(tm + 64, tc::kdesc(sh, 128, 0, kk), tc::kdesc(yl, 64, 0, kk), idesc, 1u);
        umma_commit(bar);
    }
    bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar, 0, nullptr));  // warp-uniform: the TMEM loads are .aligned
    tc_fence_after();
    // the products have read dO and dV': V' and k take their tiles
    tc::stage_rows(Yh, Vpp.hi, tok0, n, dm.H, h);
    tc::stage_rows(Yl, Vpp.lo, tok0, n, dm.H, h);
    tc::stage_rows(Xs, k, tok0, n, dm.Hg, hk);
    cp_async_commit();
    // a warp reads its lane quarter (key lanes d = 32 (warp % 4) + lane) over token columns 32 (warp / 4) ..
    const int d = 32 * (warp & 3) + lane, t0 = 32 * (warp >> 2);
    const uint32_t tq = tm + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)t0;
    if (ok) {
        // dq = scale e^g dQ~ ; dg_i += q_i . dq_i
        float x[32], p[32];
        tc::tmem_row32(tq, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int r = t0 + i;
            x[i] *= dm.scale * gexp(gs[r]);
            p[i] = tc::ld_elem(Qs, 64, r, d) * x[i];
            if (r < n) pdq[((tok0 + r) * dm.H + h) * D + d] = x[i];
        }
        atomicAdd(&dgs[t0 + lane], tc::transpose_sum(p));
        // dw = -dV' S^T, kept as a (hi, lo) pair
        const Pair dwp = pair_of(dw, nt);
        tc::tmem_row32(tq + 64, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int r = t0 + i;
            if (r < n) put_split(dwp.hi, dwp.lo, ((tok0 + r) * dm.H + h) * D + d, -x[i]);
        }
    }
    cp_async_wait_but_one();  // dS_next landed
    __syncthreads();
    // <S, dS_next> from the pairs (the two tiles share one layout), while V' and k land
    {
        float sdot = 0.0f;
        for (int idx = threadIdx.x; idx < D * D / 8; idx += blockDim.x) {
            const uint4 a = reinterpret_cast<const uint4*>(Sh)[idx], b = reinterpret_cast<const uint4*>(Sl)[idx];
            const uint4 x = reinterpret_cast<const uint4*>(Th)[idx], y = reinterpret_cast<const uint4*>(Tl)[idx];
            const __nv_bfloat162* ah = reinterpret_cast<const __nv_bfloat162*>(&a);
            const __nv_bfloat162* bh = reinterpret_cast<const __nv_bfloat162*>(&b);
            const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&x);
            const __nv_bfloat162* yh = reinterpret_cast<const __nv_bfloat162*>(&y);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 fa = __bfloat1622float2(ah[e]), fb = __bfloat1622float2(bh[e]);
                const float2 fx = __bfloat1622float2(xh[e]), fy = __bfloat1622float2(yh[e]);
                sdot += (fa.x + fb.x) * (fx.x + fy.x) + (fa.y + fb.y) * (fx.y + fy.y);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sdot += __shfl_xor_sync(0xFFFFFFFFu, sdot, o);
        if (lane == 0) red[warp] = sdot;
    }
    cp_async_wait_all();
    tc::fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0 && ok) {
        const uint32_t th = smem_u32(Th), tl = smem_u32(Tl), yh = smem_u32(Yh), yl = smem_u32(Yl);
        // K~^T = dS_next V'^T (hi hi, lo hi, hi lo)
        for (int kk = 0; kk < 8; ++kk)
            umma_f16(tm + 128, tc::kdesc(th, 128, 0, kk), tc::kdesc(yh, 64, 0, kk), idesc, kk > 0 ? 1u : 0u);
        for (int kk = 0; kk < 8; ++kk) umma_f16(tm + 128, tc::kdesc(tl, 128, 0, kk), tc::kdesc(yh, 64, 0, kk), idesc, 1u);
        for (int kk = 0; kk < 8; ++kk) umma_f16(tm + 128, tc::kdesc(th, 128, 0, kk), tc::kdesc(yl, 64, 0, kk), idesc, 1u);
        umma_commit(bar);
    }
    ok = __all_sync(0xFFFFFFFFu, ok && mbar_wait(bar, 1, nullptr));
    tc_fence_after();
    const float gl = gs[n - 1];
    if (ok) {
        // dk_j = e^{gL-gj} dK~_j ; dg_j -= k_j . dk_j ; dg_L += their sum
        float x[32], p[32];
        tc::tmem_row32(tq + 128, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int r = t0 + i;
            x[i] *= r < n ? gexp(gl - gs[r]) : 0.0f;
            p[i] = tc::ld_elem(Xs, 64, r, d) * x[i];
            if (r < n) pdk[((tok0 + r) * dm.H + h) * D + d] = x[i];
        }
        const float s = tc::transpose_sum(p);
        atomicAdd(&dgs[t0 + lane], -s);
        float tot = s;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xFFFFFFFFu, tot, o);
        if (lane == 0) atomicAdd(&dgs[n - 1], tot);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int i = 0; i < 8; ++i) s += red[i];
        dgs[n - 1] += gexp(gl) * s;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) pdg[(tok0 + i) * dm.H + h] = dgs[i];
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, kBaTmemCols);
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

constexpr size_t kSmemPrep = f1::kUsed + 1024;  // and the slack that aligns the tiles to 1024 bytes
constexpr size_t kSmemState = f2::kUsed + 1024;  // and the slack that aligns the tiles to 1024 bytes
constexpr size_t kSmemOut = f3::kUsed + 1024;  // and the slack that aligns the tiles to 1024 bytes
constexpr size_t kSmemBState = b1::kUsed + 1024;  // and the slack that aligns the tiles to 1024 bytes
// four [128][128] state tiles, four [64][128] row tiles, g, dg, the warp sums, the barrier and TMEM slot,
// and the slack that aligns the tiles to 1024 bytes
constexpr size_t kSmemBA = 4 * tc::kBlockTile + 4 * tc::kRowTile + (2 * L + 8) * 4 + 16 + 1024;
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

R97B_ERROR_READER(gdn_error_word)

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
    gdn_fwd_state<<<dim3(dm.n_seq, dm.H, D / 64), 256, kSmemState, s>>>(dm, k, a->g, a->w, a->u, a->h0, a->S, a->Vp,
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
    gdn_bwd_state<<<dim3(dm.n_seq, dm.H, D / 64), 256, kSmemBState, s>>>(dm, q, k, a->g, a->w, a->P, dO, a->dht,
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
