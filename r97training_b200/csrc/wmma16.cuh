// wmma16.cuh -- warp-level tensor-core products of shared-memory tiles: mma.sync m16n8k16 with bf16
// operands and f32 accumulators, fragments loaded by ldmatrix (plain or .trans).
//
// Tiles are bf16, row-major with a padded pitch (a multiple of 8 elements whose byte stride is an odd
// multiple of 16: 72 or 136), so every ldmatrix row address is 16-byte aligned and the eight rows of an
// 8x8 block fall in distinct bank groups. An f32 operand that must keep more than bf16's 8 bits is carried
// as two tiles, hi = bf16(x) and lo = bf16(x - hi); a product then takes two or three mma passes
// (hi*B + lo*B, or hi*hi + lo*hi + hi*lo), about 16 bits of operand precision with f32 accumulation.
//
// Fragment layouts are the PTX ISA's for mma.m16n8k16 .bf16 (A row, B col): with g = lane / 4 and
// t = lane % 4, A holds (g, 2t..2t+1), (g+8, 2t..), (g, 2t+8..), (g+8, 2t+8..); B holds (k = 2t.., n = g)
// and (k = 2t+8.., n = g); the accumulator holds (g, 2t..2t+1) and (g+8, 2t..2t+1).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace r97b {

constexpr int kP64 = 72;    // bf16 pitch of a [*, 64] tile
constexpr int kP128 = 136;  // bf16 pitch of a [*, 128] tile

__device__ __forceinline__ uint32_t s_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(s_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(s_addr(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The A fragment of the 16x16 block at (m0, k0) of opA:
//   A_T = false: opA(m, k) = A[m * pa + k]     A_T = true: opA(m, k) = A[k * pa + m]
template <bool A_T>
__device__ __forceinline__ void load_a(uint32_t (&a)[4], const __nv_bfloat16* A, int pa, int m0, int k0) {
    const int lane = threadIdx.x & 31;
    if (!A_T) {
        ldsm_x4(a, A + (m0 + (lane & 15)) * pa + k0 + ((lane >> 4) << 3));
    } else {
        ldsm_x4_t(a, A + (k0 + (lane & 7) + (((lane >> 4) & 1) << 3)) * pa + m0 + (((lane >> 3) & 1) << 3));
    }
}

// The B fragments of two adjacent n-tiles (n0 .. n0+15) at k0 of opB:
//   B_T = false: opB(k, n) = B[n * pb + k]     B_T = true: opB(k, n) = B[k * pb + n]
// b[0], b[1] serve n-tile n0; b[2], b[3] serve n0 + 8.
template <bool B_T>
__device__ __forceinline__ void load_b2(uint32_t (&b)[4], const __nv_bfloat16* B, int pb, int n0, int k0) {
    const int lane = threadIdx.x & 31;
    if (!B_T) {
        ldsm_x4(b, B + (n0 + (lane & 7) + (((lane >> 4) & 1) << 3)) * pb + k0 + (((lane >> 3) & 1) << 3));
    } else {
        ldsm_x4_t(b, B + (k0 + (lane & 7) + (((lane >> 3) & 1) << 3)) * pb + n0 + (((lane >> 4) & 1) << 3));
    }
}

// acc += opA[m0 .. m0+WM) x opB[.., n0 .. n0+WN) over k in [0, K): one warp.
template <int WM, int WN, int K, bool A_T, bool B_T>
__device__ __forceinline__ void warp_mma(float (&acc)[WM / 16][WN / 8][4], const __nv_bfloat16* A, int pa,
                                         const __nv_bfloat16* B, int pb, int m0, int n0) {
    static_assert(WM % 16 == 0 && WN % 16 == 0 && K % 16 == 0, "tile shape");
#pragma unroll
    for (int k0 = 0; k0 < K; k0 += 16) {
        uint32_t a[WM / 16][4];
#pragma unroll
        for (int i = 0; i < WM / 16; ++i) load_a<A_T>(a[i], A, pa, m0 + 16 * i, k0);
#pragma unroll
        for (int j = 0; j < WN / 16; ++j) {
            uint32_t b[4];
            load_b2<B_T>(b, B, pb, n0 + 16 * j, k0);
#pragma unroll
            for (int i = 0; i < WM / 16; ++i) {
                mma16816(acc[i][2 * j], a[i], b[0], b[1]);
                mma16816(acc[i][2 * j + 1], a[i], b[2], b[3]);
            }
        }
    }
}

template <int WM, int WN>
__device__ __forceinline__ void acc_zero(float (&acc)[WM / 16][WN / 8][4]) {
#pragma unroll
    for (int i = 0; i < WM / 16; ++i)
#pragma unroll
        for (int j = 0; j < WN / 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;
}

// Visits every accumulator element of a warp tile at (m0, n0): fn(row, col, value&).
template <int WM, int WN, typename F>
__device__ __forceinline__ void acc_for(float (&acc)[WM / 16][WN / 8][4], int m0, int n0, F&& fn) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int i = 0; i < WM / 16; ++i)
#pragma unroll
        for (int j = 0; j < WN / 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) fn(m0 + 16 * i + g + ((e >> 1) << 3), n0 + 8 * j + 2 * t + (e & 1), acc[i][j][e]);
}

// The same walk, also handing fn the fragment indices (i, j, e) -- compile-time after unrolling -- so a
// lambda can read the matching element of another accumulator of the same shape without dynamic
// indexing: fn(row, col, i, j, e).
template <int WM, int WN, typename F>
__device__ __forceinline__ void acc_walk(int m0, int n0, F&& fn) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int i = 0; i < WM / 16; ++i)
#pragma unroll
        for (int j = 0; j < WN / 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) fn(m0 + 16 * i + g + ((e >> 1) << 3), n0 + 8 * j + 2 * t + (e & 1), i, j, e);
}

// The walk by column pairs: each lane's accumulator holds two adjacent columns (2t, 2t+1) of a row, so a
// store of both is one 4-byte access. fn(row, col, i, j, h) with the pair acc[i][j][2h], acc[i][j][2h + 1]
// at (row, col) and (row, col + 1).
template <int WM, int WN, typename F>
__device__ __forceinline__ void acc_pairs(int m0, int n0, F&& fn) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int i = 0; i < WM / 16; ++i)
#pragma unroll
        for (int j = 0; j < WN / 8; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) fn(m0 + 16 * i + g + 8 * h, n0 + 8 * j + 2 * t, i, j, h);
}

// x0, x1 -> their (hi, lo) bf16 pairs at hi[at], hi[at + 1] and lo[at], lo[at + 1] (at even)
__device__ __forceinline__ void put_split2(__nv_bfloat16* hi, __nv_bfloat16* lo, int64_t at, float x0, float x1) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 hf = __bfloat1622float2(h);
    *reinterpret_cast<__nv_bfloat162*>(hi + at) = h;
    *reinterpret_cast<__nv_bfloat162*>(lo + at) = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
}

// ------------------------------------------------------------------- asynchronous global -> shared copies
// cp.async with a source size of 0 writes zeros (rows past a chunk's end); `src` must still be a valid
// address, so callers clamp it.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s_addr(dst)), "l"(src), "r"(pred ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool pred) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(s_addr(dst)), "l"(src), "r"(pred ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// every committed group but the most recent one has landed
__device__ __forceinline__ void cp_async_wait_but_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// x -> (hi, lo) bf16 pair with hi + lo ~ x to about 16 bits
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(x);
    lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

}  // namespace r97b
