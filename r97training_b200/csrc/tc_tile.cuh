// tc_tile.cuh -- chunk-sized operand tiles for CTA-wide tcgen05 products (the GatedDeltaNet kernels).
//
// A tile holds R rows x C bf16 columns (C = 64 or 128) in the 128-byte-swizzled layout the tensor core
// reads: column block b (columns 64 b .. 64 b + 63) is an [R][64] slab at byte b * R * 128; inside it row r
// takes the 128 bytes at r * 128, with its 16-byte chunk j stored at chunk position j ^ (r & 7). The same
// tile serves as a K-major operand (its columns are the contraction) and as an MN-major one (its rows are),
// so a chunk's [64 tokens][128 lanes] tile feeds both q k^T (contracting lanes) and k^T V (contracting
// tokens) without a transposed copy.
//
// Tiles are filled by cp.async (16-byte chunks, zeros past a chunk's last token) or by plain stores from
// registers; either way the writing threads fence the generic proxy against the tensor core's reads
// (fence.proxy.async) before the CTA barrier that precedes the MMAs. One thread issues the MMAs and
// commits them to an mbarrier that the CTA waits on (bounded, sm100.cuh).
#pragma once

#include "sm100.cuh"
#include "wmma16.cuh"

#include <cuda_bf16.h>

namespace r97b {
namespace tc {

constexpr int kRowTile = 64 * 128 * 2;    // bytes of a [64][128] tile
constexpr int kBlockTile = 128 * 128 * 2; // bytes of a [128][128] tile
constexpr int kSqTile = 64 * 64 * 2;      // bytes of a [64][64] tile

// byte offset of 16-byte chunk j (columns 8 j .. 8 j + 7) of row r in an R-row tile
__device__ __forceinline__ uint32_t chunk_off(int R, int r, int j) {
    return (uint32_t)((j >> 3) * R * 128 + r * 128 + (((j & 7) ^ (r & 7)) << 4));
}
// byte offset of element (r, c)
__device__ __forceinline__ uint32_t elem_off(int R, int r, int c) { return chunk_off(R, r, c >> 3) + (c & 7) * 2; }

__device__ __forceinline__ float ld_elem(const unsigned char* tile, int R, int r, int c) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(tile + elem_off(R, r, c)));
}

// Descriptor of K step kk (16 contraction elements) of an operand read K-major from an R-row tile whose
// columns are the contraction: operand rows r0 .. r0 + M (or N) - 1 (r0 a multiple of 8).
__device__ __forceinline__ uint64_t kdesc(uint32_t tile, int R, int r0, int kk) {
    return make_sdesc_sw128(tile + (uint32_t)((kk >> 2) * R * 128 + r0 * 128 + (kk & 3) * 32), 16, 1024);
}
// Descriptor of K step kk of an operand read MN-major from an R-row tile whose rows are the contraction:
// operand columns c0 .. c0 + M (or N) - 1 (c0 a multiple of 64); blocks of 64 columns lie R * 128 bytes apart.
__device__ __forceinline__ uint64_t mdesc(uint32_t tile, int R, int c0, int kk) {
    return make_sdesc_sw128(tile + (uint32_t)((c0 >> 6) * R * 128 + kk * 2048), (uint32_t)(R * 128), 1024);
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Rows [0, 64) of one head of a token-major [T, heads, 128] bf16 tensor, from token tok0, into rows
// row0 .. row0 + 63 of an R-row [R][128] tile; rows past the chunk's n tokens are zeros.
__device__ __forceinline__ void stage_rows(unsigned char* tile, const __nv_bfloat16* src, int64_t tok0, int n,
                                           int heads, int head, int R = 64, int row0 = 0) {
    for (int idx = threadIdx.x; idx < 64 * 16; idx += blockDim.x) {
        const int r = idx >> 4, j = idx & 15;
        const bool on = r < n;
        cp_async16(tile + chunk_off(R, row0 + r, j), src + ((on ? tok0 + r : tok0) * heads + head) * 128 + j * 8, on);
    }
}
// A contiguous row-major [128][128] bf16 block into a [128][128] tile.
__device__ __forceinline__ void stage_block(unsigned char* tile, const __nv_bfloat16* src) {
    for (int idx = threadIdx.x; idx < 128 * 16; idx += blockDim.x) {
        const int r = idx >> 4, j = idx & 15;
        cp_async16(tile + chunk_off(128, r, j), src + r * 128 + j * 8, true);
    }
}

// Writes v = 32 consecutive columns c0 .. c0 + 31 (c0 a multiple of 32) of row r of an R-row tile pair as
// bf16 hi = bf16(v) and lo = bf16(v - hi), four 16-byte chunks a plane.
__device__ __forceinline__ void put_row32(unsigned char* th, unsigned char* tl, int R, int r, int c0,
                                          const float (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float x0 = v[8 * j + 2 * e], x1 = v[8 * j + 2 * e + 1];
            const __nv_bfloat162 hh = __floats2bfloat162_rn(x0, x1);
            const float2 hf = __bfloat1622float2(hh);
            const __nv_bfloat162 ll = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
            hw[e] = *reinterpret_cast<const uint32_t*>(&hh);
            lw[e] = *reinterpret_cast<const uint32_t*>(&ll);
        }
        const uint32_t o = chunk_off(R, r, (c0 >> 3) + j);
        *reinterpret_cast<uint4*>(th + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(tl + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
}

// The same 32 values as (hi, lo) bf16 planes in global memory at hi[at .. at + 31], lo[at .. at + 31]
// (at a multiple of 8).
__device__ __forceinline__ void put_global32(__nv_bfloat16* hi, __nv_bfloat16* lo, int64_t at, const float (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float x0 = v[8 * j + 2 * e], x1 = v[8 * j + 2 * e + 1];
            const __nv_bfloat162 hh = __floats2bfloat162_rn(x0, x1);
            const float2 hf = __bfloat1622float2(hh);
            const __nv_bfloat162 ll = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
            hw[e] = *reinterpret_cast<const uint32_t*>(&hh);
            lw[e] = *reinterpret_cast<const uint32_t*>(&ll);
        }
        *reinterpret_cast<uint4*>(hi + at + 8 * j) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(lo + at + 8 * j) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
}

// The first `rows` rows of an R-row, 64-column tile pair (hi, lo) copied to global bf16 planes at
// hi/lo[at + r * ld + 0 .. 63]: each row leaves as one 128-byte run, a warp storing four rows at once (a
// thread that owned a row would store 32 rows' pieces in one instruction). The whole CTA calls it after the
// barrier that follows the tiles' writes.
__device__ __forceinline__ void tile_to_global(const unsigned char* th, const unsigned char* tl, int R, int rows,
                                               __nv_bfloat16* hi, __nv_bfloat16* lo, int64_t at, int64_t ld) {
    for (int idx = threadIdx.x; idx < 2 * R * 8; idx += blockDim.x) {
        const int plane = idx / (R * 8), r = (idx >> 3) % R, j = idx & 7;
        if (r >= rows) continue;
        const uint4 v = *reinterpret_cast<const uint4*>((plane ? tl : th) + chunk_off(R, r, j));
        *reinterpret_cast<uint4*>((plane ? lo : hi) + at + r * ld + j * 8) = v;
    }
}

// 32 TMEM columns of this warp's lane quarter, as floats.
__device__ __forceinline__ void tmem_row32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    tmem_ld32(taddr, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Lane l of the warp holds v[0 .. 31]; returns sum over the warp's lanes of v[l] (a butterfly that halves
// the live values each step: 31 shuffles instead of 32 x 5). v is clobbered.
__device__ __forceinline__ float transpose_sum(float (&v)[32]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const bool upper = (lane & s) != 0;
#pragma unroll
        for (int i = 0; i < s; ++i) {
            const float send = upper ? v[i] : v[i + s];
            const float keep = upper ? v[i + s] : v[i];
            v[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, s);
        }
    }
    return v[0];
}

// The dynamic shared memory rounded up to the 1024-byte boundary the swizzled tiles need.
__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
    const uint32_t a = smem_u32(p);
    return p + (((a + 1023u) & ~1023u) - a);
}

}  // namespace tc
}  // namespace r97b
