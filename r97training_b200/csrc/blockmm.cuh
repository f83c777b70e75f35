// blockmm.cuh -- small dense products of shared-memory tiles by one 256-thread CTA, f32 accumulation.
//
// The GatedDeltaNet chunk kernels are sequences of 64x64, 64x128 and 128x128 products on tiles that
// already sit in shared memory. A thread of the 16 x 16 grid (ty = tid / 16, tx = tid % 16) owns rows
// ty + 16 i and columns tx + 16 j of the result, so a warp reads two rows of the left operand (broadcast)
// and sixteen consecutive columns of the right one; tiles are stored with an odd row pitch, which keeps
// the transposed reads free of bank conflicts.
#pragma once

#include <cuda_bf16.h>

namespace r97b {

constexpr int kBmmThreads = 256;

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p) {
    return static_cast<float>(*p);
}
template <>
__device__ __forceinline__ float ld_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
    return __bfloat162float(*p);
}

// acc[i][j] += sum_k opA(m = ty + 16 i, k) * opB(k, n = tx + 16 j)
//   opA(m, k) = A[m * lda + k]  (TA = false)   or  A[k * lda + m]  (TA = true)
//   opB(k, n) = B[k * ldb + n]  (TB = false)   or  B[n * ldb + k]  (TB = true)
template <int M, int N, int K, bool TA, bool TB, typename TAe, typename TBe>
__device__ __forceinline__ void bmm(float (&acc)[M / 16][N / 16], const TAe* __restrict__ A, int lda,
                                    const TBe* __restrict__ B, int ldb) {
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll 4
    for (int k = 0; k < K; ++k) {
        float a[M / 16], b[N / 16];
#pragma unroll
        for (int i = 0; i < M / 16; ++i) a[i] = TA ? ld_f32(A + k * lda + ty + 16 * i) : ld_f32(A + (ty + 16 * i) * lda + k);
#pragma unroll
        for (int j = 0; j < N / 16; ++j) b[j] = TB ? ld_f32(B + (tx + 16 * j) * ldb + k) : ld_f32(B + k * ldb + tx + 16 * j);
#pragma unroll
        for (int i = 0; i < M / 16; ++i)
#pragma unroll
            for (int j = 0; j < N / 16; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
}

template <int M, int N>
__device__ __forceinline__ void zero_acc(float (&acc)[M / 16][N / 16]) {
#pragma unroll
    for (int i = 0; i < M / 16; ++i)
#pragma unroll
        for (int j = 0; j < N / 16; ++j) acc[i][j] = 0.0f;
}

// Writes acc (scaled) into a shared tile C[m * ldc + n].
template <int M, int N>
__device__ __forceinline__ void store_acc(const float (&acc)[M / 16][N / 16], float* C, int ldc, float scale = 1.0f) {
    const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
#pragma unroll
    for (int i = 0; i < M / 16; ++i)
#pragma unroll
        for (int j = 0; j < N / 16; ++j) C[(ty + 16 * i) * ldc + tx + 16 * j] = acc[i][j] * scale;
}

}  // namespace r97b
