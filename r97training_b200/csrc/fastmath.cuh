// Single-instruction transcendental approximations for the elementwise kernels (flush-to-zero forms of the
// PTX ex2 / rcp / rsqrt approximations). Without .ftz each of these needs a denormal-range fix-up around the
// hardware instruction, which in the HBM-bound kernels that evaluate one a channel costs more issue slots than
// the arithmetic itself. Inputs and results here are never denormal in a way that matters: the sigmoid's
// exponential underflows to 0 or overflows to +inf, either giving the right limit.
#pragma once

namespace r97b {

__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rcp_ftz(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float rsqrt_ftz(float x) {
    float y;
    asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// sigmoid(x) = 1 / (1 + e^-x) = 1 / (1 + 2^(-x log2 e))
__device__ __forceinline__ float sigmoid_ftz(float x) { return rcp_ftz(1.0f + ex2_ftz(x * -1.4426950408889634f)); }

}  // namespace r97b
