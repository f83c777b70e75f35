// adamw.cu -- AdamW on the flat f32 adapter buffer, on sm_100a.
//
// The per-element update is the reference Optimiser's, in the same f32 operations and the same order
// (reference src/optim.cpp:245-290, include/r97/optim.h:9-16):
//   g  = acc * inv_k [* clip]                 (the accumulation mean, then the global-norm clip)
//   m  = b1 m + (1 - b1) g
//   v  = b2 v + (1 - b2) g g
//   w -= lr (m / bc1 / (sqrt(v / bc2) + eps) + wd w)
// Every product and sum is an explicitly rounded f32 operation (no fused multiply-add), division and
// square root are IEEE-rounded, so the device update reproduces the reference's x86 f32 arithmetic
// bit for bit. lr, bc1 = 1 - b1^t and bc2 = 1 - b2^t come from the host, as the reference computes them.
//
// The global norm for clipping uses the reference's fixed 4096-element chunking: one f64 partial per
// chunk summed in element order, then the partials in chunk order (reference src/optim.cpp:135-170), so
// the norm is bit-identical too.
#include "r97b_internal.h"

#include <math.h>

#include <mutex>

namespace r97b {
namespace {

// One element's update in the reference's f32 operation order (every step rounded as the reference rounds).
struct AdamWConst {
    float lr, b1, b2, one_b1, one_b2, eps, wd, bc1, bc2, inv_k, cs;
    bool clip;
};

__device__ __forceinline__ void adamw_one(const AdamWConst& k, float& w, float& m, float& v, float g) {
    float gi = __fmul_rn(g, k.inv_k);
    if (k.clip) gi = __fmul_rn(gi, k.cs);
    const float mi = __fadd_rn(__fmul_rn(k.b1, m), __fmul_rn(k.one_b1, gi));
    const float vi = __fadd_rn(__fmul_rn(k.b2, v), __fmul_rn(__fmul_rn(k.one_b2, gi), gi));
    m = mi;
    v = vi;
    const float mh = __fdiv_rn(mi, k.bc1);
    const float vh = __fdiv_rn(vi, k.bc2);
    const float upd = __fadd_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), k.eps)), __fmul_rn(k.wd, w));
    w = __fsub_rn(w, __fmul_rn(k.lr, upd));
}

// Four elements a thread per step (16-byte loads and stores) over the aligned body, one at a time over the
// ragged tail.
__global__ void __launch_bounds__(256) adamw_kernel(float* __restrict__ w, float* __restrict__ m, float* __restrict__ v,
                                                    float* __restrict__ g, int64_t n, float lr, float b1, float b2,
                                                    float eps, float wd, float bc1, float bc2, float inv_k,
                                                    const float* __restrict__ clip_scale, int zero_grad,
                                                    const float* __restrict__ sched) {
    if (sched) {  // lr, bc1, bc2 from device memory (a captured graph's replays advance them)
        lr = sched[0];
        bc1 = sched[1];
        bc2 = sched[2];
    }
    const AdamWConst k{lr, b1, b2, __fsub_rn(1.0f, b1), __fsub_rn(1.0f, b2), eps, wd, bc1, bc2, inv_k,
                       clip_scale ? *clip_scale : 1.0f, clip_scale != nullptr};
    const bool vec = ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v) |
                       reinterpret_cast<uintptr_t>(g)) & 15) == 0;
    const int64_t n4 = vec ? n / 4 : 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 wv = reinterpret_cast<float4*>(w)[i], mv = reinterpret_cast<float4*>(m)[i];
        float4 vv = reinterpret_cast<float4*>(v)[i];
        const float4 gv = reinterpret_cast<const float4*>(g)[i];
        adamw_one(k, wv.x, mv.x, vv.x, gv.x);
        adamw_one(k, wv.y, mv.y, vv.y, gv.y);
        adamw_one(k, wv.z, mv.z, vv.z, gv.z);
        adamw_one(k, wv.w, mv.w, vv.w, gv.w);
        reinterpret_cast<float4*>(w)[i] = wv;
        reinterpret_cast<float4*>(m)[i] = mv;
        reinterpret_cast<float4*>(v)[i] = vv;
        if (zero_grad) reinterpret_cast<float4*>(g)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float wi = w[i], mi = m[i], vi = v[i];
        adamw_one(k, wi, mi, vi, g[i]);
        w[i] = wi;
        m[i] = mi;
        v[i] = vi;
        if (zero_grad) g[i] = 0.0f;
    }
}

constexpr int64_t kNormChunk = 4096;

// One thread per 4096-element chunk: the chunk's f64 sum of squares in element order.
__global__ void __launch_bounds__(256) chunk_sumsq_kernel(const float* __restrict__ g, int64_t n, float inv_k,
                                                          double* __restrict__ partials, int64_t nchunks) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= nchunks) return;
    const int64_t lo = c * kNormChunk;
    const int64_t hi = lo + kNormChunk < n ? lo + kNormChunk : n;
    double part = 0.0;
    for (int64_t i = lo; i < hi; ++i) {
        const double x = (double)__fmul_rn(g[i], inv_k);
        part = __dadd_rn(part, __dmul_rn(x, x));
    }
    partials[c] = part;
}

// The partials in chunk order, the norm, and the clip factor (1 when no clip applies).
__global__ void norm_finish_kernel(const double* __restrict__ partials, int64_t nchunks, float max_norm,
                                   float* __restrict__ out_norm, float* __restrict__ out_scale) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    double sq = 0.0;
    for (int64_t c = 0; c < nchunks; ++c) sq = __dadd_rn(sq, partials[c]);
    const float norm = (float)sqrt(sq);
    if (out_norm) *out_norm = norm;
    if (out_scale) *out_scale = (max_norm > 0.0f && norm > max_norm && norm > 0.0f) ? __fdiv_rn(max_norm, norm) : 1.0f;
}

// ---- the allocation-free global norm: its partials live in this file's own device array ----------------
//
// Some callers of this library cannot allocate device memory: a host framework whose allocator already
// owns the whole device budget, or a loop that must not pay cudaMalloc / cudaFree (cudaFree synchronises
// the device). r97b_global_norm_noalloc serves them with the scratch below. The array belongs to this
// library's device module, which CUDA loads on a device when that device first uses the module (at the
// latest, the first no-alloc call's address lookup); from then on that GPU holds these 512 KiB until the
// process exits.
constexpr int64_t kNoAllocMaxChunks = R97B_GLOBAL_NORM_NOALLOC_MAX_ELEMS / kNormChunk;
static __device__ __align__(256) double g_noalloc_partials[kNoAllocMaxChunks];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
double* g_noalloc_ptr[kMaxDevices] = {};

// The array's device address on the current device, looked up once per device. Host code must not pass
// `g_noalloc_partials` itself to a kernel: on the host that name is a stand-in, not a device address.
int noalloc_partials(double** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return R97B_ELAUNCH;
    if (dev < 0 || dev >= kMaxDevices) return R97B_EINVAL;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return R97B_ELAUNCH;
        }
        g_noalloc_ptr[dev] = static_cast<double*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return R97B_OK;
}

}  // namespace
}  // namespace r97b

using namespace r97b;

// See include/r97b.h. The same two kernels as r97b_global_norm, over the file's own partials array.
extern "C" int r97b_global_norm_noalloc(const float* g, int64_t n, float inv_k, float max_norm, float* out_norm,
                                        float* out_scale, void* stream) {
    if (!g || n <= 0) return R97B_EINVAL;
    if (n > R97B_GLOBAL_NORM_NOALLOC_MAX_ELEMS) return R97B_ETOOLARGE;
    double* partials = nullptr;
    const int rc = noalloc_partials(&partials);
    if (rc != R97B_OK) return rc;
    const int64_t nchunks = (n + kNormChunk - 1) / kNormChunk;
    chunk_sumsq_kernel<<<(unsigned)((nchunks + 255) / 256), 256, 0, as_stream(stream)>>>(g, n, inv_k, partials,
                                                                                          nchunks);
    norm_finish_kernel<<<1, 32, 0, as_stream(stream)>>>(partials, nchunks, max_norm, out_norm, out_scale);
    return launch_status(2);
}

// One AdamW update of `n` f32 parameters. `g` holds the accumulated gradient; it is scaled by `inv_k`
// (1 / accumulation count) and, when `clip_scale` (a device f32) is given, by that factor, exactly as
// the reference applies the mean and the clip. `zero_grad` clears `g` after reading it (the reference
// clears its accumulation buffer after the update).
extern "C" int r97b_adamw_step(float* w, float* m, float* v, float* g, int64_t n, float lr, float beta1, float beta2,
                               float eps, float weight_decay, float bc1, float bc2, float inv_k,
                               const float* clip_scale, int32_t zero_grad, void* stream) {
    if (!w || !m || !v || !g || n <= 0) return R97B_EINVAL;
    int blocks = (int)((n + 255) / 256);
    if (blocks > 148 * 16) blocks = 148 * 16;
    adamw_kernel<<<blocks, 256, 0, as_stream(stream)>>>(w, m, v, g, n, lr, beta1, beta2, eps, weight_decay, bc1, bc2,
                                                        inv_k, clip_scale, zero_grad, nullptr);
    return launch_status();
}

// The same update with lr, bc1, bc2 read from sched[0..2] (device f32) when the kernel runs.
extern "C" int r97b_adamw_step_dev(float* w, float* m, float* v, float* g, int64_t n, const float* sched, float beta1,
                                   float beta2, float eps, float weight_decay, float inv_k, const float* clip_scale,
                                   int32_t zero_grad, void* stream) {
    if (!w || !m || !v || !g || !sched || n <= 0) return R97B_EINVAL;
    const int64_t want = (n + 255) / 256;
    const unsigned blocks = (unsigned)(want < 148 * 16 ? want : 148 * 16);
    adamw_kernel<<<blocks, 256, 0, as_stream(stream)>>>(w, m, v, g, n, 0.0f, beta1, beta2, eps, weight_decay, 1.0f,
                                                        1.0f, inv_k, clip_scale, zero_grad, sched);
    return launch_status();
}

// The scratch a global-norm call needs: one f64 partial per 4096 elements.
extern "C" int64_t r97b_global_norm_scratch_bytes(int64_t n) { return ((n + kNormChunk - 1) / kNormChunk) * 8; }

// The global L2 norm of `g * inv_k` into *out_norm (device f32), and the clip factor for `max_norm` into
// *out_scale (device f32, may be null). `partials` is caller scratch of r97b_global_norm_scratch_bytes(n).
extern "C" int r97b_global_norm(const float* g, int64_t n, float inv_k, float max_norm, double* partials,
                                float* out_norm, float* out_scale, void* stream) {
    if (!g || n <= 0 || !partials) return R97B_EINVAL;
    const int64_t nchunks = (n + kNormChunk - 1) / kNormChunk;
    chunk_sumsq_kernel<<<(unsigned)((nchunks + 255) / 256), 256, 0, as_stream(stream)>>>(g, n, inv_k, partials, nchunks);
    norm_finish_kernel<<<1, 32, 0, as_stream(stream)>>>(partials, nchunks, max_norm, out_norm, out_scale);
    return launch_status(2);
}

namespace r97b {
namespace {
__global__ void add_f32_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n) {
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i + 4 <= n && ((reinterpret_cast<uintptr_t>(dst + i) | reinterpret_cast<uintptr_t>(src + i)) & 15) == 0) {
        float4 a = *reinterpret_cast<float4*>(dst + i);
        const float4 b = *reinterpret_cast<const float4*>(src + i);
        a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
        *reinterpret_cast<float4*>(dst + i) = a;
    } else {
        for (int64_t j = i; j < n && j < i + 4; ++j) dst[j] += src[j];
    }
}
}  // namespace
}  // namespace r97b

// dst += src (f32, element-wise): the optimiser's gradient accumulation (reference src/optim.cpp:231-244).
extern "C" int r97b_add_f32(float* dst, const float* src, int64_t n, void* stream) {
    if (!dst || !src || n < 0) return R97B_EINVAL;
    if (n == 0) return R97B_OK;
    const int64_t threads = (n + 3) / 4;
    r97b::add_f32_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, r97b::as_stream(stream)>>>(dst, src, n);
    return r97b::launch_status();
}
