// loss.cu -- the vocabulary head's loss and its gradient on sm_100a: softmax cross-entropy and the
// KL divergence to a teacher, one pass over a chunk of logit rows.
//
// A row is read from HBM once: a cluster of four CTAs shares it, each copying its quarter into shared
// memory (one bulk copy per 16 KB, completing on an mbarrier), then keeping, per thread, an online
// log-sum-exp of the student logits (max m_s, sum S_s) and, with a teacher, the teacher's (m_t, S_t) and
// U = sum e^{t - m_t} (t - s). The CTAs merge those, trade their partial sums through distributed shared
// memory, and each writes its quarter's gradient from shared memory -- in place over the logits when the
// caller passes the same buffer. (Rows that the quarters do not tile -- a vocabulary not a multiple of 8,
// unaligned rows -- take a one-CTA-a-row kernel that reads the row twice, the second time mostly from L2.)
// Per row:
//
//   CE  = lse_s - s[target]                     dCE/ds  = softmax(s) - onehot(target)
//   KL  = sum p_t (log p_t - log p_s)
//       = U / S_t - lse_t + lse_s               dKL/ds  = softmax(s) - softmax(t)
//   grad = grad_scale * (w_ce dCE/ds + w_kl dKL/ds), zero on a row whose target is -1.
//
// CE follows the reference's ce_position (src/loss.cpp:21-39) and its chunk kernel's contract
// (include/r97/head.h:28-50, HeadChunk); the KL objective has no counterpart in the reference.
#include "r97b_internal.h"
#include "fastmath.cuh"
#include "sm100.cuh"

#include <cuda_bf16.h>
#include <math.h>

namespace r97b {
namespace {

constexpr int kThreads = 512;

// e^x as one flush-to-zero ex2 of x log2 e (the arguments are logits less a running max: <= 0).
__device__ __forceinline__ float fexp(float x) { return ex2_ftz(x * 1.4426950408889634f); }

struct Acc {
    float m, s;       // student: running max and sum of exp(x - m)
    float mt, st, u;  // teacher: running max, sum of exp(t - mt), sum of exp(t - mt) * (t - s)
};

__device__ __forceinline__ void merge(Acc& a, const Acc& b) {
    const float m = fmaxf(a.m, b.m);
    a.s = (a.m == -INFINITY ? 0.0f : a.s * fexp(a.m - m)) + (b.m == -INFINITY ? 0.0f : b.s * fexp(b.m - m));
    a.m = m;
    const float mt = fmaxf(a.mt, b.mt);
    const float fa = a.mt == -INFINITY ? 0.0f : fexp(a.mt - mt);
    const float fb = b.mt == -INFINITY ? 0.0f : fexp(b.mt - mt);
    a.st = a.st * fa + b.st * fb;
    a.u = a.u * fa + b.u * fb;
    a.mt = mt;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

template <bool kTeacher>
__global__ void __launch_bounds__(kThreads) ce_kld_kernel(const __nv_bfloat16* __restrict__ logits,
                                                          const __nv_bfloat16* __restrict__ teacher,
                                                          const int32_t* __restrict__ targets, __nv_bfloat16* grad,
                                                          float* __restrict__ loss_ce, float* __restrict__ loss_kl,
                                                          int64_t vocab, int64_t ld, int64_t ld_t, float grad_scale,
                                                          float w_ce, float w_kl, int vec) {
    const int64_t row = blockIdx.x;
    const int32_t target = targets ? targets[row] : 0;
    // a target outside the vocabulary scores nothing, like -1, rather than reading past the row
    const bool scored = target >= 0 && target < vocab;
    const __nv_bfloat16* x = logits + row * ld;
    const __nv_bfloat16* t = kTeacher ? teacher + row * ld_t : nullptr;
    // rows 16-byte aligned (every stride a multiple of 8 elements): 8 values a load; else one at a time
    const int64_t nvec = vec ? vocab / 8 : 0;

    Acc a{-INFINITY, 0.0f, -INFINITY, 0.0f, 0.0f};
    // one 8-value vector of the row (and the teacher's) into the running sums
    auto fold = [&](const uint4& xs, const uint4& ts) {
        float v[8];
        unpack8(xs, v);
        float mx = v[0];
#pragma unroll
        for (int k = 1; k < 8; ++k) mx = fmaxf(mx, v[k]);
        const float m = fmaxf(a.m, mx);
        float s = a.m == -INFINITY ? 0.0f : a.s * fexp(a.m - m);
#pragma unroll
        for (int k = 0; k < 8; ++k) s += fexp(v[k] - m);
        a.m = m;
        a.s = s;
        if (kTeacher) {
            float tv[8];
            unpack8(ts, tv);
            float tm = tv[0];
#pragma unroll
            for (int k = 1; k < 8; ++k) tm = fmaxf(tm, tv[k]);
            const float mt = fmaxf(a.mt, tm);
            const float f = a.mt == -INFINITY ? 0.0f : fexp(a.mt - mt);
            float st = a.st * f, u = a.u * f;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float e = fexp(tv[k] - mt);
                st += e;
                u = fmaf(e, tv[k] - v[k], u);
            }
            a.mt = mt;
            a.st = st;
            a.u = u;
        }
    };
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const uint4* tvp = kTeacher ? reinterpret_cast<const uint4*>(t) : nullptr;
    int64_t i = threadIdx.x;
    for (; i + 3 * kThreads < nvec; i += 4 * kThreads) {  // four vectors in flight a thread
        uint4 xs[4], ts[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            xs[q] = xv[i + q * kThreads];
            ts[q] = kTeacher ? tvp[i + q * kThreads] : xs[q];
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) fold(xs[q], ts[q]);
    }
    for (; i < nvec; i += kThreads) fold(xv[i], kTeacher ? tvp[i] : xv[i]);
    // the ragged tail (vocab not a multiple of 8), one element a thread
    for (int64_t j = nvec * 8 + threadIdx.x; j < vocab; j += kThreads) {
        const float v = __bfloat162float(x[j]);
        Acc b{v, 1.0f, -INFINITY, 0.0f, 0.0f};
        if (kTeacher) {
            const float tv = __bfloat162float(t[j]);
            b.mt = tv;
            b.st = 1.0f;
            b.u = tv - v;
        }
        merge(a, b);
    }
    // warp, then CTA merge
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Acc b;
        b.m = __shfl_xor_sync(0xFFFFFFFFu, a.m, o);
        b.s = __shfl_xor_sync(0xFFFFFFFFu, a.s, o);
        b.mt = __shfl_xor_sync(0xFFFFFFFFu, a.mt, o);
        b.st = __shfl_xor_sync(0xFFFFFFFFu, a.st, o);
        b.u = __shfl_xor_sync(0xFFFFFFFFu, a.u, o);
        merge(a, b);
    }
    __shared__ Acc red[kThreads / 32];
    __shared__ float bc[4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = a;
    __syncthreads();
    if (threadIdx.x == 0) {
        Acc r = red[0];
        for (int w = 1; w < kThreads / 32; ++w) merge(r, red[w]);
        const float lse = r.m + logf(r.s);
        const float lse_t = kTeacher ? r.mt + logf(r.st) : 0.0f;
        bc[0] = lse;
        bc[1] = lse_t;
        // log(s) - (x_t - m), not lse - x_t: with a large row maximum, adding m first would round log(s)
        // away (the reference's ce_position keeps this order, src/loss.cpp:21-39)
        if (loss_ce) loss_ce[row] = scored && targets ? logf(r.s) - (__bfloat162float(x[target]) - r.m) : 0.0f;
        if (loss_kl) loss_kl[row] = kTeacher && scored ? r.u / r.st - lse_t + lse : 0.0f;
    }
    __syncthreads();
    if (!grad) return;
    const float lse = bc[0], lse_t = bc[1];
    __nv_bfloat16* g = grad + row * ld;
    const float ce_w = targets ? w_ce : 0.0f;
    const float sc = scored ? grad_scale : 0.0f;
    // one 8-value vector of the gradient from the row (and the teacher's)
    auto emit = [&](int64_t iv, const uint4& xs, const uint4& ts) {
        float v[8], tv[8];
        unpack8(xs, v);
        if (kTeacher) unpack8(ts, tv);
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float p = fexp(v[k] - lse);
            float d = ce_w * p;
            if (kTeacher) d += w_kl * (p - fexp(tv[k] - lse_t));
            if (targets && iv * 8 + k == target) d -= ce_w;
            o[k] = d * sc;
        }
        uint4 u;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(o[2 * k], o[2 * k + 1]);
        reinterpret_cast<uint4*>(g)[iv] = u;
    };
    i = threadIdx.x;
    for (; i + 3 * kThreads < nvec; i += 4 * kThreads) {  // four vectors in flight a thread
        uint4 xs[4], ts[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            xs[q] = xv[i + q * kThreads];
            ts[q] = kTeacher ? tvp[i + q * kThreads] : xs[q];
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) emit(i + q * kThreads, xs[q], ts[q]);
    }
    for (; i < nvec; i += kThreads) emit(i, xv[i], kTeacher ? tvp[i] : xv[i]);
    for (int64_t j = nvec * 8 + threadIdx.x; j < vocab; j += kThreads) {
        const float p = fexp(__bfloat162float(x[j]) - lse);
        float d = ce_w * p;
        if (kTeacher) d += w_kl * (p - fexp(__bfloat162float(t[j]) - lse_t));
        if (targets && j == target) d -= ce_w;
        g[j] = __float2bfloat16_rn(d * sc);
    }
}


// ------------------------------------------------------------------------- one read a row: clusters

constexpr int kCl = 4;  // CTAs a row

// Untiled bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) into this CTA's shared
// memory, completing on `bar`. Never a multicast form.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// A CTA's partial sums as the cluster trades them: the running sums, and the target's logit when the
// target lies in the CTA's quarter (else -inf).
struct Part {
    Acc a;
    float xt;
};

template <bool kTeacher>
__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kThreads)
    ce_kld_cluster(const __nv_bfloat16* __restrict__ logits, const __nv_bfloat16* __restrict__ teacher,
                   const int32_t* __restrict__ targets, __nv_bfloat16* grad, float* __restrict__ loss_ce,
                   float* __restrict__ loss_kl, int64_t vocab, int64_t ld, int64_t ld_t, float grad_scale,
                   float w_ce, float w_kl, int64_t slice) {
    extern __shared__ __align__(128) unsigned char ce_smem[];
    __shared__ uint64_t bar;
    __shared__ Part parts[kCl];
    __shared__ Acc red[kThreads / 32];
    const uint32_t q = cluster_ctarank();
    const int64_t row = blockIdx.x / kCl;
    const int64_t c0 = (int64_t)q * slice;
    const int64_t n = vocab - c0 < slice ? vocab - c0 : slice;  // > 0 and a multiple of 8 (the launcher's split)
    const int32_t target = targets ? targets[row] : 0;
    const bool scored = target >= 0 && target < vocab;
    __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(ce_smem);
    __nv_bfloat16* ts = kTeacher ? xs + slice : nullptr;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t bytes = (uint32_t)(n * 2);
        mbar_expect_tx(&bar, kTeacher ? 2 * bytes : bytes);
        const char* src = reinterpret_cast<const char*>(logits + row * ld + c0);
        const char* srct = kTeacher ? reinterpret_cast<const char*>(teacher + row * ld_t + c0) : nullptr;
        for (uint32_t o = 0; o < bytes; o += 16384) {
            const uint32_t b = bytes - o < 16384 ? bytes - o : 16384;
            bulk_load(reinterpret_cast<char*>(xs) + o, src + o, b, &bar);
            if (kTeacher) bulk_load(reinterpret_cast<char*>(ts) + o, srct + o, b, &bar);
        }
    }
    const bool ok = mbar_wait(&bar, 0, nullptr);
    const int64_t nvec = n / 8;
    const uint4* xv = reinterpret_cast<const uint4*>(xs);
    const uint4* tv = kTeacher ? reinterpret_cast<const uint4*>(ts) : nullptr;
    Acc a{-INFINITY, 0.0f, -INFINITY, 0.0f, 0.0f};
    for (int64_t i = threadIdx.x; ok && i < nvec; i += kThreads) {
        float v[8];
        unpack8(xv[i], v);
        float mx = v[0];
#pragma unroll
        for (int k = 1; k < 8; ++k) mx = fmaxf(mx, v[k]);
        const float m = fmaxf(a.m, mx);
        float sm = a.m == -INFINITY ? 0.0f : a.s * fexp(a.m - m);
#pragma unroll
        for (int k = 0; k < 8; ++k) sm += fexp(v[k] - m);
        a.m = m;
        a.s = sm;
        if (kTeacher) {
            float t8[8];
            unpack8(tv[i], t8);
            float tm = t8[0];
#pragma unroll
            for (int k = 1; k < 8; ++k) tm = fmaxf(tm, t8[k]);
            const float mt = fmaxf(a.mt, tm);
            const float f = a.mt == -INFINITY ? 0.0f : fexp(a.mt - mt);
            float st = a.st * f, u = a.u * f;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float e = fexp(t8[k] - mt);
                st += e;
                u = fmaf(e, t8[k] - v[k], u);
            }
            a.mt = mt;
            a.st = st;
            a.u = u;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Acc b;
        b.m = __shfl_xor_sync(0xFFFFFFFFu, a.m, o);
        b.s = __shfl_xor_sync(0xFFFFFFFFu, a.s, o);
        b.mt = __shfl_xor_sync(0xFFFFFFFFu, a.mt, o);
        b.st = __shfl_xor_sync(0xFFFFFFFFu, a.st, o);
        b.u = __shfl_xor_sync(0xFFFFFFFFu, a.u, o);
        merge(a, b);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = a;
    __syncthreads();
    if (threadIdx.x < kCl) {
        // this CTA's sums (and the target's logit, if it is here) into slot q of every CTA of the cluster
        Acc r = red[0];
        for (int w = 1; w < kThreads / 32; ++w) merge(r, red[w]);
        const bool here = scored && target >= c0 && target < c0 + n;
        const float xt = here ? __bfloat162float(xs[target - c0]) : -INFINITY;
        const uint32_t dst = cluster_addr(&parts[q], (uint32_t)threadIdx.x);
        st_cluster_f32(dst + 0, r.m);
        st_cluster_f32(dst + 4, r.s);
        st_cluster_f32(dst + 8, r.mt);
        st_cluster_f32(dst + 12, r.st);
        st_cluster_f32(dst + 16, r.u);
        st_cluster_f32(dst + 20, xt);
    }
    cluster_sync();  // every CTA's slots are filled; no shared memory of another CTA is touched after this
    Acc r = parts[0].a;
    float xt = parts[0].xt;
    for (int c = 1; c < kCl; ++c) {
        merge(r, parts[c].a);
        xt = fmaxf(xt, parts[c].xt);
    }
    const float lse = r.m + logf(r.s);
    const float lse_t = kTeacher ? r.mt + logf(r.st) : 0.0f;
    if (q == 0 && threadIdx.x == 0) {
        // log(s) - (x_t - m), not lse - x_t: with a large row maximum, adding m first would round log(s)
        // away (the reference's ce_position keeps this order, src/loss.cpp:21-39)
        if (loss_ce) loss_ce[row] = scored && targets ? logf(r.s) - (xt - r.m) : 0.0f;
        if (loss_kl) loss_kl[row] = kTeacher && scored ? r.u / r.st - lse_t + lse : 0.0f;
    }
    if (!grad || !ok) return;
    uint4* g = reinterpret_cast<uint4*>(grad + row * ld + c0);
    const float ce_w = targets ? w_ce : 0.0f;
    const float sc = scored ? grad_scale : 0.0f;
    for (int64_t i = threadIdx.x; i < nvec; i += kThreads) {
        float v[8], t8[8], o[8];
        unpack8(xv[i], v);
        if (kTeacher) unpack8(tv[i], t8);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float p = fexp(v[k] - lse);
            float d = ce_w * p;
            if (kTeacher) d += w_kl * (p - fexp(t8[k] - lse_t));
            if (targets && c0 + i * 8 + k == target) d -= ce_w;
            o[k] = d * sc;
        }
        uint4 u;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(o[2 * k], o[2 * k + 1]);
        g[i] = u;
    }
}

}  // namespace

R97B_ERROR_READER(loss_error_word)

}  // namespace r97b

using namespace r97b;

// Loss and gradient of `rows` logit rows (bf16, row stride `ld`), optionally against teacher logits
// (row stride `ld_t`). `grad` may equal `logits` (in-place).
extern "C" int r97b_ce_kld(const uint16_t* logits, const uint16_t* teacher, const int32_t* targets, uint16_t* grad,
                           float* loss_ce, float* loss_kl, int64_t rows, int64_t vocab, int64_t ld, int64_t ld_t,
                           float grad_scale, float w_ce, float w_kl, void* stream) {
    if (!logits || rows <= 0 || vocab <= 0 || ld < vocab || (teacher && ld_t < vocab)) return R97B_EINVAL;
    if ((reinterpret_cast<uintptr_t>(logits) & 1) || (grad && (reinterpret_cast<uintptr_t>(grad) & 1)) ||
        (teacher && (reinterpret_cast<uintptr_t>(teacher) & 1)))
        return R97B_EINVAL;
    const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const int vec = (ld % 8) == 0 && a16(logits) && (!grad || a16(grad)) &&
                    (!teacher || ((ld_t % 8) == 0 && a16(teacher)));
    if (rows > 0x7FFFFFFF) return R97B_EINVAL;
    const auto* x = reinterpret_cast<const __nv_bfloat16*>(logits);
    const auto* t = reinterpret_cast<const __nv_bfloat16*>(teacher);
    auto* g = reinterpret_cast<__nv_bfloat16*>(grad);
    // the cluster form: quarters of whole 8-value vectors, each in shared memory
    const int64_t slice = ((vocab + kCl - 1) / kCl + 7) / 8 * 8;
    const int64_t smem = (teacher ? 2 : 1) * slice * 2;
    if (vec && vocab % 8 == 0 && vocab > (kCl - 1) * slice && smem <= 200 * 1024 && rows * kCl <= 0x7FFFFFFF) {
        if (teacher) {
            if (!smem_opt_in(ce_kld_cluster<true>, (int)smem)) return R97B_ELAUNCH;
            ce_kld_cluster<true><<<(unsigned)(rows * kCl), kThreads, smem, as_stream(stream)>>>(
                x, t, targets, g, loss_ce, loss_kl, vocab, ld, ld_t, grad_scale, w_ce, w_kl, slice);
        } else {
            if (!smem_opt_in(ce_kld_cluster<false>, (int)smem)) return R97B_ELAUNCH;
            ce_kld_cluster<false><<<(unsigned)(rows * kCl), kThreads, smem, as_stream(stream)>>>(
                x, nullptr, targets, g, loss_ce, loss_kl, vocab, ld, 0, grad_scale, w_ce, 0.0f, slice);
        }
        return launch_status();
    }
    if (teacher)
        ce_kld_kernel<true><<<(unsigned)rows, kThreads, 0, as_stream(stream)>>>(x, t, targets, g, loss_ce, loss_kl,
                                                                               vocab, ld, ld_t, grad_scale, w_ce, w_kl, vec);
    else
        ce_kld_kernel<false><<<(unsigned)rows, kThreads, 0, as_stream(stream)>>>(x, nullptr, targets, g, loss_ce,
                                                                                loss_kl, vocab, ld, 0, grad_scale,
                                                                                w_ce, 0.0f, vec);
    return launch_status();
}
