// attn_fwd.cu -- the forward of causal grouped-query attention on sm_100a tensor cores (tcgen05 + TMA + TMEM).
//
// The attention core of the hybrid model's gated-attention blocks (reference: attention_twin,
// src/adjoint/host/attention.cpp:261-313): for each query row q_t of head h (key/value head h / grp),
//
//   out_t = sum_{j <= t} softmax_j(scale q_t . k_j) v_j,     lse_t = log sum_{j <= t} e^{scale q_t . k_j}
//
// with lse the natural-log log-sum-exp the backward (attn.cu) reads. One persistent, warp-specialised kernel:
// a unit is 128 query rows of one head, and it runs in two passes over its key tiles (128 keys each, up to the
// diagonal):
//
//   pass 1  S = Q K^T into TMEM; the epilogue warps keep each row's running max and sum of exponentials
//   pass 2  S = Q K^T again; P = exp2(S scale log2e - lse log2e), exactly normalised since the row's lse is
//           known, is written as bf16 into shared memory in the MMA's K-major 128-byte-swizzled layout, and
//           O += P V accumulates in TMEM with no rescaling; the epilogue drains O into bf16 rows at the end.
//
// Q K^T is computed twice (the forward's tensor work is 1.5 x a single pass), which buys an accumulator that
// is never rescaled and a P that is already final when it is written. Roles: warp 0 issues TMA loads (Q once
// per unit, resident; K and V through a ring of 16 KiB stages), warp 1 issues tcgen05.mma (S double-buffered
// in TMEM, O beside it), warps 4-11 are the epilogue (two per TMEM lane quarter, each half of the columns).
// Every wait is bounded. No cluster multicast anywhere.
#include "sm100.cuh"
#include "r97b_internal.h"
#include "fastmath.cuh"

#include <cuda_bf16.h>

namespace r97b {

namespace {

constexpr int kQB = 128;        // query rows of a unit
constexpr int kKB = 128;        // keys of a tile
constexpr int kStageBytes = 16384;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kEpiWarps = 8;

template <int D>
struct FCfg {
    static constexpr int kStages = D == 256 ? 5 : 7;
    static constexpr int kQBytes = kQB * D * 2;           // D / 64 slabs of 128 rows x 64 columns
    static constexpr int kPBytes = kQB * kKB * 2;         // one P buffer: two slabs of 128 rows x 64 keys
    static constexpr int kPOff = kQBytes;
    static constexpr int kRingOff = kPOff + 2 * kPBytes;
    static constexpr int kBarOff = kRingOff + kStages * kStageBytes;
    static constexpr int kStatOff = kBarOff + 256;        // float2 [2 (unit parity)][2 (half)][128]
    static constexpr int kSmemBytes = kStatOff + 2 * 2 * 128 * 8 + 1024;
    static constexpr int kTmemCols = 512;                 // S[2]: columns 0..255; O: 256 .. 256 + D
    static constexpr int kVBytes = 32 * D * 2;            // one V stage: 32 keys x D (MN-major slabs of 64)
};

struct FwdArgs {
    int32_t B, Hq, Hkv, S, grp, nblk, units;
    float sl2;                 // scale * log2 e
    float* lse;                // [B*Hq*S] natural log
    __nv_bfloat16* out;        // [B*Hq*S, D]
};

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// A CTA's t-th unit: a snake over the longest-first order (query blocks descending), so a CTA's heavy
// unit of one round meets a light one in the next.
__device__ __forceinline__ int unit_of(int t, int c, int G) { return t * G + ((t & 1) ? (G - 1 - c) : c); }

__device__ __forceinline__ void unit_geom(const FwdArgs& a, int u, int& bh, int& i) {
    const int heads = a.B * a.Hq;
    const int r = u / heads;
    bh = u - r * heads;
    i = a.nblk - 1 - r;
}

template <int D>
__global__ void __launch_bounds__(128 + 32 * kEpiWarps, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tQ, const __grid_constant__ CUtensorMap tK,
                    const __grid_constant__ CUtensorMap tV, const FwdArgs args) {
    using C = FCfg<D>;
    constexpr int ND = D / 64;  // 64-wide column blocks of the head
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
    uint8_t* sQ = smem;
    uint8_t* sP = smem + C::kPOff;
    uint8_t* ring = smem + C::kRingOff;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* empty_bar = full_bar + C::kStages;
    uint64_t* q_full = empty_bar + C::kStages;
    uint64_t* q_empty = q_full + 1;
    uint64_t* s_full = q_empty + 1;   // [2]
    uint64_t* s_empty = s_full + 2;   // [2]
    uint64_t* p_full = s_empty + 2;   // [2]
    uint64_t* p_empty = p_full + 2;   // [2]
    uint64_t* o_full = p_empty + 2;
    uint64_t* o_empty = o_full + 1;
    uint64_t* stat_bar = o_empty + 1;  // [2]: both halves' row statistics of a unit written
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stat_bar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float2* stats = reinterpret_cast<float2*>(smem + C::kStatOff);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&s_empty[b], kEpiWarps);
            mbar_init(&p_full[b], kEpiWarps);
            mbar_init(&p_empty[b], 1);
        }
        mbar_init(o_full, 1);
        mbar_init(o_empty, kEpiWarps);
        mbar_init(&stat_bar[0], kEpiWarps);
        mbar_init(&stat_bar[1], kEpiWarps);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch(&tQ);
        tma_prefetch(&tK);
        tma_prefetch(&tV);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int G = gridDim.x, c = blockIdx.x;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------- TMA producer
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        auto take = [&]() -> uint8_t* {  // the next free ring stage, or null when a wait gave up
            if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) return nullptr;
            return ring + stage * kStageBytes;
        };
        auto next = [&]() {
            if (++stage == C::kStages) {
                stage = 0;
                phase ^= 1u;
            }
        };
        int lt = 0;
        for (int t = 0; ok; ++t) {
            const int u = unit_of(t, c, G);
            if (u >= args.units) {
                if (t * G >= args.units) break;
                continue;
            }
            int bh, i;
            unit_geom(args, u, bh, i);
            const int b = bh / args.Hq, h = bh - b * args.Hq;
            const int qrow = bh * args.S + i * kQB;
            const int krow0 = (b * args.Hkv + h / args.grp) * args.S;
            if (!mbar_wait(q_empty, (uint32_t)(lt & 1) ^ 1u, abort_flag)) break;
            mbar_expect_tx(q_full, C::kQBytes);
#pragma unroll
            for (int s = 0; s < ND; ++s) tma_load_2d(sQ + s * 16384, &tQ, q_full, 64 * s, qrow);
            auto load_k = [&](int j) {
                for (int kb = 0; kb < ND && ok; ++kb) {
                    uint8_t* st = take();
                    if (!st) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full_bar[stage], kStageBytes);
                    tma_load_2d(st, &tK, &full_bar[stage], 64 * kb, krow0 + kKB * j);
                    next();
                }
            };
            auto load_v = [&](int j) {
                for (int kb2 = 0; kb2 < 4 && ok; ++kb2) {
                    uint8_t* st = take();
                    if (!st) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full_bar[stage], C::kVBytes);
#pragma unroll
                    for (int n = 0; n < ND; ++n)
                        tma_load_2d(st + n * 4096, &tV, &full_bar[stage], 64 * n, krow0 + kKB * j + 32 * kb2);
                    next();
                }
            };
            for (int j = 0; j <= i && ok; ++j) load_k(j);  // pass 1
            if (ok) load_k(0);                             // pass 2: S_0, then S_{j+1} ahead of P_j V_j
            for (int j = 0; j <= i && ok; ++j) {
                if (j < i) load_k(j + 1);
                load_v(j);
            }
            ++lt;
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------- MMA issuer
        constexpr uint32_t idesc_s = make_idesc_bf16(kQB, kKB, 0, 0);
        constexpr uint32_t idesc_o = make_idesc_bf16(kQB, D, 0, 1);
        int stage = 0;
        uint32_t phase = 0;
        int sc = 0, pc = 0, lt = 0;
        bool ok = true;
        // S[sc & 1] = Q K_j^T over the head's column blocks
        auto issue_s = [&]() {
            const int sb = sc & 1;
            if (!mbar_wait(&s_empty[sb], (uint32_t)((sc >> 1) & 1) ^ 1u, abort_flag)) {
                ok = false;
                return;
            }
            tc_fence_after();
            const uint32_t d = tmem_base + (uint32_t)(sb * kKB);
            for (int kb = 0; kb < ND; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
                    ok = false;
                    return;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(sQ + kb * 16384);
                const uint32_t sbk = smem_u32(ring + stage * kStageBytes);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_f16(d, make_sdesc_sw128(sa + kk * 32, 16, 1024), make_sdesc_sw128(sbk + kk * 32, 16, 1024),
                             idesc_s, (kb > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&empty_bar[stage]);
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            umma_commit(&s_full[sb]);
            ++sc;
        };
        for (int t = 0; ok; ++t) {
            const int u = unit_of(t, c, G);
            if (u >= args.units) {
                if (t * G >= args.units) break;
                continue;
            }
            int bh, i;
            unit_geom(args, u, bh, i);
            if (!mbar_wait(q_full, (uint32_t)(lt & 1), abort_flag)) break;
            tc_fence_after();
            for (int j = 0; j <= i && ok; ++j) issue_s();  // pass 1
            if (!ok) break;
            issue_s();                                      // pass 2
            if (i == 0) umma_commit(q_empty);
            for (int j = 0; j <= i && ok; ++j) {
                if (j < i) {
                    issue_s();
                    if (j + 1 == i) umma_commit(q_empty);  // the unit's last use of Q
                }
                if (!ok) break;
                const int pb = pc & 1;
                if (!mbar_wait(&p_full[pb], (uint32_t)((pc >> 1) & 1), abort_flag)) {
                    ok = false;
                    break;
                }
                if (j == 0 && !mbar_wait(o_empty, (uint32_t)(lt & 1) ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t pbase = smem_u32(sP + pb * C::kPBytes);
                for (int kb2 = 0; kb2 < 4; ++kb2) {  // 32 keys a step
                    if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sv = smem_u32(ring + stage * kStageBytes);
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const uint32_t pa = pbase + (uint32_t)((kb2 >> 1) * 16384 + (kb2 & 1) * 64 + kk * 32);
                        umma_f16(tmem_base + 256u, make_sdesc_sw128(pa, 16, 1024),
                                 make_sdesc_sw128(sv + kk * 2048, 4096, 1024), idesc_o,
                                 (j > 0 || kb2 > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty_bar[stage]);
                    if (++stage == C::kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(&p_empty[pb]);
                ++pc;
            }
            if (!ok) break;
            umma_commit(o_full);
            ++lt;
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------- epilogue
        const int q = warp & 3;           // the TMEM lane quarter this warp may read
        const int sub = (warp - 4) >> 2;  // its half of the columns
        const int row = q * 32 + lane;    // this thread's query row in the unit
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        int sc = 0, pc = 0, lt = 0;
        bool ok = true;
        // reads this thread's 64 columns of S[sc & 1] into x (scaled to log2 units, masked), frees the buffer
        auto read_s = [&](float (&x)[64], bool diag) -> bool {
            const int sb = sc & 1;
            if (!mbar_wait(&s_full[sb], (uint32_t)((sc >> 1) & 1), abort_flag)) return false;
            tc_fence_after();
            uint32_t r0[32], r1[32];
            __syncwarp();
            tmem_ld32(tmem_base + lane_off + (uint32_t)(sb * kKB + sub * 64), r0);
            tmem_ld32(tmem_base + lane_off + (uint32_t)(sb * kKB + sub * 64 + 32), r1);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[sb]);
            ++sc;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                x[e] = __uint_as_float(r0[e]) * args.sl2;
                x[32 + e] = __uint_as_float(r1[e]) * args.sl2;
            }
            if (diag) {
#pragma unroll
                for (int e = 0; e < 64; ++e)
                    if (sub * 64 + e > row) x[e] = -INFINITY;
            }
            return true;
        };
        for (int t = 0; ok; ++t) {
            const int u = unit_of(t, c, G);
            if (u >= args.units) {
                if (t * G >= args.units) break;
                continue;
            }
            int bh, i;
            unit_geom(args, u, bh, i);
            const int64_t grow = (int64_t)bh * args.S + i * kQB + row;
            // pass 1: the row's max and sum of exponentials over this thread's columns
            float m = -INFINITY, l = 0.0f;
            for (int j = 0; j <= i; ++j) {
                float x[64];
                if (!(ok = read_s(x, j == i))) break;
                float mt = x[0];
#pragma unroll
                for (int e = 1; e < 64; ++e) mt = fmaxf(mt, x[e]);
                const float mn = fmaxf(m, mt);
                if (mn == -INFINITY) continue;  // every column of this half masked so far
                float s = 0.0f;
#pragma unroll
                for (int e = 0; e < 64; ++e) s += ex2_ftz(x[e] - mn);
                l = l * ex2_ftz(m - mn) + s;
                m = mn;
            }
            if (!ok) break;
            // both halves' statistics of the row -> its log-sum-exp (log2 units); key 0 is always visible
            // (an mbarrier, not a named barrier: its wait is bounded like every other; the buffer of a unit's
            // parity is written again two units later, when the other half has long read it)
            float2* st = stats + (lt & 1) * 256;
            st[sub * 128 + row] = make_float2(m, l);
            __syncwarp();
            if (lane == 0) mbar_arrive(&stat_bar[lt & 1]);
            if (!(ok = mbar_wait(&stat_bar[lt & 1], (uint32_t)((lt >> 1) & 1), abort_flag))) break;
            const float2 o2 = st[(sub ^ 1) * 128 + row];
            const float mf = fmaxf(m, o2.x);
            const float lf = (m == -INFINITY ? 0.0f : l * ex2_ftz(m - mf)) +
                             (o2.x == -INFINITY ? 0.0f : o2.y * ex2_ftz(o2.x - mf));
            const float lse2 = mf + __log2f(lf);
            if (sub == 0) args.lse[grow] = lse2 * kLn2;
            // pass 2: P = exp2(x - lse2) into the P buffer, K-major with the 128-byte swizzle
            for (int j = 0; j <= i; ++j) {
                float x[64];
                if (!(ok = read_s(x, j == i))) break;
                const int pb = pc & 1;
                if (!(ok = mbar_wait(&p_empty[pb], (uint32_t)((pc >> 1) & 1) ^ 1u, abort_flag))) break;
                uint8_t* slab = sP + pb * C::kPBytes + sub * 16384 + row * 128;
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    uint32_t pk[4];
#pragma unroll
                    for (int h2 = 0; h2 < 4; ++h2) {
                        const float p0 = ex2_ftz(x[ch * 8 + 2 * h2] - lse2);
                        const float p1 = ex2_ftz(x[ch * 8 + 2 * h2 + 1] - lse2);
                        const __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
                        pk[h2] = *reinterpret_cast<const uint32_t*>(&b2);
                    }
                    *reinterpret_cast<uint4*>(slab + ((ch ^ (row & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                fence_proxy_async_smem();  // the generic-proxy writes, seen by the tensor core's reads
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[pb]);
                ++pc;
            }
            if (!ok) break;
            // O: this thread's row, its half of the columns, as bf16
            if (!(ok = mbar_wait(o_full, (uint32_t)(lt & 1), abort_flag))) break;
            tc_fence_after();
            __nv_bfloat16* op = args.out + grow * D + sub * (D / 2);
#pragma unroll 1
            for (int cc = 0; cc < D / 2 / 32; ++cc) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld32(tmem_base + lane_off + 256u + (uint32_t)(sub * (D / 2) + cc * 32), r);
                tmem_ld_wait();
                uint4* dst = reinterpret_cast<uint4*>(op + cc * 32);
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    uint32_t pk[4];
#pragma unroll
                    for (int h2 = 0; h2 < 4; ++h2) {
                        const __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(r[w * 8 + h2 * 2]),
                                                                        __uint_as_float(r[w * 8 + h2 * 2 + 1]));
                        pk[h2] = *reinterpret_cast<const uint32_t*>(&b2);
                    }
                    dst[w] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_empty);
            ++lt;
        }
        if (!ok) *abort_flag = 1;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

template <int D>
int launch_fwd(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const FwdArgs& args,
               cudaStream_t stream) {
    using C = FCfg<D>;
    static_assert(C::kSmemBytes <= 232448, "shared memory");
    auto kern = attn_fwd_kernel<D>;
    if (!smem_opt_in(kern, (int)C::kSmemBytes)) return R97B_ELAUNCH;
    int grid = num_sms();
    if (args.units < grid) grid = args.units;
    kern<<<grid, 128 + 32 * kEpiWarps, C::kSmemBytes, stream>>>(q, k, v, args);
    return launch_status();
}

}  // namespace

R97B_ERROR_READER(attn_fwd_error_word)

}  // namespace r97b

extern "C" int r97b_attn_fwd(const R97bAttnFwd* a, void* stream) {
    using namespace r97b;
    if (!a) return R97B_EINVAL;
    const int B = a->B, Hq = a->Hq, Hkv = a->Hkv, S = a->S, D = a->D;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || S <= 0 || S % 128 != 0 || (D != 128 && D != 256))
        return R97B_EINVAL;
    if (!a->q || !a->k || !a->v || !a->o || !a->lse) return R97B_EINVAL;
    if ((int64_t)B * Hq * S > 0x7FFFFFFF / 2 || (int64_t)B * Hkv * S > 0x7FFFFFFF / 2) return R97B_EINVAL;
    if ((reinterpret_cast<uintptr_t>(a->o) & 15) != 0) return R97B_EINVAL;
    const int64_t rq = (int64_t)B * Hq * S, rk = (int64_t)B * Hkv * S;
    CUtensorMap mQ, mK, mV;
    if (!make_map(&mQ, a->q, D, rq, D, 64, 128) || !make_map(&mK, a->k, D, rk, D, 64, 128) ||
        !make_map(&mV, a->v, D, rk, D, 64, 32))
        return R97B_EINVAL;
    FwdArgs args{};
    args.B = B;
    args.Hq = Hq;
    args.Hkv = Hkv;
    args.S = S;
    args.grp = Hq / Hkv;
    args.nblk = S / 128;
    args.units = B * Hq * args.nblk;
    args.sl2 = a->scale * kLog2e;
    args.lse = a->lse;
    args.out = reinterpret_cast<__nv_bfloat16*>(a->o);
    cudaStream_t st = as_stream(stream);
    return D == 256 ? launch_fwd<256>(mQ, mK, mV, args, st) : launch_fwd<128>(mQ, mK, mV, args, st);
}
