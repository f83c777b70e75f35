// gemm_i8.cu -- the w8a8 trunk's int8 product on tcgen05 (kind::i8): the i8a8h form of gemm_nt_q, and the
// gated narrow fold gemm_nt_q_gated with its Hadamard quantiser in the epilogue.
//
//   y[m, n] = sum_g sa[m, g] sb[n, g] sum_{k in g} a[m, k] b[n, k]          groups of 128 along K
//
// (reference src/adjoint/host/linear.cpp:246-282, gemm_nt_q_twin at dtype i8a8h.) The fold
// (src/adjoint/host/gemm_nt_q_gated.cpp:11-14, 201-320) runs the same product over b = [gate rows; up rows],
// p[m, j] = act(z[m, j]) z[m, n + j] (act = silu, or sigmoid), and per 128-wide group of p: v = W p (W the
// unnormalised Walsh-Hadamard matrix, stages in ascending h, the lower index's sum first), s = amax|v| / 127
// (1 for an all-zero group), q = rint(clamp(v / s, +-127)) -- the [M, n] product is never written unless the
// caller asks for it (out_bf16).
//
// tcgen05 has no block-scaled int8 form for an f32 scale per row and 128-wide K group, so each group's exact
// s32 product is drained from tensor memory by the epilogue warps and folded into f32 registers with its two
// scales while the next group's MMAs run into the other half of tensor memory:
//   warp 0     TMA producer: per group a [128 x 128] int8 box of a and two of b, into a 4-deep ring
//   warp 1     MMA issuer: 4 x tcgen05.mma.kind::i8 (M 128, N 256, K 32) per group into TMEM buffer g & 1
//              (warps 2 and 3 only complete warpgroup 0, whose registers go to the epilogue: setmaxnreg)
//   warps 4-11 epilogue: warp w owns TMEM lanes 32 (w % 4) .. + 31 (its rows) and columns 128 ((w - 4) / 4)
//              .. + 127; per element acc += (t sb[n]) sa[m], t the group's exact integer sum as f32
// The conversion costs one add: every accumulator starts a group holding the bits of 1.5 * 2^23 (the epilogue
// writes them back as soon as it has drained a chunk), the MMAs add the group's sum to those bits as an
// integer (|sum| <= 128 * 127 * 127 < 2^22: no carry leaves the mantissa), and the bits read back are the float
// 1.5 * 2^23 + sum exactly. The fold runs on packed f32x2 instructions (two columns each); the TMEM loads are
// 16-column chunks with the next one in flight while the current one is folded in, which the 232 registers
// an epilogue thread gets (setmaxnreg, below) leave room for beside the 128 accumulators.
// One CTA per 128 x 256 output tile (for the fold: 128 gate columns and the 128 up columns they pair with),
// one CTA an SM (196 KB of shared memory, all 512 TMEM columns). The int8 operands are addressed through
// bf16-typed tensor maps of half the width: the 128-byte swizzle moves the same bytes either way.
#include "sm100.cuh"
#include "r97b_internal.h"

#include <cuda_bf16.h>
#include <stdint.h>

namespace r97b {
namespace {

constexpr int kBM = 128, kBN = 256, kGroup = 128;
constexpr int kStages = 4;
constexpr int kABytes = kBM * kGroup;            // 16 KB
constexpr int kStageBytes = kABytes + kBN * kGroup;  // 48 KB
constexpr int kScaleOff = kStages * kStageBytes;     // column scales [2][256] f32
constexpr int kBarOff = kScaleOff + 2 * kBN * 4;
constexpr int kSmem = kBarOff + 128 + 1024;          // + barriers, + the 1024-byte alignment slack
constexpr int kThreads = 384;  // warpgroup 0: producer, MMA issuer, two idle warps; 1-2: epilogue
constexpr int kPitch = 132;                          // f32 row pitch of the epilogue's staging rows
constexpr float kTop = 127.0f;

struct I8Args {
    const float* a_scale;
    const float* b_scale;
    int64_t ld_as, ld_bs;
    int64_t M, N, K;
    int groups;   // ceil(K / 128)
    int tiles_m;
    int gated;    // the fold
    int sigmoid;  // the fold's act
    int n_half;   // the fold: N / 2
    // plain output
    void* y;
    int64_t ldy;
    int y_bf16;
    // the fold's outputs
    int8_t* q;
    int64_t ldq;
    float* q_scale;
    int64_t ld_qs;
    __nv_bfloat16* out_bf16;
    int64_t ld_ob;
};

__host__ __device__ constexpr uint32_t make_idesc_i8(int M, int N) {
    return (2u << 4)                       // D format: s32
           | (1u << 7)                     // A format: signed 8-bit
           | (1u << 10)                    // B format: signed 8-bit
           | ((uint32_t)(N >> 3) << 17)    // N / 8
           | ((uint32_t)(M >> 4) << 24);   // M / 16
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::i8 (s8 inputs, s32 accumulator), one CTA.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

constexpr uint32_t kBiasBits = 0x4B400000u;  // the float 1.5 * 2^23

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_bias16(uint32_t taddr) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
                     taddr),
                 "r"(kBiasBits)
                 : "memory");
}

// Writes the bias bits into 32 consecutive columns of the warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_bias32(uint32_t taddr) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
        "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(kBiasBits)
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Packed f32 pairs (sm_100 f32x2 arithmetic, round to nearest).
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ uint64_t pk_bits(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ void unpk(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// The 256 epilogue threads' own barrier (named barrier 1).
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB, const I8Args args) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
    float* sbs = reinterpret_cast<float*>(smem + kScaleOff);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kBarOff);
    uint64_t* empty_bar = full_bar + kStages;
    uint64_t* acc_full = empty_bar + kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tm = blockIdx.x % args.tiles_m, tn = blockIdx.x / args.tiles_m;
    const int64_t m0 = (int64_t)tm * kBM;
    // the b rows of the tile's two 128-column halves
    const int64_t b_lo = args.gated ? (int64_t)tn * 128 : (int64_t)tn * kBN;
    const int64_t b_hi = args.gated ? args.n_half + (int64_t)tn * 128 : b_lo + 128;
    const int G = args.groups;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 8);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch(&tA);
        tma_prefetch(&tB);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // The launch gives every thread 168 registers; warpgroup 0 (one elected thread a role) gives 128 of its
    // back and each epilogue warpgroup takes 64 more: 128 x 40 + 256 x 232 = 384 x 168, the launch's total
    // (per SM sub-partition: one warp of warpgroup 0 and two epilogue warps, (40 + 2 x 232) x 32 = 16128).
    if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 40;" ::: "memory");
        if (warp == 0 && lane == 0) {
            // ------------------------------------------------------------- TMA producer
            for (int g = 0; g < G; ++g) {
                const int s = g % kStages;
                if (!mbar_wait(&empty_bar[s], ((g / kStages) & 1) ^ 1u, abort_flag)) break;
                uint8_t* st = smem + s * kStageBytes;
                mbar_expect_tx(&full_bar[s], kStageBytes);
                const int x = g * (kGroup / 2);  // in the maps' bf16 units
                tma_load_2d(st, &tA, &full_bar[s], x, (int32_t)m0);
                tma_load_2d(st + kABytes, &tB, &full_bar[s], x, (int32_t)b_lo);
                tma_load_2d(st + kABytes + 128 * kGroup, &tB, &full_bar[s], x, (int32_t)b_hi);
            }
        } else if (warp == 1 && lane == 0) {
            // ------------------------------------------------------------- MMA issuer
            constexpr uint32_t idesc = make_idesc_i8(kBM, kBN);
            for (int g = 0; g < G; ++g) {
                const int s = g % kStages, b = g & 1;
                if (!mbar_wait(&acc_empty[b], (g >> 1) & 1, abort_flag)) break;
                if (!mbar_wait(&full_bar[s], (g / kStages) & 1, abort_flag)) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * kStageBytes), sb = sa + kABytes;
#pragma unroll
                for (int kk = 0; kk < kGroup / 32; ++kk)
                    umma_i8(tmem + (uint32_t)(b * kBN), make_sdesc_sw128(sa + kk * 32, 16, 1024),
                            make_sdesc_sw128(sb + kk * 32, 16, 1024), idesc, 1u);  // onto the bias bits
                umma_commit(&empty_bar[s]);
                umma_commit(&acc_full[b]);
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 232;" ::: "memory");
        // ------------------------------------------------------------- epilogue
        const int e = warp - 4, qd = warp & 3, h = e >> 2, et = threadIdx.x - 128;
        const int row = 32 * qd + lane;
        const int64_t m = m0 + row;
        const bool mrow = m < args.M;
        const int64_t brow = et < 128 ? b_lo + et : b_hi + (et - 128);
        const bool bok = brow < args.N;
        const float* sa_row = args.a_scale + (mrow ? m : 0) * args.ld_as;
        const float* sb_row = args.b_scale + (bok ? brow : 0) * args.ld_bs;
        uint64_t acc2[64];  // column pairs (2 i, 2 i + 1)
#pragma unroll
        for (int i = 0; i < 64; ++i) acc2[i] = 0;
        float sa_nx = mrow ? sa_row[0] : 0.0f, sb_nx = bok ? sb_row[0] : 0.0f;
        bool ok = true;
        const uint32_t tlane = tmem + ((uint32_t)(32 * qd) << 16) + (uint32_t)(h * 128);
        // both accumulator buffers start at the bias; the MMA issuer's first wait on each is this arrival
#pragma unroll
        for (int c = 0; c < 8; ++c) tmem_bias32(tlane + (uint32_t)((c >> 2) * kBN + (c & 3) * 32));
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&acc_empty[0]);
            mbar_arrive(&acc_empty[1]);
        }
        const uint64_t neg_bias = pk(-12582912.0f, -12582912.0f);
#pragma unroll 1
        for (int g = 0; g < G; ++g) {
            const int b = g & 1;
            // slot b was last read in group g - 2, before the previous group's barrier
            sbs[b * kBN + et] = sb_nx;
            const float sa_g = sa_nx;
            if (g + 1 < G) {
                sa_nx = mrow ? sa_row[g + 1] : 0.0f;
                sb_nx = bok ? sb_row[g + 1] : 0.0f;
            }
            epi_bar();
            ok = __all_sync(0xFFFFFFFFu, ok && mbar_wait(&acc_full[b], (g >> 1) & 1, abort_flag));
            tc_fence_after();
            if (ok) {
                const float* sc = sbs + b * kBN + h * 128;
                const uint64_t sa2 = pk(sa_g, sa_g);
                // 16-column chunks: each written back to the bias as soon as it is drained, the next one's load
                // in flight while this one is folded in
                uint32_t ra[16], rb[16];
                const uint32_t tb = tlane + (uint32_t)(b * kBN);
                auto fold = [&](const uint32_t(&r)[16], int c) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 s4 = *reinterpret_cast<const float4*>(sc + c * 16 + 4 * i);
                        acc2[c * 8 + 2 * i] = fma2(mul2(add2(pk_bits(r[4 * i], r[4 * i + 1]), neg_bias),
                                                        pk(s4.x, s4.y)), sa2, acc2[c * 8 + 2 * i]);
                        acc2[c * 8 + 2 * i + 1] = fma2(mul2(add2(pk_bits(r[4 * i + 2], r[4 * i + 3]), neg_bias),
                                                            pk(s4.z, s4.w)), sa2, acc2[c * 8 + 2 * i + 1]);
                    }
                };
                tmem_ld16(tb, ra);
#pragma unroll
                for (int c = 0; c < 8; c += 2) {
                    tmem_ld_wait();
                    tmem_bias16(tb + (uint32_t)(c * 16));
                    tmem_ld16(tb + (uint32_t)((c + 1) * 16), rb);
                    fold(ra, c);
                    tmem_ld_wait();
                    tmem_bias16(tb + (uint32_t)((c + 1) * 16));
                    if (c + 2 < 8) tmem_ld16(tb + (uint32_t)((c + 2) * 16), ra);
                    fold(rb, c + 1);
                }
                tmem_st_wait();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        float acc[128];
#pragma unroll
        for (int i = 0; i < 64; ++i) unpk(acc2[i], acc[2 * i], acc[2 * i + 1]);
        // every MMA has completed (each warp saw the last group's commit): the ring is free for staging
        float* ring = reinterpret_cast<float*>(smem);
        if (!args.gated) {
            if (ok) {
                float* st = ring + e * 32 * kPitch;
#pragma unroll
                for (int c = 0; c < 32; ++c)
                    *reinterpret_cast<float4*>(st + lane * kPitch + 4 * c) =
                        make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
                __syncwarp();
                const int64_t n = (int64_t)tn * kBN + h * 128 + 4 * lane;
                if (n < args.N) {
#pragma unroll 4
                    for (int r = 0; r < 32; ++r) {
                        const int64_t mm = m0 + 32 * qd + r;
                        if (mm >= args.M) break;
                        const float4 v = *reinterpret_cast<const float4*>(st + r * kPitch + 4 * lane);
                        if (args.y_bf16) {
                            __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
                            uint2 u;
                            u.x = *reinterpret_cast<uint32_t*>(&lo);
                            u.y = *reinterpret_cast<uint32_t*>(&hi);
                            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(args.y) + mm * args.ldy + n) = u;
                        } else {
                            *reinterpret_cast<float4*>(reinterpret_cast<float*>(args.y) + mm * args.ldy + n) = v;
                        }
                    }
                }
            }
        } else {
            // the up half hands its rows to the gate half through shared memory
            float* zrow = ring + qd * 32 * kPitch + lane * kPitch;
            if (ok && h == 1) {
#pragma unroll
                for (int c = 0; c < 32; ++c)
                    *reinterpret_cast<float4*>(zrow + 4 * c) =
                        make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
            }
            epi_bar();
            if (ok && h == 0) {
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float4 u = *reinterpret_cast<const float4*>(zrow + 4 * c);
                    const float uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float z = acc[4 * c + j];
                        const float sg = 1.0f / (1.0f + __expf(-z));
                        acc[4 * c + j] = (args.sigmoid ? sg : z * sg) * uu[j];
                    }
                }
                const int64_t j0 = (int64_t)tn * 128;
                float* st = ring + (4 + qd) * 32 * kPitch;
                if (args.out_bf16) {  // the unrotated product
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        *reinterpret_cast<float4*>(st + lane * kPitch + 4 * c) =
                            make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
                    __syncwarp();
#pragma unroll 4
                    for (int r = 0; r < 32; ++r) {
                        const int64_t mm = m0 + 32 * qd + r;
                        if (mm >= args.M) break;
                        const float4 v = *reinterpret_cast<const float4*>(st + r * kPitch + 4 * lane);
                        __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
                        uint2 w;
                        w.x = *reinterpret_cast<uint32_t*>(&lo);
                        w.y = *reinterpret_cast<uint32_t*>(&hi);
                        *reinterpret_cast<uint2*>(args.out_bf16 + mm * args.ld_ob + j0 + 4 * lane) = w;
                    }
                    __syncwarp();
                }
                // v = W p, in the reference's stage order
#pragma unroll
                for (int hh = 1; hh < 128; hh <<= 1)
#pragma unroll
                    for (int i = 0; i < 128; ++i)
                        if (!(i & hh)) {
                            const float x0 = acc[i], x1 = acc[i + hh];
                            acc[i] = x0 + x1;
                            acc[i + hh] = x0 - x1;
                        }
                float amax = 0.0f;
#pragma unroll
                for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(acc[i]));
                const float s = amax > 0.0f ? amax / kTop : 1.0f, inv = 1.0f / s;
                uint32_t* cs = reinterpret_cast<uint32_t*>(st);  // 33-word rows: conflict-free
#pragma unroll
                for (int w = 0; w < 32; ++w) {
                    uint32_t word = 0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int c = __float2int_rn(fminf(fmaxf(acc[4 * w + j] * inv, -kTop), kTop));
                        word |= (uint32_t)(c & 0xFF) << (8 * j);
                    }
                    cs[lane * 33 + w] = word;
                }
                __syncwarp();
#pragma unroll 4
                for (int r = 0; r < 32; ++r) {
                    const int64_t mm = m0 + 32 * qd + r;
                    if (mm >= args.M) break;
                    *reinterpret_cast<uint32_t*>(args.q + mm * args.ldq + j0 + 4 * lane) = cs[r * 33 + lane];
                }
                if (mrow) args.q_scale[m * args.ld_qs + j0 / 128] = s;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

bool al(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) & (uintptr_t)(bytes - 1)) == 0; }

// The rules shared by both entry points; fills the maps and the geometry.
int prepare(const int8_t* a, int64_t lda, const float* a_scale, int64_t ld_as, const int8_t* b, int64_t ldb,
            const float* b_scale, int64_t ld_bs, int64_t M, int64_t N, int64_t K, CUtensorMap* mA, CUtensorMap* mB,
            I8Args* x) {
    if (!a || !b || !a_scale || !b_scale || M < 0 || N <= 0 || K <= 0) return R97B_EINVAL;
    const int64_t groups = (K + kGroup - 1) / kGroup;
    if (K % 16 || lda < K || ldb < K || lda % 16 || ldb % 16 || !al(a, 16) || !al(b, 16) || ld_as < groups ||
        ld_bs < groups || groups > (1 << 20))
        return R97B_EINVAL;
    if (!make_map(mA, a, K / 2, M > 0 ? M : 1, lda / 2, 64, 128) || !make_map(mB, b, K / 2, N, ldb / 2, 64, 128))
        return R97B_EINVAL;
    x->a_scale = a_scale, x->b_scale = b_scale, x->ld_as = ld_as, x->ld_bs = ld_bs;
    x->M = M, x->N = N, x->K = K, x->groups = (int)groups;
    x->tiles_m = (int)((M + kBM - 1) / kBM);
    return R97B_OK;
}

int launch(const CUtensorMap& mA, const CUtensorMap& mB, const I8Args& x, int64_t tiles_n, cudaStream_t s) {
    const int64_t tiles = (int64_t)x.tiles_m * tiles_n;
    if (tiles <= 0) return R97B_OK;
    if (tiles > INT32_MAX) return R97B_EINVAL;
    if (!smem_opt_in(gemm_i8_kernel, kSmem)) return R97B_ELAUNCH;
    gemm_i8_kernel<<<(unsigned)tiles, kThreads, kSmem, s>>>(mA, mB, x);
    return launch_status();
}

}  // namespace

R97B_ERROR_READER(gemm_i8_error_word)

}  // namespace r97b

using namespace r97b;

extern "C" int r97b_gemm_i8g(const int8_t* a, int64_t lda, const float* a_scale, int64_t ld_as, const int8_t* b,
                             int64_t ldb, const float* b_scale, int64_t ld_bs, int64_t M, int64_t N, int64_t K,
                             void* y, int64_t ldy, int32_t y_bf16, void* stream) {
    CUtensorMap mA, mB;
    I8Args x{};
    int rc = prepare(a, lda, a_scale, ld_as, b, ldb, b_scale, ld_bs, M, N, K, &mA, &mB, &x);
    if (rc != R97B_OK) return rc;
    if (!y || ldy < N || N % 4 || ldy % 4 || !al(y, y_bf16 ? 8 : 16)) return R97B_EINVAL;
    x.y = y, x.ldy = ldy, x.y_bf16 = y_bf16 ? 1 : 0;
    if (M == 0) return R97B_OK;
    return launch(mA, mB, x, (N + kBN - 1) / kBN, as_stream(stream));
}

extern "C" int r97b_gemm_i8g_gated(const int8_t* a, int64_t lda, const float* a_scale, int64_t ld_as,
                                   const int8_t* b, int64_t ldb, const float* b_scale, int64_t ld_bs, int64_t M,
                                   int64_t N, int64_t K, int32_t act_sigmoid, int8_t* q, int64_t ldq, float* q_scale,
                                   int64_t ld_qs, uint16_t* out_bf16, int64_t ld_ob, void* stream) {
    CUtensorMap mA, mB;
    I8Args x{};
    int rc = prepare(a, lda, a_scale, ld_as, b, ldb, b_scale, ld_bs, M, N, K, &mA, &mB, &x);
    if (rc != R97B_OK) return rc;
    const int64_t n = N / 2;
    if (N % 2 || n % kGroup || !q || !q_scale || ldq < n || ldq % 4 || !al(q, 4) || ld_qs < n / kGroup)
        return R97B_EINVAL;
    if (out_bf16 && (ld_ob < n || ld_ob % 4 || !al(out_bf16, 8))) return R97B_EINVAL;
    x.gated = 1, x.sigmoid = act_sigmoid ? 1 : 0, x.n_half = (int)n;
    x.q = q, x.ldq = ldq, x.q_scale = q_scale, x.ld_qs = ld_qs;
    x.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16), x.ld_ob = ld_ob;
    if (M == 0) return R97B_OK;
    if (n > INT32_MAX) return R97B_EINVAL;
    return launch(mA, mB, x, n / kGroup, as_stream(stream));
}
