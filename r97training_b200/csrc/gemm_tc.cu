// gemm_tc.cu -- the tensor-core GEMM of the LoRA-over-IQR path on sm_100a (tcgen05 + TMA + TMEM).
//
//   D[M, N] = alpha * ( sum_k A1[m, k] B1[n, k]  +  sum_k A2[m, k] B2[n, k] )  (+ beta * C[m, n])
//
// The second (A2, B2) segment is the LoRA tail: the forward is Y = [X | s t] [W | B]^T and the input
// adjoint is dX = [dY | dt] [W ; A], so the adapter's products ride in the same tile loop as the base
// weight's, one extra 64-wide k block at the end of each tile (reference: lora_expand's add into y,
// src/adjoint/host/lora.cpp:416-471, and the two dX terms gemm_nt_adjoint + lora_shrink_host_adjoint).
// Each operand is bf16 and either K-major (row-major [rows, K]) or MN-major (row-major [K, rows]); the
// MN-major form lets the adjoint read the weight [N, K] as is, and the adapter-gradient GEMMs reduce
// over tokens without a transpose.
//
// Structure: one persistent CTA per SM; warp 0 issues TMA loads into a ring of shared-memory stages,
// warp 1 issues tcgen05.mma (128 x BN x 16) into a double-buffered TMEM accumulator, and warps 4-7
// drain the accumulator (tcgen05.ld) and apply the epilogue while the next tile's MMAs run.
// No cluster multicast anywhere: every CTA loads its own tiles.
#include "sm100.cuh"
#include "r97b_internal.h"
#include "fastmath.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

namespace r97b {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;               // one 128-byte swizzle row of bf16
constexpr int kThreads = 256;         // 8 warps: 0 TMA, 1 MMA, 4..7 epilogue
constexpr int kABytes = kBM * kBK * 2;  // 16 KiB

struct KernelArgs {
    int32_t M, N;
    int32_t k1_blocks, k2_blocks;
    int32_t kb_per_split, splits;
    int32_t tiles_m, tiles_n;
    int32_t band;  // M-tiles a band of the tile order walks (tile_coords)
    int32_t mode;
    float alpha, beta;
    void* out;
    int64_t ldo;
    const __nv_bfloat16* addend;
    int64_t ld_add;
    float* ws_part;  // kEpiSplitBf16: f32 partial tiles [splits][tiles][kBM][BN]
    int* ws_cnt;     // kEpiSplitBf16: per-tile count of finished splits (back to 0 after the tile's fix-up)
    __nv_bfloat16* out2;  // kEpiSwiglu: silu(g) u
    int64_t ldo2;
    int32_t half_n;       // kEpiSwiglu / kEpiSwigluBwd: F, the offset of the up columns
};

// SwiGLU's pieces, with the arithmetic of the standalone SwiGLU kernels (layers.cu), so the fused
// epilogues produce the same bits.
__device__ __forceinline__ float sw_sigm(float x) { return sigmoid_ftz(x); }
__device__ __forceinline__ float sw_silu(float x) { return x * sw_sigm(x); }
__device__ __forceinline__ float sw_silu_grad(float x) {
    const float s = sw_sigm(x);
    return s * (1.0f + x * (1.0f - s));
}
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void load32_bf16(const __nv_bfloat16* p, float (&v)[32]) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint4 q = reinterpret_cast<const uint4*>(p)[w];
        const uint32_t xs[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xs[h]));
            v[w * 8 + 2 * h] = f.x;
            v[w * 8 + 2 * h + 1] = f.y;
        }
    }
}

__device__ __forceinline__ void store32_bf16(__nv_bfloat16* p, const float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        uint4 pk;
        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[i], v[i + 1]);
        __nv_bfloat162 h1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]);
        __nv_bfloat162 h3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
        pk.x = *reinterpret_cast<uint32_t*>(&h0);
        pk.y = *reinterpret_cast<uint32_t*>(&h1);
        pk.z = *reinterpret_cast<uint32_t*>(&h2);
        pk.w = *reinterpret_cast<uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(p + i) = pk;
    }
}

// The 128 epilogue threads (warps 4-7) synchronise among themselves on named barrier 1.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// ... and agree on a flag: true only if it is true in every epilogue thread.
__device__ __forceinline__ bool epi_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

template <int BN>
struct Cfg {
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = (200 * 1024) / kStageBytes > 8 ? 8 : (200 * 1024) / kStageBytes;
    static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// The tile order: bands of up to `band` M-tiles, N-tiles walked inside a band with M fastest, so one wave of
// persistent CTAs works on a band's A rows (which stay in L2 across the band's waves) against a few
// N-tiles of B, instead of all of A against two or three N-tiles.
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int band, int& tm, int& tn) {
    const int b = tile / (band * tiles_n);
    const int m_base = b * band;
    const int gm = min(band, tiles_m - m_base);
    const int r = tile - b * band * tiles_n;
    tm = m_base + r % gm;
    tn = r / gm;
}

// v[i] += beta * addend[m, n0 + i]: four 16-byte loads when the 32 columns are in range and aligned.
__device__ __forceinline__ void add_addend32(const KernelArgs& args, int m, int n0, bool full, float (&v)[32]) {
    const __nv_bfloat16* ap = args.addend + (int64_t)m * args.ld_add + n0;
    if (full && (reinterpret_cast<uintptr_t>(ap) & 15) == 0) {
        uint4 q[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) q[w] = reinterpret_cast<const uint4*>(ap)[w];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const uint32_t xs[4] = {q[w].x, q[w].y, q[w].z, q[w].w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xs[h]));
                v[w * 8 + 2 * h] += args.beta * f.x;
                v[w * 8 + 2 * h + 1] += args.beta * f.y;
            }
        }
    } else {
        for (int i = 0; i < 32; ++i)
            if (full || n0 + i < args.N) v[i] += args.beta * __bfloat162float(ap[i]);
    }
}

// The epilogue of 32 accumulator columns [n0, n0 + 32) of row m (r = the raw f32 bits), per `mode`.
__device__ __forceinline__ void epilogue32(const KernelArgs& args, int mode, int m, int n0, const uint32_t (&r)[32]) {
    const bool full = n0 + 32 <= args.N;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * args.alpha;
    if (mode == kEpiStoreBf16) {
        if (args.addend) add_addend32(args, m, n0, full, v);
        __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(args.out) + (int64_t)m * args.ldo + n0;
        if (full && ((reinterpret_cast<uintptr_t>(op) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
                uint4 pk;
                __nv_bfloat162 h0 = __floats2bfloat162_rn(v[i], v[i + 1]);
                __nv_bfloat162 h1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
                __nv_bfloat162 h2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]);
                __nv_bfloat162 h3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
                pk.x = *reinterpret_cast<uint32_t*>(&h0);
                pk.y = *reinterpret_cast<uint32_t*>(&h1);
                pk.z = *reinterpret_cast<uint32_t*>(&h2);
                pk.w = *reinterpret_cast<uint32_t*>(&h3);
                *reinterpret_cast<uint4*>(op + i) = pk;
            }
        } else {
            for (int i = 0; i < 32; ++i)
                if (n0 + i < args.N) op[i] = __float2bfloat16_rn(v[i]);
        }
    } else if (mode == kEpiStoreF32) {
        float* op = reinterpret_cast<float*>(args.out) + (int64_t)m * args.ldo + n0;
        if (args.addend) add_addend32(args, m, n0, full, v);
        if (full && ((reinterpret_cast<uintptr_t>(op) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(op + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else {
            for (int i = 0; i < 32; ++i)
                if (n0 + i < args.N) op[i] = v[i];
        }
    } else if (mode == kEpiSwigluBwd) {
        // d = the rounded da; dg = d u silu'(g), du = d silu(g)
        const __nv_bfloat16* gp = args.addend + (int64_t)m * args.ld_add + n0;
        __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(args.out) + (int64_t)m * args.ldo + n0;
        if (full && ((reinterpret_cast<uintptr_t>(gp) | reinterpret_cast<uintptr_t>(op)) & 15) == 0) {
            float g[32], u[32], og[32];
            load32_bf16(gp, g);
            load32_bf16(gp + args.half_n, u);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float d = bf16_round(v[i]);
                og[i] = d * u[i] * sw_silu_grad(g[i]);
                v[i] = d * sw_silu(g[i]);
            }
            store32_bf16(op, og);
            store32_bf16(op + args.half_n, v);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                if (n0 + i < args.N) {
                    const float d = bf16_round(v[i]);
                    const float g = __bfloat162float(gp[i]), u = __bfloat162float(gp[args.half_n + i]);
                    op[i] = __float2bfloat16_rn(d * u * sw_silu_grad(g));
                    op[args.half_n + i] = __float2bfloat16_rn(d * sw_silu(g));
                }
            }
        }
    } else if (mode == kEpiAtomicF32) {
        float* op = reinterpret_cast<float*>(args.out) + (int64_t)m * args.ldo + n0;
        if (full && ((reinterpret_cast<uintptr_t>(op) & 15) == 0)) {
            // one 16-byte vector reduction per four columns: a quarter of the L2 atomic operations
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                atomicAdd(reinterpret_cast<float4*>(op + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
        } else {
            for (int i = 0; i < 32; ++i)
                if (n0 + i < args.N) atomicAdd(op + i, v[i]);
        }
    } else {  // kEpiAtomicF32T: out[n, m] += acc[m, n]
        float* op = reinterpret_cast<float*>(args.out) + (int64_t)n0 * args.ldo + m;
        for (int i = 0; i < 32; ++i)
            if (full || n0 + i < args.N) atomicAdd(op + (int64_t)i * args.ldo, v[i]);
    }
}

template <int BN, int A_MN, int B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tA1, const __grid_constant__ CUtensorMap tB1,
                const __grid_constant__ CUtensorMap tA2, const __grid_constant__ CUtensorMap tB2,
                const KernelArgs args) {
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
    uint64_t* empty_bar = full_bar + C::kStages;
    uint64_t* tfull_bar = empty_bar + C::kStages;
    uint64_t* tempty_bar = tfull_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* split_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 128);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch(&tA1);
        tma_prefetch(&tB1);
        if (args.k2_blocks > 0) {
            tma_prefetch(&tA2);
            tma_prefetch(&tB2);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int k_total = args.k1_blocks + args.k2_blocks;
    const int tiles = args.tiles_m * args.tiles_n;
    const int units = tiles * args.splits;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------- TMA producer
        int stage = 0;
        uint32_t phase = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            const int split = u / tiles;
            const int tile = u % tiles;
            int tm, tn;
            tile_coords(tile, args.tiles_m, args.tiles_n, args.band, tm, tn);
            const int kb0 = split * args.kb_per_split;
            const int kb1 = min(k_total, kb0 + args.kb_per_split);
            bool ok = true;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                uint8_t* sa = smem + stage * C::kStageBytes;
                uint8_t* sb = sa + kABytes;
                mbar_expect_tx(&full_bar[stage], C::kStageBytes);
                const bool seg2 = kb >= args.k1_blocks;
                const CUtensorMap* ma = seg2 ? &tA2 : &tA1;
                const CUtensorMap* mb = seg2 ? &tB2 : &tB1;
                const int k = (seg2 ? kb - args.k1_blocks : kb) * kBK;
                const int m0 = tm * kBM, n0 = tn * BN;
                if (A_MN) {
                    tma_load_2d(sa, ma, &full_bar[stage], m0, k);
                    tma_load_2d(sa + 8192, ma, &full_bar[stage], m0 + 64, k);
                } else {
                    tma_load_2d(sa, ma, &full_bar[stage], k, m0);
                }
                if (B_MN) {
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, mb, &full_bar[stage], n0 + 64 * j, k);
                } else {
                    tma_load_2d(sb, mb, &full_bar[stage], k, n0);
                }
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------- MMA issuer
        constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, A_MN, B_MN);
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
            const int split = u / tiles;
            const int kb0 = split * args.kb_per_split;
            const int kb1 = min(k_total, kb0 + args.kb_per_split);
            const int acc = local & 1;
            if (!mbar_wait(&tempty_bar[acc], ((local >> 1) & 1) ^ 1u, abort_flag)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
            bool ok = true;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + stage * C::kStageBytes);
                const uint32_t sb = sa + kABytes;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint64_t ad = A_MN ? make_sdesc_sw128(sa + kk * 2048, 8192, 1024)
                                             : make_sdesc_sw128(sa + kk * 32, 16, 1024);
                    const uint64_t bd = B_MN ? make_sdesc_sw128(sb + kk * 2048, 8192, 1024)
                                             : make_sdesc_sw128(sb + kk * 32, 16, 1024);
                    umma_f16(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&empty_bar[stage]);
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            umma_commit(&tfull_bar[acc]);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------- epilogue
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const bool split_mode = args.mode == kEpiSplitBf16;
        int local = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
            const int tile = u % tiles;
            int tm, tn;
            tile_coords(tile, args.tiles_m, args.tiles_n, args.band, tm, tn);
            const int acc = local & 1;
            bool ok = mbar_wait(&tfull_bar[acc], (local >> 1) & 1, abort_flag);
            if (split_mode) ok = epi_all(ok);  // the fix-up below syncs the four warps: they leave together
            if (!ok) break;
            tc_fence_after();
            const int m = tm * kBM + q * 32 + lane;
            const bool mrow = m < args.M;
            if (split_mode) {
                // store this split's partial tile, release the accumulator, count the split in; the tile's
                // last split sums every split's partial in split order and stores the bf16 result
                const int split = u / tiles;
                const int row = q * 32 + lane;
                float* part = args.ws_part + (((int64_t)split * tiles + tile) * kBM + row) * BN;
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t r[32];
                    __syncwarp();
                    tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
                    tmem_ld_wait();
                    float4* dst = reinterpret_cast<float4*>(part + c * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        dst[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                             __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
                }
                tc_fence_before();
                mbar_arrive(&tempty_bar[acc]);
                __threadfence();
                epi_sync();
                if (threadIdx.x == 128) {
                    const int done = atomicAdd(args.ws_cnt + tile, 1) + 1;
                    const int last = done == args.splits;
                    if (last) atomicExch(args.ws_cnt + tile, 0);
                    *split_flag = last;
                }
                epi_sync();
                if (*split_flag) {
                    __threadfence();
                    const float* p0 = args.ws_part + ((int64_t)tile * kBM + row) * BN;
                    const int64_t split_stride = (int64_t)tiles * kBM * BN;
#pragma unroll 1
                    for (int c = 0; c < BN / 32; ++c) {
                        const int n0 = tn * BN + c * 32;
                        if (!mrow || n0 >= args.N) continue;
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = 0.0f;
                        for (int sp = 0; sp < args.splits; ++sp) {
                            const float4* src = reinterpret_cast<const float4*>(p0 + sp * split_stride + c * 32);
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                const float4 x = __ldcg(src + i);
                                v[4 * i] += x.x;
                                v[4 * i + 1] += x.y;
                                v[4 * i + 2] += x.z;
                                v[4 * i + 3] += x.w;
                            }
                        }
                        uint32_t r[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
                        epilogue32(args, kEpiStoreBf16, m, n0, r);
                    }
                }
                continue;
            }
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                __syncwarp();  // tcgen05.ld is .sync.aligned: the warp must be converged
                tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
                tmem_ld_wait();
                const int n0 = tn * BN + c * 32;
                if (!mrow || n0 >= args.N) continue;
                epilogue32(args, args.mode, m, n0, r);
            }
            tc_fence_before();
            mbar_arrive(&tempty_bar[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}


// ---------------------------------------------------------------------------- the CTA-pair kernel
// A cluster of two CTAs on two SMs computes 256 x 256 tiles with tcgen05.mma.cta_group::2: CTA rank r
// loads rows [128 r, 128 r + 128) of the tile's A and of its B into its own shared memory (same offsets
// in both), the leader (rank 0) issues M = 256, N = 256 MMAs that read both CTAs' halves, and each CTA
// drains its own 128 rows of the accumulator from its own tensor memory. Per SM that is half the operand
// bytes per multiply-add of the single-CTA 128 x 256 tile. The peer's TMA loads complete on the leader's
// "full" barrier; the leader's commits arrive on both CTAs' "empty" and "accumulator full" barriers; both
// CTAs' epilogues arrive on the leader's "accumulator empty" barrier. Every wait is bounded.
struct CfgPair {
    static constexpr int kHalfBytes = 128 * kBK * 2;           // one CTA's 128 x 64 slice of A or B: 16 KiB
    static constexpr int kStageBytes = 2 * kHalfBytes;         // its A and B slices
    static constexpr int kStages = 6;
    static constexpr int kTmemCols = 512;                      // two 256-column accumulators
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;
};

template <int A_MN, int B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tA1, const __grid_constant__ CUtensorMap tB1,
                     const __grid_constant__ CUtensorMap tA2, const __grid_constant__ CUtensorMap tB2,
                     const KernelArgs args) {
    using C = CfgPair;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
    uint64_t* empty_bar = full_bar + C::kStages;
    uint64_t* tfull_bar = empty_bar + C::kStages;
    uint64_t* tempty_bar = tfull_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0: the leader, 1: its peer
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full_bar[s], 1);   // the leader's expect_tx; both CTAs' bytes
            mbar_init(&empty_bar[s], 1);  // the leader's commit
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 256);  // both CTAs' 128 epilogue threads (used on the leader)
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, C::kTmemCols);
        tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch(&tA1);
        tma_prefetch(&tB1);
        if (args.k2_blocks > 0) {
            tma_prefetch(&tA2);
            tma_prefetch(&tB2);
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int k_total = args.k1_blocks + args.k2_blocks;
    const int tiles = args.tiles_m * args.tiles_n;  // 256 x 256 tiles
    const int units = tiles * args.splits;
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------- TMA producer (both CTAs)
        int stage = 0;
        uint32_t phase = 0;
        for (int u = pair; u < units; u += pairs) {
            const int split = u / tiles;
            const int tile = u % tiles;
            int tm, tn;
            tile_coords(tile, args.tiles_m, args.tiles_n, args.band, tm, tn);
            const int kb0 = split * args.kb_per_split;
            const int kb1 = min(k_total, kb0 + args.kb_per_split);
            bool ok = true;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                uint8_t* sa = smem + stage * C::kStageBytes;
                uint8_t* sb = sa + C::kHalfBytes;
                const uint32_t bar = cluster_addr(&full_bar[stage], 0);  // the leader's
                if (leader) mbar_expect_tx(&full_bar[stage], 2 * C::kStageBytes);
                const bool seg2 = kb >= args.k1_blocks;
                const CUtensorMap* ma = seg2 ? &tA2 : &tA1;
                const CUtensorMap* mb = seg2 ? &tB2 : &tB1;
                const int k = (seg2 ? kb - args.k1_blocks : kb) * kBK;
                const int m0 = tm * 256 + 128 * (int)rank;
                // SwiGLU: rank 0 brings the tile's gate rows and rank 1 the matching up rows, so the pair's
                // 256 accumulator columns are [g | u] of the same 128 output columns
                const int n0 = args.mode == kEpiSwiglu ? (rank ? args.half_n : 0) + tn * 128
                                                       : tn * 256 + 128 * (int)rank;
                if (A_MN) {
                    tma_load_2d_pair(sa, ma, bar, m0, k);
                    tma_load_2d_pair(sa + 8192, ma, bar, m0 + 64, k);
                } else {
                    tma_load_2d_pair(sa, ma, bar, k, m0);
                }
                if (B_MN) {
                    tma_load_2d_pair(sb, mb, bar, n0, k);
                    tma_load_2d_pair(sb + 8192, mb, bar, n0 + 64, k);
                } else {
                    tma_load_2d_pair(sb, mb, bar, k, n0);
                }
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
        }
    } else if (warp == 1 && lane == 0 && leader) {
        // ------------------------------------------------------------- MMA issuer (the leader)
        constexpr uint32_t idesc = make_idesc_bf16(256, 256, A_MN, B_MN);
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        for (int u = pair; u < units; u += pairs, ++local) {
            const int split = u / tiles;
            const int kb0 = split * args.kb_per_split;
            const int kb1 = min(k_total, kb0 + args.kb_per_split);
            const int acc = local & 1;
            if (!mbar_wait(&tempty_bar[acc], ((local >> 1) & 1) ^ 1u, abort_flag)) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 256);
            bool ok = true;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + stage * C::kStageBytes);
                const uint32_t sb = sa + C::kHalfBytes;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint64_t ad = A_MN ? make_sdesc_sw128(sa + kk * 2048, 8192, 1024)
                                             : make_sdesc_sw128(sa + kk * 32, 16, 1024);
                    const uint64_t bd = B_MN ? make_sdesc_sw128(sb + kk * 2048, 8192, 1024)
                                             : make_sdesc_sw128(sb + kk * 32, 16, 1024);
                    umma_f16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                }
                umma_commit_pair(&empty_bar[stage], 0x3);
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
            umma_commit_pair(&tfull_bar[acc], 0x3);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------- epilogue (both CTAs)
        const int q = warp & 3;
        int local = 0;
        for (int u = pair; u < units; u += pairs, ++local) {
            const int tile = u % tiles;
            int tm, tn;
            tile_coords(tile, args.tiles_m, args.tiles_n, args.band, tm, tn);
            const int acc = local & 1;
            if (!mbar_wait(&tfull_bar[acc], (local >> 1) & 1, abort_flag)) break;
            tc_fence_after();
            const int m = tm * 256 + 128 * (int)rank + q * 32 + lane;
            const bool mrow = m < args.M;
            if (args.mode == kEpiSwiglu) {
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    uint32_t rg[32], ru[32];
                    __syncwarp();
                    tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 256 + c * 32), rg);
                    tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 256 + 128 + c * 32), ru);
                    tmem_ld_wait();
                    if (!mrow) continue;
                    const int j0 = tn * 128 + c * 32;
                    float g[32], u[32], a[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        g[i] = bf16_round(__uint_as_float(rg[i]) * args.alpha);
                        u[i] = bf16_round(__uint_as_float(ru[i]) * args.alpha);
                        a[i] = sw_silu(g[i]) * u[i];
                    }
                    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(args.out) + (int64_t)m * args.ldo + j0;
                    store32_bf16(op, g);
                    store32_bf16(op + args.half_n, u);
                    store32_bf16(args.out2 + (int64_t)m * args.ldo2 + j0, a);
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < 256 / 32; ++c) {
                    uint32_t r[32];
                    __syncwarp();
                    tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 256 + c * 32), r);
                    tmem_ld_wait();
                    const int n0 = tn * 256 + c * 32;
                    if (!mrow || n0 >= args.N) continue;
                    epilogue32(args, args.mode, m, n0, r);
                }
            }
            tc_fence_before();
            mbar_arrive_cluster(cluster_addr(&tempty_bar[acc], 0));
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while the other may still signal its barriers or use its TMEM
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::kTmemCols);
    }
}

// ------------------------------------------------------------------------------------ host side

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool encode_fn() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode != nullptr;
}

}  // namespace

// A row-major bf16 matrix [outer, inner] (inner contiguous, row stride `ld` elements) as a 2D tensor
// map with a (box_inner, box_outer) box and the 128-byte swizzle. Out-of-range boxes read zeros.
bool make_map(CUtensorMap* map, const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_inner,
              int box_outer) {
    if (!encode_fn()) return false;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || (ld * 2) % 16 != 0) return false;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Operand X of logical shape [rows, K] (rows = M for A, N for B) with its majorness.
bool operand_map(CUtensorMap* map, const R97bMat& m, int64_t rows, int64_t K, int box_rows) {
    if (m.mn_major)  // stored [K, rows]
        return make_map(map, m.ptr, rows, K, m.ld, 64, 64);
    return make_map(map, m.ptr, K, rows, m.ld, 64, box_rows);
}

int num_sms() {
    // per device: a process may drive GPUs of different SM counts
    static std::atomic<int> cache[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

namespace {

// How launch() splits the reduction: k blocks per split and the resulting number of splits.
void split_geometry(const R97bGemm& g, int& kb_per_split, int& splits) {
    const int k_total = (int)((g.K1 + kBK - 1) / kBK) + (g.K2 > 0 ? (int)((g.K2 + kBK - 1) / kBK) : 0);
    int sp = g.splits > 1 ? g.splits : 1;
    if (sp > k_total) sp = k_total;
    kb_per_split = (k_total + sp - 1) / sp;
    splits = (k_total + kb_per_split - 1) / kb_per_split;
}

int pick_bn(const R97bGemm& g) {
    int bn = g.bn;
    if (bn == 0) bn = g.N <= 64 ? 64 : (g.N <= 128 ? 128 : (g.M <= 128 ? 256 : 512));
    if (bn == 512 && g.mode == kEpiSplitBf16) bn = 256;  // the split fix-up runs in the single-SM kernel
    return bn;
}

// The split-K workspace of kEpiSplitBf16: per-tile counters (rounded up to 256 bytes), then the f32
// partial tiles [splits][tiles][kBM][bn]. 0 when the call does not split.
int64_t split_ws_bytes(const R97bGemm& g, int64_t* cnt_bytes) {
    if (g.mode != kEpiSplitBf16) return 0;
    const int bn = pick_bn(g);
    int kbs, splits;
    split_geometry(g, kbs, splits);
    if (splits <= 1) return 0;
    const int64_t tiles = ((g.M + kBM - 1) / kBM) * ((g.N + bn - 1) / bn);
    const int64_t cb = (tiles * 4 + 255) / 256 * 256;
    if (cnt_bytes) *cnt_bytes = cb;
    return cb + (int64_t)splits * tiles * kBM * bn * 4;
}

// M-tiles a band of the tile order walks: 16 unless R97B_GEMM_BAND (1 .. 64) says otherwise, read once.
int tile_band() {
    static const int band = [] {
        const char* e = getenv("R97B_GEMM_BAND");
        const int v = e ? atoi(e) : 0;
        return v >= 1 && v <= 64 ? v : 16;
    }();
    return band;
}

template <int BN, int A_MN, int B_MN>
int launch(const R97bGemm& g, cudaStream_t stream) {
    using C = Cfg<BN>;
    CUtensorMap a1, b1, a2, b2;
    if (!operand_map(&a1, g.a1, g.M, g.K1, kBM)) return R97B_EINVAL;
    if (!operand_map(&b1, g.b1, g.N, g.K1, BN)) return R97B_EINVAL;
    if (g.K2 > 0) {
        if (!operand_map(&a2, g.a2, g.M, g.K2, kBM)) return R97B_EINVAL;
        if (!operand_map(&b2, g.b2, g.N, g.K2, BN)) return R97B_EINVAL;
    } else {
        a2 = a1;
        b2 = b1;
    }
    KernelArgs k{};
    k.M = (int32_t)g.M;
    k.N = (int32_t)g.N;
    k.k1_blocks = (int32_t)((g.K1 + kBK - 1) / kBK);
    k.k2_blocks = g.K2 > 0 ? (int32_t)((g.K2 + kBK - 1) / kBK) : 0;
    int kbs, splits;
    split_geometry(g, kbs, splits);
    k.kb_per_split = kbs;
    k.splits = splits;
    k.tiles_m = (int32_t)((g.M + kBM - 1) / kBM);
    k.tiles_n = (int32_t)((g.N + BN - 1) / BN);
    k.band = tile_band();
    k.mode = g.mode;
    if (g.mode == kEpiSplitBf16) {
        if (splits <= 1) {
            k.mode = kEpiStoreBf16;
        } else {
            int64_t cb = 0;
            const int64_t need = split_ws_bytes(g, &cb);
            if (!g.ws || (reinterpret_cast<uintptr_t>(g.ws) & 255) != 0 || g.ws_bytes < need) return R97B_EINVAL;
            k.ws_cnt = reinterpret_cast<int*>(g.ws);
            k.ws_part = reinterpret_cast<float*>(reinterpret_cast<char*>(g.ws) + cb);
        }
    }
    k.alpha = g.alpha;
    k.beta = g.beta;
    k.out = g.out;
    k.ldo = g.ldo;
    k.addend = reinterpret_cast<const __nv_bfloat16*>(g.addend);
    k.ld_add = g.ld_add;
    k.half_n = (int32_t)g.N;
    const int units = k.tiles_m * k.tiles_n * k.splits;
    int grid = num_sms();
    if (units < grid) grid = units;
    auto kern = gemm_kernel<BN, A_MN, B_MN>;
    if (!smem_opt_in(kern, (int)C::kSmemBytes)) return R97B_ELAUNCH;
    kern<<<grid, kThreads, C::kSmemBytes, stream>>>(a1, b1, a2, b2, k);
    return launch_status();
}

template <int A_MN, int B_MN>
int launch_pair(const R97bGemm& g, cudaStream_t stream) {
    using C = CfgPair;
    CUtensorMap a1, b1, a2, b2;
    if (!operand_map(&a1, g.a1, g.M, g.K1, 128)) return R97B_EINVAL;
    if (!operand_map(&b1, g.b1, g.N, g.K1, 128)) return R97B_EINVAL;
    if (g.K2 > 0) {
        if (!operand_map(&a2, g.a2, g.M, g.K2, 128)) return R97B_EINVAL;
        if (!operand_map(&b2, g.b2, g.N, g.K2, 128)) return R97B_EINVAL;
    } else {
        a2 = a1;
        b2 = b1;
    }
    KernelArgs k{};
    k.M = (int32_t)g.M;
    k.N = (int32_t)g.N;
    k.k1_blocks = (int32_t)((g.K1 + kBK - 1) / kBK);
    k.k2_blocks = g.K2 > 0 ? (int32_t)((g.K2 + kBK - 1) / kBK) : 0;
    int kbs, splits;
    split_geometry(g, kbs, splits);
    k.kb_per_split = kbs;
    k.splits = splits;
    k.tiles_m = (int32_t)((g.M + 255) / 256);
    k.tiles_n = (int32_t)((g.N + 255) / 256);
    k.band = tile_band();
    k.mode = g.mode;
    k.alpha = g.alpha;
    k.beta = g.beta;
    k.out = g.out;
    k.ldo = g.ldo;
    k.addend = reinterpret_cast<const __nv_bfloat16*>(g.addend);
    k.ld_add = g.ld_add;
    k.out2 = reinterpret_cast<__nv_bfloat16*>(g.out2);
    k.ldo2 = g.ldo2;
    k.half_n = (int32_t)(g.mode == kEpiSwiglu ? g.N / 2 : g.N);
    const int units = k.tiles_m * k.tiles_n * k.splits;
    int pairs = num_sms() / 2;
    if (units < pairs) pairs = units;
    auto kern = gemm_pair_kernel<A_MN, B_MN>;
    if (!smem_opt_in(kern, (int)C::kSmemBytes)) return R97B_ELAUNCH;
    kern<<<2 * pairs, kThreads, C::kSmemBytes, stream>>>(a1, b1, a2, b2, k);
    return launch_status();
}

template <int BN>
int dispatch_major(const R97bGemm& g, cudaStream_t s) {
    const int a = g.a1.mn_major ? 1 : 0, b = g.b1.mn_major ? 1 : 0;
    if (a == 0 && b == 0) return launch<BN, 0, 0>(g, s);
    if (a == 0 && b == 1) return launch<BN, 0, 1>(g, s);
    if (a == 1 && b == 0) return launch<BN, 1, 0>(g, s);
    return launch<BN, 1, 1>(g, s);
}

}  // namespace

R97B_ERROR_READER(gemm_error_word)

int64_t gemm_workspace_bytes(const R97bGemm& g) {
    if (g.M <= 0 || g.N <= 0 || g.K1 <= 0 || g.mode < kEpiStoreBf16 || g.mode > kEpiSwigluBwd) return -1;
    const int bn = pick_bn(g);
    if (bn != 64 && bn != 128 && bn != 256 && bn != 512) return -1;
    return split_ws_bytes(g, nullptr);
}

int gemm_run(const R97bGemm& g, cudaStream_t stream) {
    if (g.M <= 0 || g.N <= 0 || g.K1 <= 0 || !g.out || !g.a1.ptr || !g.b1.ptr) return R97B_EINVAL;
    if (g.K2 > 0 && (!g.a2.ptr || !g.b2.ptr || g.a2.mn_major != g.a1.mn_major || g.b2.mn_major != g.b1.mn_major))
        return R97B_EINVAL;
    if (g.mode < kEpiStoreBf16 || g.mode > kEpiSwigluBwd) return R97B_EINVAL;
    if (g.M > 0x7FFFFFFF || g.N > 0x7FFFFFFF) return R97B_EINVAL;
    if (g.mode == kEpiSwiglu) {  // the CTA pair only: its two halves of B are the gate and the up rows
        const int64_t F = g.N / 2;
        if (g.N % 256 != 0 || !g.out2 || g.ldo % 8 || g.ldo2 % 8 || g.ldo < g.N || g.ldo2 < F || g.addend ||
            g.splits > 1 || (reinterpret_cast<uintptr_t>(g.out) & 15) || (reinterpret_cast<uintptr_t>(g.out2) & 15))
            return R97B_EINVAL;
        const int a = g.a1.mn_major ? 1 : 0, b = g.b1.mn_major ? 1 : 0;
        if (a == 0 && b == 0) return launch_pair<0, 0>(g, stream);
        if (a == 0 && b == 1) return launch_pair<0, 1>(g, stream);
        if (a == 1 && b == 0) return launch_pair<1, 0>(g, stream);
        return launch_pair<1, 1>(g, stream);
    }
    if (g.mode == kEpiSwigluBwd && (!g.addend || g.ld_add < 2 * g.N || g.splits > 1)) return R97B_EINVAL;
    const int bn = pick_bn(g);
    if (bn == 512) {  // the CTA-pair kernel: 256 x 256 tiles over two SMs
        const int a = g.a1.mn_major ? 1 : 0, b = g.b1.mn_major ? 1 : 0;
        if (a == 0 && b == 0) return launch_pair<0, 0>(g, stream);
        if (a == 0 && b == 1) return launch_pair<0, 1>(g, stream);
        if (a == 1 && b == 0) return launch_pair<1, 0>(g, stream);
        return launch_pair<1, 1>(g, stream);
    }
    switch (bn) {
        case 64: return dispatch_major<64>(g, stream);
        case 128: return dispatch_major<128>(g, stream);
        case 256: return dispatch_major<256>(g, stream);
        default: return R97B_EINVAL;
    }
}

}  // namespace r97b
