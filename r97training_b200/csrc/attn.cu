// attn.cu -- the backward of causal grouped-query attention on sm_100a tensor cores (tcgen05 + TMA + TMEM).
//
// The attention core of the hybrid model's gated-attention blocks (reference: attention_host_adjoint,
// src/adjoint/host/attention.cpp:261-414, whose arithmetic is the standard softmax adjoint) given the
// forward's output O and its per-row log-sum-exp:
//
//   P  = exp(scale q k^T - lse)                 (causal: key <= query)
//   dV = P^T dO                                 (summed over the query heads that share a key/value head)
//   dS = scale P o (dO V^T - Delta),  Delta = rowsum(dO o O)
//   dK = dS^T Q,   dQ = dS K
//
// as passes of one persistent, warp-specialised kernel template (warp 0 TMA loads into a ring of
// shared-memory stages, warp 1 issues tcgen05.mma into a double-buffered TMEM accumulator, and EPW warps
// per TMEM lane quarter (warps 4 ...) drain it with tcgen05.ld, each a slice of the columns, and run the
// pass's epilogue -- 4 per quarter for the exp / product epilogues of the 128 x 128 tiles):
//
//   kPDS  128 x 128 causal tiles of S = Q K^T and dP = dO V^T (k = head dim) into two accumulators, epilogue
//         P = exp2(S scale log2e - lse log2e) and dS = scale P (dP - Delta), both stored bf16
//   kDKV  128 keys x D tiles of dV = P^T dO (or dK = dS^T Q): P / dS and dO / Q read MN-major, the
//         reduction running over the group's query heads and the query blocks at or after the key block
//   kDQ   128 queries x D tiles of dQ = dS K: dS K-major, K MN-major, key blocks up to the query block
//
// P and dS live in a caller-provided workspace ([B*Hq*S, S] bf16 each; only the causal tiles are written
// and read). Tiles of kDKV and kDQ carry unequal work (the causal triangle), so they are handed out
// longest-first in a snake order across the CTAs. No cluster multicast anywhere.
#include "sm100.cuh"
#include "r97b_internal.h"
#include "fastmath.cuh"

#include <cuda_bf16.h>

namespace r97b {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kABytes = kBM * kBK * 2;  // 16 KiB
constexpr float kLog2e = 1.4426950408889634f;

enum Kind { kPDS = 0, kDKV = 1, kDQ = 2 };

struct AttnArgs {
    int32_t B, Hq, Hkv, S, D, grp, nblk;
    int32_t units;
    float scale;
    const float* lse;            // [B*Hq*S] natural-log log-sum-exp of each query row (scaled scores)
    const float* delta;          // [B*Hq*S] rowsum(dO o O)
    __nv_bfloat16* out;          // kPDS (P): [B*Hq*S, S]; kDKV: [B*Hkv*S, D]; kDQ: [B*Hq*S, D]
    __nv_bfloat16* out2;         // kPDS: dS [B*Hq*S, S]
};

template <int BN, int NACC = 1>
struct ACfg {
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    // kPDS (two accumulators): a 4 KB staging slot per epilogue warp for its P and dS rows (32 rows of 64 B
    // each, pitch 80 B), so the tiles leave as coalesced rows; that space comes out of the ring
    static constexpr int kStageOut = NACC == 2 ? 16 * 32 * 80 * 2 : 0;
    static constexpr int kRing = NACC == 2 ? 224 * 1024 - kStageOut : 200 * 1024;
    static constexpr int kStages = kRing / kStageBytes > 8 ? 8 : kRing / kStageBytes;
    static constexpr int kAccCols = NACC * BN;  // one tile's accumulators (kPDS: S and dP side by side)
    static constexpr int kTmemCols = 2 * kAccCols;
    static constexpr int kSmemBytes = kStages * kStageBytes + kStageOut + 1024 + 256;
};

// Unit `t`-th of CTA `c` (of G) in the pass's order: round-robin for the equal tiles of kPDS, a snake
// over the longest-first order for kDKV / kDQ (a CTA's heavy unit of one round meets a light one in the next).
template <int KIND>
__device__ __forceinline__ int unit_of(int t, int c, int G) {
    if (KIND == kPDS) return t * G + c;
    return t * G + ((t & 1) ? (G - 1 - c) : c);
}

// (bh, i, j) of a causal tile: T = nblk (nblk + 1) / 2 tiles per head, j <= i.
__device__ __forceinline__ void tri_tile(int u, int nblk, int& bh, int& i, int& j) {
    const int T = nblk * (nblk + 1) / 2;
    bh = u / T;
    const int t = u - bh * T;
    int ii = (int)((sqrtf(8.0f * (float)t + 1.0f) - 1.0f) * 0.5f);
    while (ii * (ii + 1) / 2 > t) --ii;
    while ((ii + 1) * (ii + 2) / 2 <= t) ++ii;
    i = ii;
    j = t - ii * (ii + 1) / 2;
}

// The unit's output tile and its number of 64-deep k blocks.
//   kPDS: (bh, i, j)          kDKV: (bg = b * Hkv + g, j = key block)          kDQ: (bh, i = query block)
template <int KIND>
__device__ __forceinline__ void unit_geom(const AttnArgs& a, int u, int& x0, int& x1, int& x2, int& nk) {
    if (KIND == kPDS) {  // S's k blocks, then dP's
        tri_tile(u, a.nblk, x0, x1, x2);
        nk = 2 * (a.D / kBK);
    } else if (KIND == kDKV) {
        const int groups = a.B * a.Hkv;
        x1 = u / groups;  // key block, ascending = longest first
        x0 = u - x1 * groups;
        x2 = 0;
        nk = a.grp * (a.nblk - x1) * 2;
    } else {
        const int heads = a.B * a.Hq;
        const int r = u / heads;
        x0 = u - r * heads;
        x1 = a.nblk - 1 - r;  // query block, descending = longest first
        x2 = 0;
        nk = (x1 + 1) * 2;
    }
}

template <int KIND, int BN, int EPW>
__global__ void __launch_bounds__(128 + 128 * EPW, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tB,
                    const __grid_constant__ CUtensorMap tA2, const __grid_constant__ CUtensorMap tB2,
                    const AttnArgs args) {
    using C = ACfg<BN, KIND == kPDS ? 2 : 1>;
    constexpr int A_MN = KIND == kDKV ? 1 : 0;
    constexpr int B_MN = (KIND == kDKV || KIND == kDQ) ? 1 : 0;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (base_u32 & 1023u)) & 1023u);
    uint8_t* stage_out = smem + C::kStages * C::kStageBytes;  // kPDS: the epilogue warps' staging slots
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(stage_out + C::kStageOut);
    uint64_t* empty_bar = full_bar + C::kStages;
    uint64_t* tfull_bar = empty_bar + C::kStages;
    uint64_t* tempty_bar = tfull_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull_bar[b], 1);
            mbar_init(&tempty_bar[b], 128 * EPW);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch(&tA);
        tma_prefetch(&tB);
        if (KIND == kPDS) {
            tma_prefetch(&tA2);
            tma_prefetch(&tB2);
        }
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
        for (int t = 0; ok; ++t) {
            const int u = unit_of<KIND>(t, c, G);
            if (u >= args.units) {
                if (t * G >= args.units) break;
                continue;
            }
            int x0, x1, x2, nk;
            unit_geom<KIND>(args, u, x0, x1, x2, nk);
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                uint8_t* sa = smem + stage * C::kStageBytes;
                uint8_t* sb = sa + kABytes;
                mbar_expect_tx(&full_bar[stage], C::kStageBytes);
                if (KIND == kPDS) {
                    const int bh = x0, b = bh / args.Hq, h = bh - b * args.Hq;
                    const int qrow = bh * args.S + x1 * kBM;
                    const int krow = (b * args.Hkv + h / args.grp) * args.S + x2 * kBM;
                    const int nd = args.D / kBK;
                    const bool second = kb >= nd;  // dO, V after Q, K
                    const int kc = (second ? kb - nd : kb) * kBK;
                    tma_load_2d(sa, second ? &tA2 : &tA, &full_bar[stage], kc, qrow);
                    tma_load_2d(sb, second ? &tB2 : &tB, &full_bar[stage], kc, krow);
                } else if (KIND == kDKV) {
                    const int bg = x0, b = bg / args.Hkv, g = bg - b * args.Hkv, j = x1;
                    const int per_head = (args.nblk - j) * 2;
                    const int hh = kb / per_head, rem = kb - hh * per_head;
                    const int qrow = (b * args.Hq + g * args.grp + hh) * args.S + (j + (rem >> 1)) * kBM + (rem & 1) * kBK;
                    tma_load_2d(sa, &tA, &full_bar[stage], j * kBM, qrow);
                    tma_load_2d(sa + 8192, &tA, &full_bar[stage], j * kBM + 64, qrow);
#pragma unroll
                    for (int jj = 0; jj < BN / 64; ++jj) tma_load_2d(sb + jj * 8192, &tB, &full_bar[stage], 64 * jj, qrow);
                } else {
                    const int bh = x0, b = bh / args.Hq, h = bh - b * args.Hq;
                    const int qrow = bh * args.S + x1 * kBM;
                    const int kcol = kb * kBK;  // key position inside the head
                    const int krow = (b * args.Hkv + h / args.grp) * args.S + kcol;
                    tma_load_2d(sa, &tA, &full_bar[stage], kcol, qrow);
#pragma unroll
                    for (int jj = 0; jj < BN / 64; ++jj) tma_load_2d(sb + jj * 8192, &tB, &full_bar[stage], 64 * jj, krow);
                }
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------- MMA issuer
        constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, A_MN, B_MN);
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool ok = true;
        for (int t = 0; ok; ++t) {
            const int u = unit_of<KIND>(t, c, G);
            if (u >= args.units) {
                if (t * G >= args.units) break;
                continue;
            }
            int x0, x1, x2, nk;
            unit_geom<KIND>(args, u, x0, x1, x2, nk);
            const int acc = local & 1;
            if (!mbar_wait(&tempty_bar[acc], ((local >> 1) & 1) ^ 1u, abort_flag)) break;
            tc_fence_after();
            const uint32_t d_base = tmem_base + (uint32_t)(acc * C::kAccCols);
            const int nd = args.D / kBK;
            for (int kb = 0; kb < nk; ++kb) {
                if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + stage * C::kStageBytes);
                const uint32_t sb = sa + kABytes;
                // kPDS: S accumulates over the first nd k blocks, dP (BN columns further) over the next nd
                const bool second = KIND == kPDS && kb >= nd;
                const uint32_t d_tmem = d_base + (second ? (uint32_t)BN : 0u);
                const int kb0 = second ? nd : 0;
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
            ++local;
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------- epilogue
        const int q = warp & 3;           // the TMEM lane quarter this warp may read
        const int sub = (warp - 4) >> 2;  // its slice of the columns
        constexpr int kChunks = BN / 32 / EPW;
        const int c0 = sub * kChunks;
        const int row = q * 32 + lane;  // this thread's accumulator row
        int local = 0;
        for (int t = 0;; ++t) {
            const int u = unit_of<KIND>(t, c, G);
            if (u >= args.units) {
                if (t * G >= args.units) break;
                continue;
            }
            int x0, x1, x2, nk;
            unit_geom<KIND>(args, u, x0, x1, x2, nk);
            const int acc = local & 1;
            if (!mbar_wait(&tfull_bar[acc], (local >> 1) & 1, abort_flag)) break;
            tc_fence_after();
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * C::kAccCols);
            if (KIND == kPDS) {
                // P = exp2(S scale log2e - lse log2e) (causal), dS = scale P (dP - Delta); both stored
                const int bh = x0, i = x1, j = x2;
                const int qpos = i * kBM + row;
                const int64_t grow = (int64_t)bh * args.S + qpos;
                const float lse2 = args.lse[grow] * kLog2e;
                const float dlt = args.delta[grow];
                const float sl2 = args.scale * kLog2e;
                // this warp's staging slot: its 32 rows' 32 values of P, then of dS, as bf16 rows of 64 B at an
                // 80-byte pitch (a quarter-warp's 16-byte accesses then fall in distinct banks)
                uint8_t* slot = stage_out + (warp - 4) * (32 * 80 * 2);
                const int64_t grow0 = (int64_t)bh * args.S + i * kBM + q * 32;  // the warp's first row
#pragma unroll 1
                for (int cc = c0; cc < c0 + kChunks; ++cc) {
                    uint32_t rs[32], rd[32];
                    __syncwarp();
                    tmem_ld32(tbase + (uint32_t)(cc * 32), rs);
                    tmem_ld32(tbase + (uint32_t)(BN + cc * 32), rd);
                    tmem_ld_wait();
                    float pv[32], dv[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const int kpos = j * kBM + cc * 32 + e;
                        const float pe = kpos <= qpos ? ex2_ftz(__uint_as_float(rs[e]) * sl2 - lse2) : 0.0f;
                        // dS is formed from P as stored (bf16), the P that dV reads
                        const float pb = __bfloat162float(__float2bfloat16_rn(pe));
                        pv[e] = pe;
                        dv[e] = args.scale * pb * (__uint_as_float(rd[e]) - dlt);
                    }
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        uint32_t pk[4], dk[4];
#pragma unroll
                        for (int h2 = 0; h2 < 4; ++h2) {
                            const __nv_bfloat162 b2 = __floats2bfloat162_rn(pv[w * 8 + h2 * 2], pv[w * 8 + h2 * 2 + 1]);
                            const __nv_bfloat162 d2 = __floats2bfloat162_rn(dv[w * 8 + h2 * 2], dv[w * 8 + h2 * 2 + 1]);
                            pk[h2] = *reinterpret_cast<const uint32_t*>(&b2);
                            dk[h2] = *reinterpret_cast<const uint32_t*>(&d2);
                        }
                        *reinterpret_cast<uint4*>(slot + lane * 80 + w * 16) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                        *reinterpret_cast<uint4*>(slot + 32 * 80 + lane * 80 + w * 16) = make_uint4(dk[0], dk[1], dk[2], dk[3]);
                    }
                    __syncwarp();
                    // out: four lanes a row (64 contiguous bytes), eight rows a store
#pragma unroll
                    for (int s8 = 0; s8 < 4; ++s8) {
                        const int r = s8 * 8 + (lane >> 2), part = lane & 3;
                        const uint4 vp = *reinterpret_cast<const uint4*>(slot + r * 80 + part * 16);
                        const uint4 vd = *reinterpret_cast<const uint4*>(slot + 32 * 80 + r * 80 + part * 16);
                        const int64_t at = (grow0 + r) * args.S + j * kBM + cc * 32 + part * 8;
                        *reinterpret_cast<uint4*>(args.out + at) = vp;
                        *reinterpret_cast<uint4*>(args.out2 + at) = vd;
                    }
                }
            } else {
                const int64_t orow = (int64_t)x0 * args.S + x1 * kBM + row;
                __nv_bfloat16* op = args.out + orow * args.D;
#pragma unroll 1
                for (int cc = c0; cc < c0 + kChunks; ++cc) {
                    uint32_t r[32];
                    __syncwarp();
                    tmem_ld32(tbase + (uint32_t)(cc * 32), r);
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
            }
            tc_fence_before();
            mbar_arrive(&tempty_bar[acc]);
            ++local;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

// Delta[row] = sum_d dO[row, d] O[row, d] (f32), one warp per row.
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ o,
                                  float* __restrict__ delta, int64_t rows, int D) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    float s = 0.0f;
    for (int d0 = lane * 8; d0 < D; d0 += 256) {
        const uint4 a = *reinterpret_cast<const uint4*>(dout + r * D + d0);
        const uint4 b = *reinterpret_cast<const uint4*>(o + r * D + d0);
        const uint32_t xa[4] = {a.x, a.y, a.z, a.w}, xb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 pa = *reinterpret_cast<const __nv_bfloat162*>(&xa[k]);
            const __nv_bfloat162 pb = *reinterpret_cast<const __nv_bfloat162*>(&xb[k]);
            s = fmaf(__bfloat162float(pa.x), __bfloat162float(pb.x), s);
            s = fmaf(__bfloat162float(pa.y), __bfloat162float(pb.y), s);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) delta[r] = s;
}

template <int KIND, int BN>
int launch_pass(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& a2, const CUtensorMap& b2,
                const AttnArgs& args, cudaStream_t stream) {
    using C = ACfg<BN, KIND == kPDS ? 2 : 1>;
    constexpr int EPW = KIND == kPDS ? 4 : 2;
    static_assert((BN / 32) % EPW == 0, "column slices");
    auto kern = attn_bwd_kernel<KIND, BN, EPW>;
    if (!smem_opt_in(kern, (int)C::kSmemBytes)) return R97B_ELAUNCH;
    int grid = num_sms();
    if (args.units < grid) grid = args.units;
    kern<<<grid, 128 + 128 * EPW, C::kSmemBytes, stream>>>(a, b, a2, b2, args);
    return launch_status();
}

int64_t ws_bytes(int64_t B, int64_t Hq, int64_t S) {
    const int64_t pbytes = B * Hq * S * S * 2;
    return 2 * pbytes + B * Hq * S * 4;
}

}  // namespace

R97B_ERROR_READER(attn_error_word)

}  // namespace r97b

extern "C" int64_t r97b_attn_bwd_workspace_bytes(int32_t B, int32_t Hq, int32_t S) {
    if (B <= 0 || Hq <= 0 || S <= 0) return -1;
    return r97b::ws_bytes(B, Hq, S);
}

extern "C" int r97b_attn_bwd(const R97bAttnBwd* a, void* stream) {
    using namespace r97b;
    if (!a) return R97B_EINVAL;
    const int B = a->B, Hq = a->Hq, Hkv = a->Hkv, S = a->S, D = a->D;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || S <= 0 || S % 128 != 0 || (D != 128 && D != 256))
        return R97B_EINVAL;
    if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->dq || !a->dk || !a->dv || !a->ws)
        return R97B_EINVAL;
    if ((int64_t)B * Hq * S > 0x7FFFFFFF / 2 || a->ws_bytes < ws_bytes(B, Hq, S)) return R97B_EINVAL;
    if ((reinterpret_cast<uintptr_t>(a->ws) & 255) != 0) return R97B_EINVAL;
    cudaStream_t st = as_stream(stream);
    const int64_t rq = (int64_t)B * Hq * S, rk = (int64_t)B * Hkv * S;
    __nv_bfloat16* P = reinterpret_cast<__nv_bfloat16*>(a->ws);
    __nv_bfloat16* dS = P + rq * S;
    float* delta = reinterpret_cast<float*>(dS + rq * S);

    CUtensorMap mQ, mK, mV, mdO, mP_k, mdS_k, mP_mn, mdS_mn, mQ_mn, mdO_mn, mK_mn;
    bool ok = make_map(&mQ, a->q, D, rq, D, 64, 128) && make_map(&mK, a->k, D, rk, D, 64, 128) &&
              make_map(&mV, a->v, D, rk, D, 64, 128) && make_map(&mdO, a->dout, D, rq, D, 64, 128) &&
              make_map(&mdS_k, dS, S, rq, S, 64, 128) && make_map(&mP_mn, P, S, rq, S, 64, 64) &&
              make_map(&mdS_mn, dS, S, rq, S, 64, 64) && make_map(&mQ_mn, a->q, D, rq, D, 64, 64) &&
              make_map(&mdO_mn, a->dout, D, rq, D, 64, 64) && make_map(&mK_mn, a->k, D, rk, D, 64, 64);
    (void)mP_k;
    if (!ok) return R97B_EINVAL;

    AttnArgs args{};
    args.B = B;
    args.Hq = Hq;
    args.Hkv = Hkv;
    args.S = S;
    args.D = D;
    args.grp = Hq / Hkv;
    args.nblk = S / 128;
    args.scale = a->scale;
    args.lse = a->lse;
    args.delta = delta;
    int rc;
    {
        const int rows_per_block = 8;
        attn_delta_kernel<<<(unsigned)((rq + rows_per_block - 1) / rows_per_block), 32 * rows_per_block, 0, st>>>(
            reinterpret_cast<const __nv_bfloat16*>(a->dout), reinterpret_cast<const __nv_bfloat16*>(a->o), delta,
            rq, D);
        if ((rc = launch_status()) != R97B_OK) return rc;
    }
    const int tri = args.nblk * (args.nblk + 1) / 2;
    // P and dS tiles in one pass (S = Q K^T and dP = dO V^T into two accumulators)
    args.units = B * Hq * tri;
    args.out = P;
    args.out2 = dS;
    if ((rc = launch_pass<kPDS, 128>(mQ, mK, mdO, mV, args, st)) != R97B_OK) return rc;
    // dV = P^T dO
    args.units = B * Hkv * args.nblk;
    args.out = reinterpret_cast<__nv_bfloat16*>(a->dv);
    rc = D == 256 ? launch_pass<kDKV, 256>(mP_mn, mdO_mn, mP_mn, mdO_mn, args, st)
                  : launch_pass<kDKV, 128>(mP_mn, mdO_mn, mP_mn, mdO_mn, args, st);
    if (rc != R97B_OK) return rc;
    // dK = dS^T Q
    args.out = reinterpret_cast<__nv_bfloat16*>(a->dk);
    rc = D == 256 ? launch_pass<kDKV, 256>(mdS_mn, mQ_mn, mdS_mn, mQ_mn, args, st)
                  : launch_pass<kDKV, 128>(mdS_mn, mQ_mn, mdS_mn, mQ_mn, args, st);
    if (rc != R97B_OK) return rc;
    // dQ = dS K
    args.units = B * Hq * args.nblk;
    args.out = reinterpret_cast<__nv_bfloat16*>(a->dq);
    rc = D == 256 ? launch_pass<kDQ, 256>(mdS_k, mK_mn, mdS_k, mK_mn, args, st)
                  : launch_pass<kDQ, 128>(mdS_k, mK_mn, mdS_k, mK_mn, args, st);
    return rc;
}
