// qlinear.cu -- one LoRA-adapted linear over a stored (IQR) weight, forward and backward, as single C calls:
// the reference's gemm_nt_q + lora_shrink + lora_expand rows for one adapter slot (reference
// src/adjoint/host/linear.cpp:246-317, lora.cpp:226-523; device src/adjoint/device/linear.hip, lora.hip),
// composed from this library's entry points:
//
//   forward   W = decode(w) (unless the caller's buffer already holds it), t = s x A^T,
//             y = x W^T + t B^T (+ addend)                        -- the tail rides in y's tile loop
//   backward  dt = s dy B, dx = dy W + dt A, dA += dt^T x, dB += dy^T t
//
// The narrow products (t, dt: `rank` columns) run on the split tilings the step uses; the adapter
// gradients accumulate in f32.
#include "r97b_internal.h"

namespace {

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// (bn, splits) of a narrow bf16 product with `n` output columns over a reduction of k (the step's rule).
void narrow_tiling(int64_t m, int64_t n, int64_t k, int* bn, int* splits) {
    *bn = n <= 64 ? 64 : 128;
    const int64_t units = cdiv(m, 128) * cdiv(n, *bn);
    *splits = (units < 100 && (n <= 64 || k >= 8192)) ? 2 : 1;
}

// (bn, splits) of an adapter-gradient product (f32 atomics, reduction over k tokens): the split count s
// (at most 8, and k / s >= 1024) that minimises ceil(tiles s / SMs) / s, the waves of work a tile's share
// takes, ties to the fewer splits.
void grad_tiling(int64_t m, int64_t n, int64_t k, int* bn, int* splits) {
    *bn = n >= 128 ? 128 : 64;
    const int64_t tiles = cdiv(m, 128) * cdiv(n, *bn);
    const int64_t sms = r97b::num_sms();
    const int smax = (int)std::max<int64_t>(1, std::min<int64_t>(8, k / 1024));
    int best = 1;
    for (int s = 2; s <= smax; ++s)
        if (cdiv(tiles * s, sms) * best < cdiv(tiles * best, sms) * s) best = s;
    *splits = best;
}

R97bMat mat(const void* p, int64_t ld, int mn) {
    R97bMat m{};
    m.ptr = p;
    m.ld = ld;
    m.mn_major = mn;
    return m;
}

// The narrow product out[M, r] = alpha * a[M, K] b^T with b K-major [r, K] (b_mn 0) or stored [K, r] (b_mn 1).
R97bGemm narrow(int64_t M, int64_t r, int64_t K, const void* a, const void* b, int b_mn, void* out, float alpha,
                void* ws, int64_t ws_bytes) {
    R97bGemm g{};
    g.M = M;
    g.N = r;
    g.K1 = K;
    g.a1 = mat(a, K, 0);
    g.b1 = mat(b, b_mn ? r : K, b_mn);
    int bn, sp;
    narrow_tiling(M, r, K, &bn, &sp);
    g.bn = bn;
    g.splits = sp;
    g.mode = sp > 1 ? R97B_EPI_SPLIT_BF16 : R97B_EPI_STORE_BF16;
    g.alpha = alpha;
    g.beta = 1.0f;
    g.out = out;
    g.ldo = r;
    g.ws = ws;
    g.ws_bytes = ws_bytes;
    return g;
}

bool shapes_ok(int64_t M, int64_t N, int64_t K, int32_t rank) {
    return M > 0 && N > 0 && K > 0 && rank > 0 && K % 8 == 0 && N % 8 == 0 && rank % 8 == 0;
}

}  // namespace

extern "C" int64_t r97b_qlinear_lora_workspace_bytes(int64_t M, int64_t N, int64_t K, int32_t rank) {
    if (!shapes_ok(M, N, K, rank)) return -1;
    const R97bGemm f = narrow(M, rank, K, nullptr, nullptr, 0, nullptr, 1.0f, nullptr, 0);
    const R97bGemm b = narrow(M, rank, N, nullptr, nullptr, 1, nullptr, 1.0f, nullptr, 0);
    const int64_t x = r97b::gemm_workspace_bytes(f), y = r97b::gemm_workspace_bytes(b);
    if (x < 0 || y < 0) return -1;
    return x > y ? x : y;
}

extern "C" int r97b_qlinear_lora_fwd(const R97bQLinearLora* a, void* stream) {
    if (!a || !shapes_ok(a->M, a->N, a->K, a->rank) || !a->w_bf16 || !a->x || !a->A || !a->B || !a->t || !a->y)
        return R97B_EINVAL;
    if (!a->w_decoded) {
        if (!a->w || a->w->rows != a->N || a->w->cols != a->K) return R97B_EINVAL;
        int rc = r97b_iqr_dequant_bf16(a->w, static_cast<uint16_t*>(a->w_bf16), a->K, stream);
        if (rc != R97B_OK) return rc;
    }
    cudaStream_t st = r97b::as_stream(stream);
    R97bGemm g = narrow(a->M, a->rank, a->K, a->x, a->A, 0, a->t, a->scale, a->ws, a->ws_bytes);
    int rc = r97b::gemm_run(g, st);
    if (rc != R97B_OK) return rc;
    R97bGemm y{};
    y.M = a->M;
    y.N = a->N;
    y.K1 = a->K;
    y.K2 = a->rank;
    y.a1 = mat(a->x, a->K, 0);
    y.b1 = mat(a->w_bf16, a->K, 0);
    y.a2 = mat(a->t, a->rank, 0);
    y.b2 = mat(a->B, a->rank, 0);
    y.mode = R97B_EPI_STORE_BF16;
    y.alpha = 1.0f;
    y.beta = 1.0f;
    y.out = a->y;
    y.ldo = a->N;
    y.addend = a->addend;
    y.ld_add = a->N;
    return r97b::gemm_run(y, st);
}

extern "C" int r97b_qlinear_lora_bwd(const R97bQLinearLoraBwd* a, void* stream) {
    if (!a || !shapes_ok(a->M, a->N, a->K, a->rank) || !a->w_bf16 || !a->x || !a->A || !a->B || !a->t || !a->dy ||
        !a->dt || !a->dx || !a->dA || !a->dB)
        return R97B_EINVAL;
    cudaStream_t st = r97b::as_stream(stream);
    // dt = s dy B  (B stored [N, r]: the narrow product's operand read MN-major)
    R97bGemm g = narrow(a->M, a->rank, a->N, a->dy, a->B, 1, a->dt, a->scale, a->ws, a->ws_bytes);
    int rc = r97b::gemm_run(g, st);
    if (rc != R97B_OK) return rc;
    // dx = dy W + dt A  (W stored [N, K], A stored [r, K]: both MN-major)
    R97bGemm x{};
    x.M = a->M;
    x.N = a->K;
    x.K1 = a->N;
    x.K2 = a->rank;
    x.a1 = mat(a->dy, a->N, 0);
    x.b1 = mat(a->w_bf16, a->K, 1);
    x.a2 = mat(a->dt, a->rank, 0);
    x.b2 = mat(a->A, a->K, 1);
    x.mode = R97B_EPI_STORE_BF16;
    x.alpha = 1.0f;
    x.beta = 1.0f;
    x.out = a->dx;
    x.ldo = a->K;
    if ((rc = r97b::gemm_run(x, st)) != R97B_OK) return rc;
    // dA [r, K] += dt^T x : reduction over the tokens, the output stored transposed
    int bn, sp;
    R97bGemm da{};
    da.M = a->K;
    da.N = a->rank;
    da.K1 = a->M;
    da.a1 = mat(a->x, a->K, 1);
    da.b1 = mat(a->dt, a->rank, 1);
    grad_tiling(a->K, a->rank, a->M, &bn, &sp);
    da.bn = bn;
    da.splits = sp;
    da.mode = R97B_EPI_ATOMIC_F32T;
    da.alpha = 1.0f;
    da.out = a->dA;
    da.ldo = a->K;
    if ((rc = r97b::gemm_run(da, st)) != R97B_OK) return rc;
    // dB [N, r] += dy^T t
    R97bGemm db{};
    db.M = a->N;
    db.N = a->rank;
    db.K1 = a->M;
    db.a1 = mat(a->dy, a->N, 1);
    db.b1 = mat(a->t, a->rank, 1);
    grad_tiling(a->N, a->rank, a->M, &bn, &sp);
    db.bn = bn;
    db.splits = sp;
    db.mode = R97B_EPI_ATOMIC_F32;
    db.alpha = 1.0f;
    db.out = a->dB;
    db.ldo = a->rank;
    return r97b::gemm_run(db, st);
}
