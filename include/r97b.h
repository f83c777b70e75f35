/* include/r97b.h -- the C ABI of libr97b200.so, the B200 (sm_100a) kernels of the LoRA-over-IQR
 * training path.
 *
 * Conventions shared by every entry point:
 *   - pointers are DEVICE pointers unless a comment says otherwise; sizes are element counts;
 *   - `stream` is a cudaStream_t passed as void* (null = the legacy default stream);
 *   - every call is asynchronous on `stream` and returns an int status (R97B_OK or an error code);
 *   - bf16 tensors are passed as uint16_t* (raw bits), f32 as float*, row-major, dense unless a
 *     leading dimension says otherwise.
 * No torch, CUDA-runtime or C++ types cross this boundary.
 *
 * Each declaration names the reference interface it replaces (file:line in the reference tree).
 */
#ifndef R97B_H
#define R97B_H

#include <stdint.h>

#include "r97b_iqr.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
    R97B_OK = 0,
    R97B_EINVAL = 1,   /* arguments outside the kernel's rules (same meaning as the reference's 1) */
    R97B_ELAUNCH = 2,  /* a launch failed */
    R97B_EDEVICE = 3,  /* a device-side check fired (see r97b_device_error) */
    R97B_ETOOLARGE = 4, /* the input exceeds the fixed capacity of an allocation-free entry point */
};

/* ------------------------------------------------------------------------------ library */

/* The library's ABI version (bumped on any signature change). */
int r97b_abi_version(void);

/* The device error word the kernels set (bit 0: a bounded wait expired; bit 1: a kernel rejected its
 * arguments) -- read and cleared. Synchronises the current device. */
int r97b_device_error(unsigned int* out_bits);

/* The CUDA runtime error (a cudaError_t value) behind the most recent R97B_ELAUNCH of any entry point, read
 * and cleared (0 when none since the last read), and the runtime's name for such a value. */
int r97b_last_launch_error(void);
const char* r97b_launch_error_name(int code);

/* ------------------------------------------------------------------------------ plumbing */
/* Device memory and streams for a C++ host that drives the kernels (the adjoint-row plugin,
 * libr97host.so), so that it needs no CUDA headers of its own. Replace: the reference's rad_dev_alloc /
 * rad_dev_free / rad_memcpy / rad_stream_create device layer as its device rows use it
 * (src/adjoint/device/scratch.cpp, linear.hip:423-430). */

/* Device allocation (cudaMalloc: 256-byte aligned); bytes == 0 gives null and R97B_OK. */
int r97b_mem_alloc(void** out, int64_t bytes);
int r97b_mem_free(void* p);
/* Asynchronous copy on `stream`: kind 0 host->device, 1 device->host, 2 device->device. */
int r97b_memcpy(void* dst, const void* src, int64_t bytes, int32_t kind, void* stream);
int r97b_memset(void* dst, int32_t byte, int64_t bytes, void* stream);
/* A non-blocking stream on the current device, and a wait for everything queued on one. */
int r97b_stream_create(void** out);
int r97b_stream_sync(void* stream);
/* The CUDA runtime's text for the last error (not cleared). */
const char* r97b_last_cuda_error(void);

/* ------------------------------------------------------------------------------ IQR decode */

/* Reference-compatible decode: stored trellis/affine IQR codes -> int8 grid [rows, cols] plus bf16 scale
 * bits [rows, cols/128], asynchronously on `stream`. Returns 0, or 1 when the description is outside
 * the decode's rules (r97_iqr_validate) or `stream` cannot be launched on. All plane pointers and
 * outputs are device pointers.
 * Replaces: reference src/iqr_decode.h:378-386 (extern "C" int r97_iqr_decode) and its HIP kernel
 * src/adjoint/device/iqr_decode.hip:32-56. */
int r97_iqr_decode(const R97IqrDecodeDesc* desc, R97IqrStream stream);

/* The GEMM operand form of the same decode: W[r, k] = bf16(code[r, k] * scale[r, k/128]) written as
 * bf16 bits into `out_w` (row stride `ld_w` elements), for rows [row0, row0 + rows). The desc's
 * out_codes / out_scale are ignored. One extra bf16 rounding of the product against the int8+scale
 * pair the reference's kernels read (reference src/adjoint/host/linear.cpp:132-163 value_at).
 * Replaces: the decode half of the reference's stored-weight dX path, linear.hip:601-622. */
int r97b_iqr_dequant_bf16(const R97IqrDecodeDesc* desc, uint16_t* out_w, int64_t ld_w, void* stream);

/* The stored pair of a decoded weight -- int8 codes [rows, cols] and bf16 scale bits [rows, ceil(cols/group)]
 * (reference src/stored_weight.h StoredWeight) -- as the GEMM operand: W[r, k] = bf16(code * scale), the
 * product and rounding r97b_iqr_dequant_bf16 uses, into `out_w` (row stride `ld_w`).
 * Replaces: the int8-pair reader of the reference's stored-weight dX path (linear.hip:520-600). */
int r97b_codes_dequant_bf16(const int8_t* codes, const uint16_t* scale, int64_t rows, int64_t cols, int64_t group,
                            uint16_t* out_w, int64_t ld_w, void* stream);

/* ------------------------------------------------------------------------------ GEMM */

/* One bf16 operand of logical shape [rows, K]: K-major means stored row-major [rows, K] with row stride
 * `ld`; MN-major means stored row-major [K, rows] with row stride `ld`. */
typedef struct R97bMat {
    const void* ptr;
    int64_t ld;
    int32_t mn_major;
    int32_t _pad;
} R97bMat;

enum {
    R97B_EPI_STORE_BF16 = 0,  /* out[m, n] = bf16(alpha * acc + beta * addend[m, n]) */
    R97B_EPI_STORE_F32 = 1,   /* out[m, n] = alpha * acc + beta * addend[m, n]      */
    R97B_EPI_ATOMIC_F32 = 2,  /* out[m, n] += alpha * acc  (f32, split-K allowed)   */
    R97B_EPI_ATOMIC_F32T = 3, /* out[n, m] += alpha * acc  (f32, split-K allowed)   */
    R97B_EPI_SPLIT_BF16 = 4,  /* out[m, n] = bf16(alpha * acc + beta * addend[m, n]) with the reduction
                               * split `splits` ways: each split stores its f32 partial tile in `ws`, and
                               * the last split of a tile to finish sums the partials in split order
                               * (deterministic) and stores the result */
    R97B_EPI_SWIGLU = 5,      /* the gate/up projection with its SwiGLU: B1 (and B2) hold the gate rows
                               * [0, F) and the up rows [F, 2F), N = 2F, F a multiple of 128; out = [g | u]
                               * (bf16, ldo) and out2[m, j] = bf16(silu(g[m, j]) u[m, j]) (ldo2). Each
                               * 256-column tile of the CTA pair computes gate columns [128 t, 128 t + 128)
                               * and the matching up columns together. */
    R97B_EPI_SWIGLU_BWD = 6,  /* the down projection's input adjoint with SwiGLU's: acc = da [M, F];
                               * addend = [g | u] [M, 2F] (ld_add); out[m, j] = bf16(d u silu'(g)),
                               * out[m, F + j] = bf16(d silu(g)), d = bf16(alpha acc), F = N */
};

/* D[M, N] = alpha * (A1[M, K1] B1[N, K1]^T + A2[M, K2] B2[N, K2]^T) (+ beta * addend), on tcgen05 tensor
 * cores with f32 accumulation in TMEM. K2 = 0 drops the second segment; when present, a2/b2 have the
 * same majorness as a1/b1. `splits` > 1 splits the reduction (atomic epilogues, and R97B_EPI_SPLIT_BF16
 * with a workspace `ws` of at least r97b_gemm_workspace_bytes(g) bytes, 256-byte aligned, zeroed once
 * before its first use: its tile counters return to zero at the end of every call, so it stays reusable,
 * but calls that share one workspace must not overlap on the GPU). `bn` picks the
 * tile: 64, 128 or 256 wide on one SM (128 rows), 512 for a 256 x 256 tile computed by a pair of SMs
 * (tcgen05 cta_group::2, half the operand bytes per multiply-add); 0 picks by shape (the pair for
 * M, N > 128).
 * Replaces: the reference's linear_dx_kernel (src/adjoint/device/linear.hip:172-285) and the LoRA
 * kernels shrink_dx / shrink_da / expand_dt / expand_db (src/adjoint/device/lora.hip:268-399). */
typedef struct R97bGemm {
    int64_t M, N, K1, K2;
    R97bMat a1, b1, a2, b2;
    int32_t mode;
    int32_t splits;
    float alpha;
    float beta;
    void* out;
    int64_t ldo;
    const void* addend;
    int64_t ld_add;
    int32_t bn;
    int32_t _pad;
    void* ws;          /* R97B_EPI_SPLIT_BF16 with splits > 1: the split-K workspace */
    int64_t ws_bytes;
    void* out2;        /* R97B_EPI_SWIGLU: the SwiGLU output */
    int64_t ldo2;
} R97bGemm;

int r97b_gemm(const R97bGemm* g, void* stream);

/* Bytes of workspace r97b_gemm needs for `g` (0 unless g->mode is R97B_EPI_SPLIT_BF16 with splits > 1);
 * -1 for a description r97b_gemm would reject. */
int64_t r97b_gemm_workspace_bytes(const R97bGemm* g);

/* ------------------------------------------------------------------------------ attention */

/* The backward of causal grouped-query attention softmax(scale q k^T) v, given the forward's output `o` and
 * its per-row natural-log log-sum-exp `lse` (of the scaled scores): dq, dk, dv. q, o, dout, dq are bf16
 * [B, Hq, S, D]; k, v, dk, dv bf16 [B, Hkv, S, D]; lse f32 [B, Hq, S]; query head h reads key/value head
 * h / (Hq / Hkv). S a multiple of 128, D 128 or 256, every pointer 16-byte aligned. `ws` (256-byte
 * aligned, r97b_attn_bwd_workspace_bytes bytes) holds the P and dS tiles and the row sums dO . O.
 * Replaces: the reference's attention adjoint (src/adjoint/host/attention.cpp:261-414, the softmax and
 * value products of attention_host_adjoint; its device twin src/adjoint/device/attention.hip). */
typedef struct R97bAttnBwd {
    int32_t B, Hq, Hkv, S, D;
    float scale;
    const void* q;
    const void* k;
    const void* v;
    const void* o;
    const void* dout;
    const float* lse;
    void* dq;
    void* dk;
    void* dv;
    void* ws;
    int64_t ws_bytes;
} R97bAttnBwd;

int r97b_attn_bwd(const R97bAttnBwd* a, void* stream);

/* The forward of causal grouped-query attention: q [B, Hq, S, D], k and v [B, Hkv, S, D] (bf16, dense; query
 * head h reads key/value head h / (Hq / Hkv)), o [B, Hq, S, D] bf16 and lse [B * Hq * S] f32, the natural-log
 * log-sum-exp of each query row's scaled scores (what r97b_attn_bwd reads). S a multiple of 128, D 128 or
 * 256. tcgen05 tensor cores, two passes over each 128-row query block's keys (the row statistics, then the
 * normalised P V). Replaces: attention_twin, src/adjoint/host/attention.cpp:261-313, and the prefill kernels
 * of the reference's device attention row. */
typedef struct R97bAttnFwd {
    int32_t B, Hq, Hkv, S, D;
    float scale;
    const void* q;
    const void* k;
    const void* v;
    void* o;
    float* lse;
} R97bAttnFwd;

int r97b_attn_fwd(const R97bAttnFwd* a, void* stream);
int64_t r97b_attn_bwd_workspace_bytes(int32_t B, int32_t Hq, int32_t S);

/* ------------------------------------------------------------------------------ LoRA linear */

/* One LoRA-adapted linear over a stored weight, forward: W = decode(w) into w_bf16 (skipped when
 * w_decoded, i.e. w_bf16 already holds this weight -- keep it for the backward), t = scale x A^T,
 * y = x W^T + t B^T (+ addend). x [M, K], A [rank, K], B [N, rank], t [M, rank], y and addend [M, N], w_bf16
 * [N, K]: bf16, row-major, dense; K, N and rank multiples of 8. ws: r97b_qlinear_lora_workspace_bytes,
 * zeroed once before its first use (the split-K GEMM's; reusable, not shared between concurrent calls).
 * Replaces: the reference's gemm_nt_q + lora_shrink + lora_expand rows for one slot
 * (src/adjoint/host/linear.cpp:246-317, lora.cpp:226-305, 416-451; device linear.hip, lora.hip K5-K8). */
typedef struct R97bQLinearLora {
    int64_t M, N, K;
    int32_t rank;
    float scale;                   /* alpha / rank */
    const R97IqrDecodeDesc* w;     /* the stored weight [N, K] */
    void* w_bf16;
    int32_t w_decoded;
    int32_t _pad;
    const void* x;
    const void* A;
    const void* B;
    void* t;
    void* y;
    const void* addend;
    void* ws;
    int64_t ws_bytes;
} R97bQLinearLora;

/* Its backward: dt = scale dy B, dx = dy W + dt A, dA += dt^T x, dB += dy^T t (dA [rank, K] and dB [N, rank]
 * f32, accumulated); t is the forward's. Replaces: the same rows' adjoints (linear.cpp:220-243, 246-317,
 * lora.cpp:320-401, 453-521). */
typedef struct R97bQLinearLoraBwd {
    int64_t M, N, K;
    int32_t rank;
    float scale;
    const void* w_bf16;
    const void* x;
    const void* A;
    const void* B;
    const void* t;
    const void* dy;
    void* dt;
    void* dx;
    float* dA;
    float* dB;
    void* ws;
    int64_t ws_bytes;
} R97bQLinearLoraBwd;

int r97b_qlinear_lora_fwd(const R97bQLinearLora* a, void* stream);
int r97b_qlinear_lora_bwd(const R97bQLinearLoraBwd* a, void* stream);
int64_t r97b_qlinear_lora_workspace_bytes(int64_t M, int64_t N, int64_t K, int32_t rank);

/* ------------------------------------------------------------------------------ norms */

/* y = x * rsqrt(mean(x^2) + eps) * (w + wadd) * mult per row of n (x, y bf16 [rows, n]; w f32 [n] or null;
 * rstd f32 [rows] or null receives the row's rsqrt). n a multiple of 8, pointers 16-byte aligned.
 * Replaces: the forward the reference's rmsnorm twin states, src/adjoint/host/elementwise.cpp:459-528. */
int r97b_rmsnorm_fwd(const uint16_t* x, const float* w, uint16_t* y, float* rstd, int64_t rows, int64_t n, float eps,
                     float wadd, float mult, void* stream);

/* dx = mult (s c dy - s^3 x / n sum(dy x c)) + addend, c = w + wadd (addend bf16 or null).
 * Replaces: rmsnorm_adjoint_kernel, src/adjoint/device/elementwise.hip:258,707 (host row
 * src/adjoint/host/elementwise.cpp:531-670). */
int r97b_rmsnorm_bwd(const uint16_t* x, const float* w, const uint16_t* dy, const uint16_t* addend, uint16_t* dx,
                     int64_t rows, int64_t n, float eps, float wadd, float mult, void* stream);

/* o = x * rsqrt(mean(x^2) + eps) * w * act(z), act = silu (act_sigmoid = 0) or sigmoid; per row of n.
 * x and o are dense [rows, n]; z (and dz below) may sit inside wider token rows: with z_heads > 0, row r of z
 * is at (r / z_heads) * z_tok_stride + (r % z_heads) * n (the z columns of a fused projection); z_heads = 0
 * means dense. Replaces: the gdn_gated_rmsnorm forward, src/adjoint/host/gdn_prep.cpp:501-531. */
int r97b_gated_rmsnorm_fwd(const uint16_t* x, const uint16_t* z, int64_t z_tok_stride, int32_t z_heads, const float* w,
                           uint16_t* o, int64_t rows, int64_t n, float eps, int32_t act_sigmoid, void* stream);

/* dx, dz of the gated norm for the cotangent dout (dz laid out like z). Replaces: gated_rmsnorm_adjoint_kernel,
 * src/adjoint/device/gdn_prep.hip:643-731 (host row src/adjoint/host/gdn_prep.cpp:541-592). */
int r97b_gated_rmsnorm_bwd(const uint16_t* x, const uint16_t* z, int64_t z_tok_stride, int32_t z_heads, const float* w,
                           const uint16_t* dout, uint16_t* dx, uint16_t* dz, int64_t rows, int64_t n, float eps,
                           int32_t act_sigmoid, void* stream);

/* ------------------------------------------------------------------------------ loss */

/* Per logit row (bf16, row stride ld; 16-byte aligned rows are read 8 values a load, others one at a
 * time): CE = lse - x[target] into loss_ce[row] (a target of -1, or one outside [0, vocab): not scored,
 * loss 0, gradient 0), KL(softmax(teacher) || softmax(x)) into loss_kl[row] when teacher is given, and
 * grad = grad_scale * (w_ce (softmax - onehot) + w_kl (softmax(x) - softmax(teacher))) as bf16; grad may
 * equal logits (in place), targets may be null (KL only). loss_ce / loss_kl / grad may be null.
 * Replaces: HeadCeKernel / head_ce_kernel, include/r97/head.h:28-55 and src/adjoint/device/head.hip:61-106;
 * the KL term has no counterpart in the reference. */
int r97b_ce_kld(const uint16_t* logits, const uint16_t* teacher, const int32_t* targets, uint16_t* grad,
                float* loss_ce, float* loss_kl, int64_t rows, int64_t vocab, int64_t ld, int64_t ld_t,
                float grad_scale, float w_ce, float w_kl, void* stream);

/* ------------------------------------------------------------------------------ AdamW */

/* One AdamW update of n f32 parameters, bit-identical to the reference's f32 update: g is scaled by inv_k
 * and by *clip_scale (device f32, or null), then m, v and w are updated; zero_grad clears g afterwards.
 * lr, bc1 = 1 - beta1^t and bc2 = 1 - beta2^t are the caller's (reference src/optim.cpp:223-307). */
int r97b_adamw_step(float* w, float* m, float* v, float* g, int64_t n, float lr, float beta1, float beta2, float eps,
                    float weight_decay, float bc1, float bc2, float inv_k, const float* clip_scale,
                    int32_t zero_grad, void* stream);

/* The same update with lr, bc1 and bc2 read from device memory when the kernel runs (sched[0] = lr,
 * sched[1] = bc1, sched[2] = bc2, f32), so that a CUDA graph holding the update advances the schedule by a
 * write to sched before each replay instead of being captured again. Same arithmetic, bit for bit. */
int r97b_adamw_step_dev(float* w, float* m, float* v, float* g, int64_t n, const float* sched, float beta1,
                        float beta2, float eps, float weight_decay, float inv_k, const float* clip_scale,
                        int32_t zero_grad, void* stream);

/* dst += src over n f32 (the optimiser's gradient accumulation; reference src/optim.cpp:231-244). */
int r97b_add_f32(float* dst, const float* src, int64_t n, void* stream);

/* Bytes of scratch r97b_global_norm needs for n elements (one f64 per 4096). */
int64_t r97b_global_norm_scratch_bytes(int64_t n);

/* The global L2 norm of g * inv_k (bit-identical to the reference's chunked f64 sum,
 * src/optim.cpp:132-176) into *out_norm, and the clip factor for max_norm into *out_scale (both device f32;
 * out_scale may be null). `partials` is caller scratch of r97b_global_norm_scratch_bytes(n). */
int r97b_global_norm(const float* g, int64_t n, float inv_k, float max_norm, double* partials, float* out_norm,
                     float* out_scale, void* stream);

/* The largest n r97b_global_norm_noalloc accepts: 65536 partials of 4096 elements. */
#define R97B_GLOBAL_NORM_NOALLOC_MAX_ELEMS (65536LL * 4096LL)

/* r97b_global_norm for callers that cannot allocate device memory -- a host framework whose allocator
 * already owns the device's memory, or a loop that cannot afford cudaMalloc / cudaFree (cudaFree
 * synchronises the whole device). It takes no scratch argument and allocates nothing: its f64 partials
 * live in a fixed 512 KiB array inside the library. A GPU holds that array from the first time it uses the
 * library's kernels (at the latest, this entry point's first call on it) until the process exits. Same
 * results as r97b_global_norm (the same kernels, bit for bit).
 *  - n > R97B_GLOBAL_NORM_NOALLOC_MAX_ELEMS (268,435,456) returns R97B_ETOOLARGE and launches nothing.
 *  - The first call on a device looks up the array's device address (cudaGetSymbolAddress) with that
 *    device current; make that first call before any stream capture.
 *  - All calls share the one array, which keeps the last call's partials; calls whose kernels overlap on
 *    the GPU (two streams, two host threads) race on it, so serialise them.
 * No counterpart in the reference: its optimiser runs on the host. */
int r97b_global_norm_noalloc(const float* g, int64_t n, float inv_k, float max_norm, float* out_norm,
                             float* out_scale, void* stream);

/* ------------------------------------------------------------------------------ GatedDeltaNet */

/* The geometry of one chunked GDN call: n_seq ragged sequences over T tokens (the chunk table comes from
 * r97b_gdn_chunk_table on the host, copied to the device), H value heads sharing Hg query/key heads,
 * head_k = head_v = 128 and chunk = 64 (the only values the kernels take), and the output scale
 * (1/sqrt(head_k) in the reference's architecture). */
typedef struct R97bGdnDims {
    int32_t n_seq, H, Hg, n_chunks;
    int32_t head_k, head_v, chunk, flags; /* flags: R97B_GDN_* below, 0 for the fused layer */
    int64_t T;
    float scale;
    int32_t _pad2;
    const int32_t* chunk_tok0; /* device [n_chunks]: first token of each chunk */
    const int32_t* chunk_len;  /* device [n_chunks]: its length (<= chunk)     */
    const int32_t* seq_chunk0; /* device [n_seq + 1]: first chunk of each sequence */
} R97bGdnDims;

/* The forward reads A (f32 [T, H, 64]: row i of each chunk's (I+M)^-1, its lower triangle with the
 * diagonal; the rest is ignored) instead of solving for it: the reference's gdn_chunk_scan, which takes
 * the gdn_kkt_solve output as an operand. */
#define R97B_GDN_A_GIVEN 1
/* The backward writes the scan's own cotangent of A into R97bGdnBwd.dA (f32 [T, H, 64], lower triangle
 * with the diagonal, zeros above) and leaves the solve's adjoint out of dk, dbeta and dg; the caller
 * applies it with r97b_gdn_kkt_bwd (the reference's gdn_kkt_solve adjoint). */
#define R97B_GDN_SPLIT_KKT 2

/* Fills the chunk table of cu_seqlens (host arrays; any output may be null) and returns the chunk count,
 * or -1 on a bad cu_seqlens. */
int32_t r97b_gdn_chunk_table(const int32_t* cu_host, int32_t n_seq, int32_t chunk, int32_t* tok0_host,
                             int32_t* len_host, int32_t* seq_chunk0_host);

/* Forward operands. q, k: bf16 [T, Hg, 128] (L2-normalised); v: bf16 [T, H, 128]; g: f32 [T, H], the
 * within-chunk cumulative log decay; beta: f32 [T, H]; h0: f32 [n_seq, H, 128(v), 128(k)] or null (zero).
 * Outputs: A f32 [T, H, 64] (the reference's gdn_kkt_solve output, row i of each chunk's (I+M)^-1),
 * w, u f32 [T, H, 128], S f32 [n_chunks, H, 128(k), 128(v)] (the state entering each chunk), Vp f32
 * [T, H, 128], P f32 [n_chunks, H, 64, 64], o bf16 [T, H, 128] and ht f32 [n_seq, H, 128, 128] or null.
 * A, w, S, Vp and P are what the backward reads; u is scratch. w and P are opaque to the caller: they
 * are kept as bf16 (hi, lo) pairs -- hi = bf16(x), lo = bf16(x - hi), the hi plane first -- in the bytes
 * of the f32 buffers described here, which are what the tensor-core passes stream. */
typedef struct R97bGdnFwd {
    const uint16_t *q, *k, *v;
    const float *g, *beta, *h0;
    float *A, *w, *u, *S, *Vp, *P;
    uint16_t* o;
    float* ht;
} R97bGdnFwd;

/* Backward operands: the forward's inputs and saved A, w, S, Vp, P; dO bf16 [T, H, 128]; dht f32 or null.
 * Scratch: dS f32 [n_chunks, H, 128, 128], dVp, dw f32 [T, H, 128]. pdq, pdk, pdg are not read: the
 * partial sums of the state-reading pass accumulate in dq, dk and dg; the fields keep the struct's layout
 * and may be null.
 * Outputs: dq, dk f32 [T, H, 128] per VALUE head (sum the heads sharing a key head with
 * r97b_gdn_sum_heads), dv f32 [T, H, 128], dbeta, dg f32 [T, H], dh0 f32 or null. */
typedef struct R97bGdnBwd {
    const uint16_t *q, *k, *v;
    const float *g, *beta;
    const float *A, *w, *S, *Vp, *P;
    const uint16_t* dO;
    const float* dht;
    float *dS, *dVp, *dw, *pdq, *pdk, *pdg;
    float *dq, *dk, *dv, *dbeta, *dg, *dh0;
    float* dA; /* R97B_GDN_SPLIT_KKT only: the scan's cotangent of A, f32 [T, H, 64]; else unused */
} R97bGdnBwd;

/* The forward of the reference's gdn_kkt_solve + gdn_chunk_scan pair (src/adjoint/host/gdn_kkt.cpp:221-270,
 * gdn_scan.cpp:418-485). Replaces: gdn_kkt_adjoint_kernel / gdn_scan_adjoint_kernel's forward replays and
 * radiance's chunked GDN forward (src/adjoint/device/gdn_kkt.hip, gdn_scan.hip). */
int r97b_gdn_fwd(const R97bGdnDims* dims, const R97bGdnFwd* args, void* stream);

/* The adjoint of the same pair: the scan's adjoint and the kkt solve's adjoint composed
 * (src/adjoint/host/gdn_scan.cpp:487-580 + gdn_kkt.cpp:272-352). Replaces: gdn_scan_adjoint_kernel and
 * gdn_kkt_adjoint_kernel, src/adjoint/device/gdn_scan.hip:235-600 and gdn_kkt.hip:229-424. */
int r97b_gdn_bwd(const R97bGdnDims* dims, const R97bGdnBwd* args, void* stream);

/* The kkt solve's adjoint alone (reference src/adjoint/host/gdn_kkt.cpp:272-352), for the split form:
 * from k bf16 [T, Hg, 128], g, beta f32 [T, H], the solve's output A and its cotangent dA (f32 [T, H, 64],
 * lower triangles) it WRITES dk f32 [T, H, 128] per value head, dbeta and dg f32 [T, H].
 * Replaces: gdn_kkt_adjoint_kernel, src/adjoint/device/gdn_kkt.hip:229-424. */
int r97b_gdn_kkt_bwd(const R97bGdnDims* dims, const uint16_t* k, const float* g, const float* beta, const float* A,
                     const float* dA, float* dk, float* dbeta, float* dg, void* stream);

/* dst[t, j, :] = sum_{h in key head j's value heads} src[t, h, :] (f32 [T, H, 128] -> [T, Hg, 128]). */
int r97b_gdn_sum_heads(const float* src, float* dst, int64_t T, int32_t H, int32_t Hg, void* stream);

/* ------------------------------------------------------------------------------ block kernels */

/* The GDN input prep: causal depthwise conv (width 4, weight f32 [conv_dim, 4], no bias) + silu over the first
 * conv_dim = (2 Hg + H) * 128 columns of x (bf16 rows of ldx: q | k | v channels), then the L2 norm
 * (eps 1e-6) of every q and k head. Out: q, k bf16 [T, Hg, 128], v bf16 [T, H, 128]. cu: device i32
 * [n_seq + 1]; the conv window never crosses a sequence start (a cold prefill).
 * Replaces: the conv / l2 phases of gdn_conv_prep, src/adjoint/host/gdn_prep.cpp:204-365 and
 * src/adjoint/device/gdn_prep.hip:242-359. */
int r97b_conv_prep_fwd(const uint16_t* x, int64_t ldx, const float* conv_w, const int32_t* cu, int32_t n_seq,
                       int64_t T, int32_t Hg, int32_t H, uint16_t* q, uint16_t* k, uint16_t* v, void* stream);

/* Its adjoint from the f32 cotangents of q, k ([T, dqk_heads, 128]: dqk_heads = Hg, or H when they are still
 * per value head -- the heads sharing a key head are summed as they are read) and v ([T, H, 128]), into dx
 * (the first conv_dim columns of bf16 rows of lddx), in one pass with no scratch.
 * Replaces: gdn_conv_prep_host_adjoint's conv / l2 terms, src/adjoint/host/gdn_prep.cpp:367-455. */
int r97b_conv_prep_bwd(const uint16_t* x, int64_t ldx, const float* conv_w, const int32_t* cu, int32_t n_seq,
                       int64_t T, int32_t Hg, int32_t H, const float* dq, const float* dk, const float* dv,
                       int32_t dqk_heads, uint16_t* dx, int64_t lddx, void* stream);

/* beta = sigmoid(b), g = within-chunk running sum of -exp(A_log) softplus(a + dt_bias) (threshold 20), from
 * ba rows (bf16, ldba) holding b in columns [0, H) and a in [H, 2H); chunks (at most 64 tokens each) from
 * r97b_gdn_chunk_table with chunk 64. Replaces: the gate phase of gdn_conv_prep,
 * src/adjoint/host/gdn_prep.cpp:320-336. */
int r97b_gates_fwd(const uint16_t* ba, int64_t ldba, const float* a_log, const float* dt_bias,
                   const int32_t* chunk_tok0, const int32_t* chunk_len, int32_t n_chunks, int32_t H, float* g,
                   float* beta, void* stream);

/* The adjoint of r97b_gates_fwd into dba (bf16 rows of lddba). Replaces:
 * src/adjoint/host/gdn_prep.cpp:467-488. */
int r97b_gates_bwd(const uint16_t* ba, int64_t ldba, const float* a_log, const float* dt_bias,
                   const int32_t* chunk_tok0, const int32_t* chunk_len, int32_t n_chunks, int32_t H,
                   const float* dg, const float* dbeta, uint16_t* dba, int64_t lddba, void* stream);

/* y = silu(gate) * up over fused rows [gate (n) | up (n)]. Replaces: silu_mul's twin,
 * src/adjoint/host/elementwise.cpp:278-293. */
int r97b_swiglu_fwd(const uint16_t* gu, int64_t ldgu, int64_t rows, int64_t n, uint16_t* y, int64_t ldy,
                    void* stream);

/* Its adjoint into fused rows dgu. Replaces: silu_mul_host_adjoint, src/adjoint/host/elementwise.cpp:295-312. */
int r97b_swiglu_bwd(const uint16_t* gu, int64_t ldgu, int64_t rows, int64_t n, const uint16_t* dy, int64_t lddy,
                    uint16_t* dgu, int64_t lddgu, void* stream);

/* Per (token, head) row of head_dim (128 or 256): RMSNorm (gain w f32 [head_dim], eps) then NeoX RoPE on the
 * first `rot` dims (cos / sin tables f32 [S, rot/2]), from rows of x (row_stride, head h at h * head_stride)
 * into out[b, head, s, :] for a fixed-length batch (T = B * S). rot / 2 / (head_dim / 32) must be a power of
 * two up to 16 (rot 16..256 at head_dim 256, 8..128 at 128). Replaces: the q/k norm + rope forward,
 * src/adjoint/host/qk.cpp and rope.cpp. */
int r97b_qk_norm_rope_fwd(const uint16_t* x, int64_t row_stride, int32_t head_stride, int32_t heads,
                          int32_t head_dim, const float* w, const float* cos_tab, const float* sin_tab, int32_t rot,
                          int64_t T, int32_t S, float eps, uint16_t* out, void* stream);

/* Its adjoint into dx (rows of dx_stride, the same head layout). Replaces: qk_adjoint_kernel,
 * src/adjoint/device/qk.hip:254-488. */
int r97b_qk_norm_rope_bwd(const uint16_t* x, int64_t row_stride, int32_t head_stride, int32_t heads,
                          int32_t head_dim, const float* w, const float* cos_tab, const float* sin_tab, int32_t rot,
                          int64_t T, int32_t S, float eps, const uint16_t* dout, uint16_t* dx, int64_t dx_stride,
                          void* stream);

/* [T, heads, head_dim] rows -> [B, heads, S, head_dim] (reverse = 1: back into the rows); head_dim 128 or
 * 256. */
int r97b_to_bhsd(const uint16_t* x, int64_t row_stride, int32_t head_stride, int32_t heads, int32_t head_dim,
                 int64_t T, int32_t S, uint16_t* out, int32_t reverse, void* stream);

/* y[t, h * head_dim + d] = attn[b, h, s, d] * sigmoid(gate[t, h * gate_hs + d]): the gated attention's
 * output gate (head_dim 128 or 256). Replaces: the gate half of attention.cpp's twin and gate_ste_kernel,
 * attention.hip:562. */
int r97b_gate_mul_fwd(const uint16_t* attn, const uint16_t* gate, int64_t gate_stride, int32_t gate_hs,
                      int32_t heads, int32_t head_dim, int64_t T, int32_t S, uint16_t* y, void* stream);

/* Its adjoint: dattn [B, heads, S, head_dim] and dgate (rows of dgate_stride). */
int r97b_gate_mul_bwd(const uint16_t* attn, const uint16_t* gate, int64_t gate_stride, int32_t gate_hs,
                      int32_t heads, int32_t head_dim, int64_t T, int32_t S, const uint16_t* dy, uint16_t* dattn,
                      uint16_t* dgate, int64_t dgate_stride, void* stream);

/* out[t, :] = table[ids[t], :] (bf16, zero for an id outside [0, vocab)). Replaces: embed_lookup's twin,
 * src/adjoint/host/linear.cpp:388-418 (a stop: no adjoint). */
int r97b_embed(const uint16_t* table, int64_t ld, int64_t vocab, const int32_t* ids, int64_t T, int64_t n,
               uint16_t* out, void* stream);

/* dst (bf16, ld_dst) = src (f32, ld_src), rows x cols: the adapter's bf16 mirrors after an update. */
int r97b_cast_f32_bf16(const float* src, int64_t ld_src, uint16_t* dst, int64_t ld_dst, int64_t rows, int64_t cols,
                       void* stream);

/* One segment of a batched cast: rows x cols (cols a multiple of 8) f32 -> bf16; `unit0` = the 8-element
 * units of every segment before it in the table. src and dst rows 16-byte aligned. */
typedef struct R97bCastSeg {
    const float* src;
    int64_t ld_src;
    void* dst;
    int64_t ld_dst;
    int64_t rows;
    int64_t cols;
    int64_t unit0;
} R97bCastSeg;

/* Every segment of a table (in DEVICE memory, nseg entries, `units` = the table's total 8-element units)
 * cast in one launch: the adapter's bf16 mirrors refreshed after an update (the reference keeps one f32
 * master per adapter tensor and hands the device its bf16 view, src/delta_lora.cpp). */
int r97b_cast_segments(const R97bCastSeg* segs, int32_t nseg, int64_t units, void* stream);

/* ---- the w8a8 trunk's activation quantisers (reference src/adjoint/host/quant.cpp:43-370, the
 * quant_act_i8g / had_quant_act_i8g records; docs/adjoints/quant.md s1, s3) ----
 * Per row and group of `group` columns: v = the group, rotated by the unnormalised Walsh-Hadamard matrix of
 * order `group` (W W = group I) when `rotate`; s = amax|v| / 127 (1 for an all-zero group); codes =
 * rint(clamp(v / s, -127, 127)), nearest even, as int8; scale[row, g] = s (f32).
 * x: bf16 [rows, n] (row pitch ldx); codes: int8 [rows, n] (pitch ldc); scale: f32 [rows, ceil(n / group)].
 * rotate: group a power of two of at most 256 dividing n, n a multiple of 4, x rows 8-byte (16-byte for
 * 256) aligned, codes rows 4-byte (8-byte) aligned. Not rotated: group <= 0 or > n is one group a row, and a
 * group that does not divide n leaves a short last group. R97B_EINVAL outside these rules (the reference
 * twin's std::invalid_argument). */
int r97b_quant_act_i8g(const uint16_t* x, int64_t ldx, int64_t rows, int64_t n, int64_t group, int32_t rotate,
                       int8_t* codes, int64_t ldc, float* scale, void* stream);
/* The straight-through adjoint (quant.cpp quant_adjoint): dx = W (m . g / s), m = 0 where the clamp engaged
 * (|v / s| > 127, v recomputed from x), W the same rotation (the identity when not rotated); the scale's
 * cotangent is dropped. g: f32 [rows, n] (pitch ldg), the codes' cotangent; scale: the forward's; dx: f32
 * [rows, n] (pitch lddx), written, or added to when `accumulate`. g and dx rows 16-byte aligned on the
 * rotated path. */
int r97b_quant_act_i8g_bwd(const uint16_t* x, int64_t ldx, int64_t rows, int64_t n, int64_t group, int32_t rotate,
                           const float* scale, const float* g, int64_t ldg, float* dx, int64_t lddx,
                           int32_t accumulate, void* stream);

/* ---- the int8 trunk's fused producers: an elementwise part, then the rotated quantiser above over the part's
 * f32 value (reference src/adjoint/host/quant.cpp:821-1100, rmsnorm_had_quant_i8g / gated_had_quant_i8g /
 * gate_had_quant_i8g; device src/adjoint/device/quant.hip) ----
 * part R97B_PART_RMSNORM:     v = x s (w + wadd) mult, s = 1 / sqrt(mean(x^2) + eps); x bf16 [rows, n], w f32
 *                             [n] or null (then wadd must be 0)
 * part R97B_PART_SILU_MUL:    v = silu(g) u; x = gate_up bf16 [rows, 2 n] (pitch ldx >= 2 n), the gate first
 * part R97B_PART_SIGMOID_MUL: v = sigmoid(a) b; x = a, x2 = b, bf16 [rows, n]
 * codes: int8 [rows, n] (pitch ldc, a multiple of 8, 8-byte aligned); scale: f32 [rows, n / group] (pitch lds);
 * out: v as bf16 [rows, n] (pitch ldo, a multiple of 8, 16-byte aligned) or null. group: a power of two of at
 * most 256 dividing n; n a multiple of 8; x / x2 rows 16-byte aligned. */
enum { R97B_PART_RMSNORM = 0, R97B_PART_SILU_MUL = 1, R97B_PART_SIGMOID_MUL = 2 };
int r97b_fused_quant_i8g(int32_t part, const uint16_t* x, int64_t ldx, const uint16_t* x2, int64_t ldx2,
                         const float* w, float eps, float wadd, float mult, int64_t rows, int64_t n, int64_t group,
                         int8_t* codes, int64_t ldc, float* scale, int64_t lds, uint16_t* out, int64_t ldo,
                         void* stream);
/* Their adjoint: dv = W (m . g / s) + g_out (m = 0 where |v / s| > 127, v recomputed; g the codes' cotangent
 * f32 [rows, n], g_out the `out` write's or null), then the part's adjoint into dx (rmsnorm: dx [rows, n];
 * silu_mul: d gate_up [rows, 2 n]; sigmoid mul: da in dx, db in dx2), written or added to when `accumulate`.
 * The gain is not differentiated (the record's frozen operand). g, g_out, dx, dx2 rows 16-byte aligned (pitches
 * multiples of 4); the rmsnorm part takes n <= 16384. */
int r97b_fused_quant_i8g_bwd(int32_t part, const uint16_t* x, int64_t ldx, const uint16_t* x2, int64_t ldx2,
                             const float* w, float eps, float wadd, float mult, int64_t rows, int64_t n,
                             int64_t group, const float* scale, int64_t lds, const float* g, int64_t ldg,
                             const float* g_out, int64_t ldgo, float* dx, int64_t lddx, float* dx2, int64_t lddx2,
                             int32_t accumulate, void* stream);

/* y[r, c] = x[r, c] s[r, c / group]: f32 x [rows, cols] (pitch ldx), f32 s [rows, ceil(cols / group)] (pitch
 * lds), y [rows, cols] (pitch ldy) f32 (may be x) or bf16 when y_bf16. The group scales of the int8 trunk's
 * products on a float operand or result: the dequantised weight code[n, k] b_scale[n, k / 128] and the
 * activation scale a dX takes (reference src/adjoint/host/linear.cpp:286-317, gemm_nt_q_adjoint). */
int r97b_group_scale(const float* x, int64_t ldx, int64_t rows, int64_t cols, int64_t group, const float* s,
                     int64_t lds, void* y, int64_t ldy, int32_t y_bf16, void* stream);

/* ---- the w8a8 trunk's int8 product (tcgen05 kind::i8), groups of 128 along K ----
 * y[m, n] = sum_g a_scale[m, g] b_scale[n, g] sum_{k in g} a[m, k] b[n, k]: gemm_nt_q at dtype i8a8h
 * (reference src/adjoint/host/linear.cpp:246-282; its device row src/adjoint/device/linear.hip:748-760 serves
 * group 128 only). a: int8 [M, K] (pitch lda), b: int8 [N, K] (pitch ldb), both 16-byte aligned with K, lda,
 * ldb multiples of 16; a_scale: f32 [M, ceil(K / 128)] (pitch ld_as), b_scale: f32 [N, ceil(K / 128)]
 * (pitch ld_bs). y: [M, N] (pitch ldy, N and ldy multiples of 4), f32, or bf16 when y_bf16 (16- / 8-byte
 * aligned). Products accumulate exactly in s32 per group and in f32 across groups. */
int r97b_gemm_i8g(const int8_t* a, int64_t lda, const float* a_scale, int64_t ld_as, const int8_t* b, int64_t ldb,
                  const float* b_scale, int64_t ld_bs, int64_t M, int64_t N, int64_t K, void* y, int64_t ldy,
                  int32_t y_bf16, void* stream);
/* The gated narrow fold, gemm_nt_q_gated (reference src/adjoint/host/gemm_nt_q_gated.cpp:11-14, 256-320): the
 * same product over b = [gate rows; up rows] (N = 2 n, n a multiple of 128), p[m, j] = act(z[m, j]) z[m, n + j]
 * (act: silu, or the sigmoid when act_sigmoid), and per 128-wide group of p the rotated quantiser of
 * had_quant_act_i8g: v = W p, s = amax|v| / 127 (1 for an all-zero group), q = rint(clamp(v / s, +-127)).
 * q: int8 [M, n] (pitch ldq, a multiple of 4, 4-byte aligned); q_scale: f32 [M, n / 128] (pitch ld_qs);
 * out_bf16: the unrotated p as bf16 [M, n] (pitch ld_ob, a multiple of 4, 8-byte aligned), or null. */
int r97b_gemm_i8g_gated(const int8_t* a, int64_t lda, const float* a_scale, int64_t ld_as, const int8_t* b,
                        int64_t ldb, const float* b_scale, int64_t ld_bs, int64_t M, int64_t N, int64_t K,
                        int32_t act_sigmoid, int8_t* q, int64_t ldq, float* q_scale, int64_t ld_qs,
                        uint16_t* out_bf16, int64_t ld_ob, void* stream);

/* How many kernels this library has launched in this process (a diagnostic for the bench). */
uint64_t r97b_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* R97B_H */
