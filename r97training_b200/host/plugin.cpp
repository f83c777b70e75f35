// plugin.cpp -- the load-time registration of libr97host.so and its two non-row kernels: the head's CE
// chunk (HeadCeKernel) and the vocab head's cast (VocabHeadKernels).
//
// Loaded into a process that holds the reference's registry, the plugin's static initialiser registers
// the device adjoint rows (gemm_nt, lora_shrink, lora_expand[_mm], rmsnorm, gdn_gated_rmsnorm,
// gdn_kkt_solve, gdn_chunk_scan), the head's CE kernel and the vocab head's kernels, in the same
// direction the reference's device plugin takes (src/adjoint/device/plugin.hip, head.hip:112-118): the
// plugin resolves the host's symbols at load, never the other way round. In a process without them the
// weak references are null and nothing registers.
#include "common.h"
#include "../../include/r97host.h"

namespace r97b_host {
void register_linear_rows();
void register_norm_rows();
void register_gdn_rows();
void register_quant_rows();

namespace {

// The head's CE over one chunk of logit rows (reference include/r97/head.h:28-55, head.hip:61-106):
// loss = lse - x[target] and grad = (softmax - onehot) * grad_scale as bf16, zero for an unscored row
// (id -1). Queues on the chunk's stream (the row stream when null) and does not wait.
bool head_ce_chunk(const r97::HeadChunk& chunk, const char** error) {
    if (!chunk.logits || !chunk.ids) {
        if (error) *error = "a chunk needs its logits and its ids";
        return false;
    }
    if (chunk.positions <= 0 || chunk.vocab <= 0) {
        if (error) *error = "a chunk needs rows and a vocabulary";
        return false;
    }
    if (!chunk.grad && !chunk.loss) return true;
    void* stream = chunk.stream ? chunk.stream : row_stream();
    const int st = r97b_ce_kld(static_cast<const uint16_t*>(chunk.logits), nullptr, chunk.ids,
                               static_cast<uint16_t*>(chunk.grad), chunk.loss, nullptr, chunk.positions, chunk.vocab,
                               chunk.vocab, 0, chunk.grad_scale, 1.0f, 0.0f, stream);
    if (st != R97B_OK) {
        if (error) *error = st == R97B_EINVAL ? "the chunk's buffers are misaligned or its sizes out of range"
                                              : r97b_last_cuda_error();
        return false;
    }
    return true;
}

// dst (bf16) <- src (f32), `values` of them, on `stream` (reference vocab_head.h:104-106).
bool vocab_head_cast(void* dst, const void* src, int64_t values, void* stream) {
    if (!dst || !src || values < 0) return false;
    if (values == 0) return true;
    return r97b_cast_f32_bf16(static_cast<const float*>(src), values, static_cast<uint16_t*>(dst), values, 1, values,
                              stream ? stream : row_stream()) == R97B_OK;
}

// The tied head's transpose reads radiance's class planes (VocabHeadPlan), which exist only in the
// reference's container reader; this build has none, so it says so and does nothing.
bool vocab_head_transpose(const r97::VocabHeadPlan&, const void*, int64_t, float*, void*, std::string* error) {
    if (error)
        *error = "r97b: vocab_head_transpose: the head's class planes come from radiance's container, which this "
                 "build does not read; the tied head's dX runs through r97b_gemm";
    return false;
}

struct Registration {
    Registration() {
        register_linear_rows();
        register_norm_rows();
        register_gdn_rows();
        register_quant_rows();
        if (r97::head_ce_register) r97::head_ce_register(head_ce_chunk);
        if (r97::register_vocab_head_kernels)
            r97::register_vocab_head_kernels(r97::VocabHeadKernels{vocab_head_transpose, vocab_head_cast});
    }
};
const Registration registration;

}  // namespace

r97::HeadCeKernel head_ce_kernel() { return head_ce_chunk; }

}  // namespace r97b_host

// ---- C entry points for a caller without the reference's host (tests, tools)

extern "C" {

// Whether the plugin found the reference's registry when it loaded (1) or registered nowhere (0).
int r97host_registered(void) { return r97::adjoint_register ? 1 : 0; }

// Runs the plugin's HeadCeKernel on a chunk laid out as the reference's HeadChunk; 0 on success, 1 with
// the kernel's message in *error otherwise.
int r97host_head_ce(const void* chunk, const char** error) {
    if (!chunk) return 1;
    return r97b_host::head_ce_kernel()(*static_cast<const r97::HeadChunk*>(chunk), error) ? 0 : 1;
}

// The step's gradient stage into a reference ParamSet (a pointer to std::vector<r97::Param>), as the
// walk's grad_stage_flush at the end of a step; 0 on success.
int r97host_grad_stage_flush(void* paramset) {
    return r97::device::grad_stage_flush(static_cast<r97::ParamSet*>(paramset)) ? 0 : 1;
}

void r97host_grad_stage_discard(void) { r97::device::grad_stage_discard(); }

// The scratch allocator's counters: live bytes, peak bytes, allocations since the last reset.
void r97host_scratch_stats(int64_t* live, int64_t* peak, int64_t* allocations) {
    const r97::device::ScratchStats s = r97::device::scratch_stats();
    if (live) *live = s.live_bytes;
    if (peak) *peak = s.peak_bytes;
    if (allocations) *allocations = s.allocations;
}

// Waits for the plugin's row stream.
int r97host_sync(void) { return r97b_stream_sync(r97b_host::row_stream()); }

}  // extern "C"
