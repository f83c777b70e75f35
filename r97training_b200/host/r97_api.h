// r97_api.h -- the reference trainer's plugin-facing C++ types and registry entry points, declared so
// that this library binds to them by name and layout.
//
// The adjoint-row plugin (libr97host.so) is loaded into a process that already holds the reference's
// registry (its trainer, or any program linking its adjoint_registry.cpp and stored_weight.cpp): rows
// register themselves at load time the way the reference's own device rows do (reference
// include/r97/adjoint.h:183-235, src/adjoint/device/plugin.hip). The structs below must match the
// reference's member for member -- the registry and the walk hand them across the library boundary by
// reference -- so their members, order and types follow reference include/r97/op.h:18-60,
// include/r97/params.h:14-22, include/r97/batch.h:12-17, include/r97/step.h:18-27, include/r97/adjoint.h:49-168, include/r97/head.h:28-55,
// src/stored_weight.h:27-55 and src/adjoint/device/scratch.h / grad_stage.h.
//
// The host's entry points (registration, the stored-weight table, the head's registration) are declared
// weak: a process without the reference's registry still loads the plugin, and its rows then register
// nowhere -- the behaviour of the reference plugin's fallback definitions (plugin.hip:55-80).
#pragma once

#include <cstdint>
#include <functional>
#include <string>
#include <utility>
#include <variant>
#include <vector>

namespace r97 {

// ---------------------------------------------------------------- records (reference op.h)

struct Operand {
    std::string buffer;
    std::string dtype;
    std::vector<int64_t> shape;
    int64_t row_lo = 0;
    int64_t rows = 0;
    bool written = false;
    bool in_place = false;
    std::vector<int64_t> view_shape;
    std::vector<int64_t> view_stride;
    int64_t view_off = 0;
    const void* enc = nullptr;
};

struct OpRecord {
    std::string op;
    std::vector<std::pair<std::string, std::variant<int64_t, std::string>>> params;
    std::vector<Operand> operands;
    int64_t block = -1;
    int64_t position = 0;
    int64_t n = 0;
};

// ---------------------------------------------------------------- trainable leaves (reference params.h)

struct Param {
    std::string name;
    std::vector<int64_t> shape;
    std::vector<float> value;
};
using ParamSet = std::vector<Param>;

// ---------------------------------------------------------------- a step (reference batch.h, step.h)

struct TokenSeq {
    std::vector<int32_t> ids;    // the sequence's token ids
    std::vector<uint8_t> score;  // 1 where token i is a target predicted at position i - 1
};
using Batch = std::vector<TokenSeq>;

struct StepResult {
    double loss;      // summed over the batch's scored tokens
    int64_t scored;   // how many scored tokens the loss covered
};

// grads == nullptr means forward only
using StepFn = std::function<StepResult(const Batch&, const ParamSet& params, ParamSet* grads)>;

// ---------------------------------------------------------------- the adjoint contract (reference adjoint.h)

using OpParam = std::pair<std::string, std::variant<int64_t, std::string>>;

enum class Side { host, device };

struct AdValue {
    std::string dtype;
    std::vector<int64_t> shape;
    std::vector<double> value;
    const void* raw = nullptr;
    const void* enc = nullptr;
};

struct AdjointCall {
    const OpRecord& rec;
    const std::vector<AdValue>& fwd;
    const std::vector<AdValue>& cot;
    std::vector<AdValue>* dc;
    ParamSet* grads;
    const char* prefix;
    std::function<std::string(int64_t slot)> slot_prefix;
    bool fused_slots = false;
    const std::vector<int64_t>* read_rows = nullptr;
    struct RowCount {
        int64_t zeroed_unreadable = 0;
        int64_t readable = 0;
        int64_t refused_non_finite = 0;
    };
    RowCount* row_count = nullptr;
};

using TwinFn = void (*)(const OpRecord& rec, const std::vector<AdValue>& operands, std::vector<AdValue>* out);
using AdjointFn = void (*)(const AdjointCall& call);
using ParamPred = bool (*)(const std::vector<OpParam>& params);

// The host's registry (reference src/adjoint_registry.cpp).
void adjoint_register(const char* op, Side side, AdjointFn fn, const std::vector<int>& frozen, ParamPred pred)
    __attribute__((weak));

// ---------------------------------------------------------------- stored weights (reference stored_weight.h)

struct StoredWeight {
    int64_t rows = 0;
    int64_t cols = 0;
    int64_t groups = 0;
    std::vector<int8_t> codes;
    std::vector<uint16_t> scale;
};
const StoredWeight* stored_weight_find(const void* enc, int64_t rows, int64_t cols) __attribute__((weak));

// ---------------------------------------------------------------- the head's CE chunk (reference head.h)

struct HeadChunk {
    void* logits = nullptr;
    void* grad = nullptr;
    float* loss = nullptr;
    int32_t* ids = nullptr;
    int64_t positions = 0;
    int64_t vocab = 0;
    float grad_scale = 1.0f;
    void* stream = nullptr;
};
using HeadCeKernel = bool (*)(const HeadChunk& chunk, const char** error);
void head_ce_register(HeadCeKernel fn) __attribute__((weak));

// ---------------------------------------------------------------- the vocab head's kernels (reference vocab_head.h)

struct VocabHeadPlan;  // radiance's class planes; opaque here
struct VocabHeadKernels {
    bool (*transpose)(const VocabHeadPlan& plan, const void* dy, int64_t rows, float* d_x, void* stream,
                      std::string* error);
    bool (*cast)(void* dst, const void* src, int64_t values, void* stream);
};
void register_vocab_head_kernels(const VocabHeadKernels& kernels) __attribute__((weak));

// ---------------------------------------------------------------- device memory the rows use (plugin side)
// The reference keeps these in its device library (src/adjoint/device/scratch.h, grad_stage.h); this
// plugin is that library here, so it defines them.

namespace device {

struct ScratchStats {
    int64_t live_bytes = 0;
    int64_t peak_bytes = 0;
    int64_t allocations = 0;
};
ScratchStats scratch_stats();
void scratch_reset();
// A block of at least `bytes` (256-byte aligned), or null when the device has no room. Blocks are
// stream-ordered on the plugin's row stream: a freed block may serve the next allocation before the
// kernels queued on that stream finish, so a caller that reads a block from another stream synchronises
// that stream before scratch_free.
void* scratch_alloc(int64_t bytes);
void scratch_free(void* p);

struct ScratchBlock {
    void* p = nullptr;
    explicit ScratchBlock(int64_t bytes) : p(scratch_alloc(bytes)) {}
    ~ScratchBlock() { scratch_free(p); }
    ScratchBlock(const ScratchBlock&) = delete;
    ScratchBlock& operator=(const ScratchBlock&) = delete;
    ScratchBlock(ScratchBlock&&) = delete;
    ScratchBlock& operator=(ScratchBlock&&) = delete;
    explicit operator bool() const { return p != nullptr; }
};

float* grad_stage_slot(const std::string& name, const std::vector<int64_t>& shape);
int64_t grad_stage_bytes();
bool grad_stage_flush(ParamSet* grads);
void grad_stage_discard();

}  // namespace device
}  // namespace r97
