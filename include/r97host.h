/* r97host.h -- the C entry points of libr97host.so, the adjoint-row plugin.
 *
 * The plugin's real interface is the reference's C++ one: loaded into a process that holds the
 * reference's registry (adjoint_register, stored_weight_find, head_ce_register,
 * register_vocab_head_kernels), it registers its device rows and kernels there at load time, the way
 * the reference's device plugin does (reference src/adjoint/device/plugin.hip, include/r97/adjoint.h:
 * 183-235, include/r97/head.h:50-55, src/vocab_head.h:78-85). The functions below serve a caller that
 * has no reference host of its own -- a test or a tool -- and have no counterpart in the reference. */
#ifndef R97HOST_H
#define R97HOST_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 1 when the plugin found the reference's registry at load and registered its rows, else 0. */
int r97host_registered(void);

/* The plugin's HeadCeKernel on a chunk laid out as the reference's r97::HeadChunk (logits, grad, loss,
 * ids, positions, vocab, grad_scale, stream); 0 on success, 1 with a message in *error. */
int r97host_head_ce(const void* chunk, const char** error);

/* Adds the step's gradient stage into a reference ParamSet (std::vector<r97::Param>*), one bf16 rounding
 * per leaf, and frees the stage: the walk's grad_stage_flush at the end of a step. 0 on success. */
int r97host_grad_stage_flush(void* paramset);
/* Frees the stage without copying it out. */
void r97host_grad_stage_discard(void);

/* The scratch allocator's counters since its last reset. */
void r97host_scratch_stats(int64_t* live, int64_t* peak, int64_t* allocations);

/* Waits for everything the plugin's rows queued. */
int r97host_sync(void);

/* ---- the reference's Optimiser over device memory (include/r97/optim.h:26-90, src/optim.cpp) ----
 * AdamW with the reference's schedule (linear warm-up, cosine to lr * lr_floor_frac at total_steps),
 * global-norm clipping of the accumulated mean, gradient accumulation over accum_steps calls and weight
 * decay skipped for parameters whose name contains a no_decay substring. The parameters are one flat f32
 * device buffer `w` holding the named parameters in order (counts[i] elements each); the optimiser keeps
 * its moments and accumulation buffer on the device. Its updates are bit-identical to the reference
 * Optimiser's and its serialised state is the reference's "R97OPT" byte format, so either restores the
 * other's checkpoint. All work is queued on `stream`; serialise and restore synchronise it. */
typedef struct R97hostAdamW {
    float lr, beta1, beta2, eps, weight_decay, clip_norm;
    int32_t warmup_steps, total_steps;
    float lr_floor_frac;
    int32_t accum_steps;
} R97hostAdamW;

/* A new optimiser, or null (message in r97host_optim_error). */
void* r97host_optim_create(const R97hostAdamW* cfg, int32_t nparams, const char* const* names, const int64_t* counts,
                           float* w, const char* const* no_decay, int32_t n_no_decay, void* stream);
/* Adds `grad` (device, the flat layout of w) into the accumulation; every accum_steps-th call applies one
 * update. 1: updated, 0: accumulated, -1: error. */
int r97host_optim_step(void* opt, const float* grad);
int r97host_optim_state(void* opt, int32_t* updates_done, int32_t* pending);
/* Writes the serialised state to out when cap is large enough; returns its size in bytes (-1 on error). */
int64_t r97host_optim_serialise(void* opt, uint8_t* out, int64_t cap);
/* Replaces the state (weights included) from serialised bytes; 0 on success, 1 (state unchanged) on bad
 * bytes. */
int r97host_optim_restore(void* opt, const uint8_t* bytes, int64_t size);
void r97host_optim_destroy(void* opt);
const char* r97host_optim_error(void);

/* ---- the adapter directory in PEFT's layout (reference include/r97/adapter_io.h, src/adapter_io.cpp) ----
 * adapter_config.json (PEFT's keys in PEFT's order) and adapter_model.safetensors (tensors sorted by name,
 * `base_model.model.<module>.lora_A.weight`, f32 or bf16): the files the reference's trainer writes and its
 * server reads. */
typedef struct R97hostAdapterConfig {
    const char* base_model;      /* base_model_name_or_path */
    int64_t rank;                /* r */
    double alpha;                /* lora_alpha */
    const char* const* targets;  /* target_modules */
    int32_t n_targets;
    const char* input_basis;     /* radiance_input_basis ("fwht128"), or null / "" for a natural trunk */
    int32_t dtype;               /* 0: F32, 1: BF16 (round to nearest even) */
} R97hostAdapterConfig;

/* Writes dir/adapter_config.json and dir/adapter_model.safetensors (dir created if missing) for nparams
 * parameters named `<module>.lora_A` / `.lora_B` with [rows, cols] shapes (2 int64 each), their f32
 * values concatenated in that order in `values` -- host memory, or device memory (values_on_device,
 * copied on `stream`). 0 on success, 1 with a message in r97host_adapter_error. */
int r97host_adapter_write(const char* dir, const R97hostAdapterConfig* cfg, int32_t nparams, const char* const* names,
                          const int64_t* shapes, const float* values, int32_t values_on_device, void* stream);
/* Reads an adapter directory into host `values` laid out as the named parameters in order (each must be in
 * the file with its shape, and the file must hold no others), with the config's rank and alpha and the
 * file's dtype (0 F32, 1 BF16; bf16 widened exactly). 0 on success, 1 with a message. */
int r97host_adapter_read(const char* dir, int32_t nparams, const char* const* names, const int64_t* shapes,
                         float* values, int64_t* rank, double* alpha, int32_t* dtype);
const char* r97host_adapter_error(void);

/* ---- the token-budget batcher of the training loop (include/r97/batcher.h:1-102, src/batcher.cpp) ----
 * Plans each epoch from the sequences' token counts and (seed, epoch) exactly as the reference's
 * r97::Batcher does -- the same sub-batches of the same sequences in the same order, step for step -- so a
 * position saved by either resumes on the other. Sequences are named by their input index. */
/* A batcher over n sequences of lengths[i] tokens; sequences over token_budget are skipped. Null, with the
 * reason in r97host_batcher_error, for a budget <= 0 or devices < 1 (the reference's invalid_argument). */
void* r97host_batcher_create(const int64_t* lengths, int64_t n, int64_t token_budget, int32_t devices,
                             uint64_t seed);
void r97host_batcher_destroy(void* batcher);
/* The step at the position (Batcher::next): counts[d] = sequences of sub-batch d (devices entries at most),
 * indices = their input indices, sub-batch after sub-batch. Returns the sub-batch count and advances; 0 at
 * the epoch's end (the position stays there); -1 when cap cannot hold the step (nothing consumed). */
int32_t r97host_batcher_next(void* batcher, int64_t* counts, int64_t* indices, int64_t cap);
int64_t r97host_batcher_steps_in_epoch(void* batcher, int64_t epoch);
void r97host_batcher_position(void* batcher, int64_t* epoch, int64_t* step);
/* Batcher::seek: a negative epoch is the first, the step is clamped into [0, steps_in_epoch]. */
void r97host_batcher_seek(void* batcher, int64_t epoch, int64_t step);
void r97host_batcher_reset(void* batcher);
/* The skipped input indices in input order (the first cap written to out); returns how many there are. */
int64_t r97host_batcher_skipped(void* batcher, int64_t* out, int64_t cap);
int64_t r97host_batcher_skipped_tokens(void* batcher);
const char* r97host_batcher_error(void);

/* ---- chat JSONL to token ids with an assistant loss mask (include/r97/chatdata.h, src/chatdata.cpp) ----
 * The reference's ChatData: a conversation is kept through its last assistant turn, trailing assistant turns
 * are dropped until its render fits max_tokens (none left: skipped), and each kept assistant turn scores the
 * tokens from the end of its generation prompt to its last control token. The renderer (chat template and
 * tokenizer) is the container's in the reference (radiance, not in this tree); this library ships the
 * ChatML renderer over a byte vocabulary (ids 0-255 the bytes, 256 <|im_start|>, 257 <|im_end|>, both
 * control tokens) that the reference's mask test states its expectations in. */
void* r97host_chatdata_create_chatml_bytes(void);
void r97host_chatdata_destroy(void* chatdata);
/* Reads a JSONL document of len bytes ({"messages": [{"role", "content"}, ...]} a line), appending the kept
 * sequences and adding {conversations, kept, shortened, skipped, tokens, scored} into stats[6]. 1, or 0 with
 * "line N: <why>" in r97host_chatdata_error (the lines before it kept). */
int32_t r97host_chatdata_read(void* chatdata, const char* text, int64_t len, int32_t max_tokens, int64_t* stats);
int32_t r97host_chatdata_read_file(void* chatdata, const char* path, int32_t max_tokens, int64_t* stats);
/* One JSONL line rendered and scored, not appended: 0 kept, 1 shortened, 2 skipped, 3 error; the first cap
 * ids and scores written, the sequence's length in *n. */
int32_t r97host_chatdata_line(void* chatdata, const char* text, int64_t len, int32_t max_tokens, int32_t* ids,
                              uint8_t* score, int64_t cap, int64_t* n);
int64_t r97host_chatdata_count(void* chatdata);
int64_t r97host_chatdata_seq_len(void* chatdata, int64_t i);
void r97host_chatdata_seq(void* chatdata, int64_t i, int32_t* ids, uint8_t* score);
const char* r97host_chatdata_error(void* chatdata);

/* ---- the training step as C++ over libr97b200.so: the reference's StepFn (include/r97/step.h:18-27; the
 * device join's make_device_step, include/r97/step_device.h:164, src/step_device.cpp:355-1678) ----
 * The LoRA step of the hybrid model (embedding, layers of 3 GatedDeltaNet : 1 gated attention each followed
 * by a SwiGLU MLP, final RMSNorm, tied IQR head with cross-entropy) forward and backward, driving this
 * library's kernels without Python. The caller owns the frozen weights (device buffers); the step owns its
 * activations (one arena sized at creation) and workspaces. */
typedef struct R97hostIqrWeight {  /* a stored projection in the trunk form (u4 codes, f32 scale per 128) */
    const void* codes;   /* uint8 [rows, cols * bits / 8] */
    const float* scale;  /* f32 [rows, cols / 128] */
    int64_t rows, cols;
    uint32_t mad_a, mad_b;
    int32_t bits, state_bits, run_rows, _pad;
} R97hostIqrWeight;

typedef struct R97hostStepConfig {
    int32_t hidden, layers, gdn_per_attn, gdn_heads, gdn_qk_heads, head_k;
    int32_t attn_heads, attn_kv_heads, attn_head_dim, rotary_dim, ffn, vocab;
    int32_t rank, seq, micro_batch, lora_mlp, head_chunk, _pad;
    float alpha, eps;
} R97hostStepConfig;

typedef struct R97hostStepWeights {
    /* every projection, layer by layer, group by group: a GDN layer's in_proj_qkvz, in_proj_ba, out_proj, an
     * attention layer's q_proj (query and gate per head), k_proj, v_proj, o_proj, then each layer's
     * gate_proj, up_proj, down_proj */
    const R97hostIqrWeight* proj;
    /* 6 per layer: w_in, w_post, then conv_w [conv_dim, 4], a_log, dt_bias, gnorm_w (GDN) or q_norm, k_norm,
     * -, - (attention); f32 */
    const float* const* norms;
    const float* w_final;
    R97hostIqrWeight head;  /* the tied head / embedding [vocab, hidden] */
    const float* rope_cos;  /* f32 [seq, rotary_dim / 2] */
    const float* rope_sin;
} R97hostStepWeights;

/* A step, or null with the reason in r97host_step_error. Runs a dry pass of the whole step to size its arena. */
void* r97host_step_create(const R97hostStepConfig* cfg, const R97hostStepWeights* w);
void r97host_step_destroy(void* step);
const char* r97host_step_error(void);
/* The flat f32 adapter: its element count, and leaf i's reference name (`<module>.lora_A` / `.lora_B`),
 * offset and [rows, cols] shape. */
int64_t r97host_step_adapter_numel(void* step);
int32_t r97host_step_param_count(void* step);
const char* r97host_step_param(void* step, int32_t i, int64_t* offset, int64_t* rows, int64_t* cols);
/* Bytes of the step's activation arena. */
int64_t r97host_step_arena_bytes(void* step);
/* One step on `stream`: ids and targets (-1: unscored) device i32 [micro_batch * seq], n_scored the number of
 * targets >= 0 (the gradient is of the mean: scale 1 / n_scored), adapter_w the flat f32 adapter (device), its
 * gradient ADDED into adapter_g (device). *loss_sum = the CE summed over the scored rows. Synchronises the
 * stream at the end. 0, or 1 with a message. */
int r97host_step_run(void* step, const int32_t* ids, const int32_t* targets, int64_t n_scored,
                     const float* adapter_w, float* adapter_g, double* loss_sum, void* stream);
/* The same step through the reference's StepFn: a Batch of n_seq sequences (lengths[s] token ids and score
 * bytes each, concatenated; at most seq tokens, padded unscored), a ParamSet of nparams leaves (names, [rows,
 * cols] shapes, f32 values concatenated) and, when grads_out is given, the ParamSet of gradients it returns,
 * written in the same layout. 0, or 1 with a message in r97host_step_error. */
int r97host_step_call(void* step, int32_t n_seq, const int64_t* lengths, const int32_t* ids, const uint8_t* score,
                      int32_t nparams, const char* const* names, const int64_t* shapes, const float* values,
                      float* grads_out, double* loss, int64_t* scored);
/* For a C++ caller with the reference's headers -- its Trainer (include/r97/trainer.h), which takes a StepFn: a
 * heap-allocated r97::StepFn over the step (cast to r97::StepFn* and copy), freed with r97host_step_fn_free.
 * A Batch may hold up to micro_batch sequences of up to seq tokens each. */
void* r97host_step_fn_new(void* step);
void r97host_step_fn_free(void* fn);

#ifdef __cplusplus
}
#endif
#endif
