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

#ifdef __cplusplus
}
#endif
#endif
