// r97b_internal.h -- declarations shared by the .cu files of libr97b200.so (not part of the ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/r97b.h"

namespace r97b {

constexpr int kEpiStoreBf16 = R97B_EPI_STORE_BF16;
constexpr int kEpiStoreF32 = R97B_EPI_STORE_F32;
constexpr int kEpiAtomicF32 = R97B_EPI_ATOMIC_F32;
constexpr int kEpiAtomicF32T = R97B_EPI_ATOMIC_F32T;
constexpr int kEpiSplitBf16 = R97B_EPI_SPLIT_BF16;
constexpr int kEpiSwiglu = R97B_EPI_SWIGLU;
constexpr int kEpiSwigluBwd = R97B_EPI_SWIGLU_BWD;

int gemm_run(const R97bGemm& g, cudaStream_t stream);
// A row-major bf16 matrix [outer, inner] (row stride `ld` elements) as a 2D TMA tensor map with a
// (box_inner, box_outer) box and the 128-byte swizzle (gemm_tc.cu).
bool make_map(CUtensorMap* map, const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_inner,
              int box_outer);
int num_sms();
// Opts kernel `fn` into at least `bytes` of dynamic shared memory on the device that is current. The
// runtime keeps this attribute per device; it is raised (never lowered) per (kernel, device), under a lock;
// returns false when the runtime refuses it (capi.cu).
bool smem_opt_in(const void* fn, int bytes);
template <typename F>
inline bool smem_opt_in(F* fn, int bytes) {
    return smem_opt_in(reinterpret_cast<const void*>(fn), bytes);
}
int64_t gemm_workspace_bytes(const R97bGemm& g);
// Each tcgen05 translation unit's error word (sm100.cuh), read and cleared.
unsigned gemm_error_word();
unsigned attn_error_word();
unsigned attn_fwd_error_word();
unsigned gdn_error_word();
unsigned loss_error_word();
unsigned gemm_i8_error_word();

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Counts this library's kernel launches (r97b_launch_count); `n` = the launches the caller just queued.
void add_launches(int n);

// Records the CUDA error behind an R97B_ELAUNCH (r97b_last_launch_error reads it).
void note_launch_error(cudaError_t e);

inline int launch_status(int n = 1) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        note_launch_error(e);
        return R97B_ELAUNCH;
    }
    add_launches(n);
    return R97B_OK;
}

}  // namespace r97b
