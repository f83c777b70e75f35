// capi.cu -- library-level entry points of libr97b200.so: the ABI version, the device error word, the
// GEMM, and the device memory / stream plumbing a C++ host (the adjoint-row plugin) drives kernels with.
#include "r97b_internal.h"

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

namespace r97b {
namespace {
std::atomic<unsigned long long> g_launches{0};
}
void add_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

namespace {
std::atomic<int> g_launch_error{0};
}
void note_launch_error(cudaError_t e) { g_launch_error.store((int)e, std::memory_order_relaxed); }

// The attribute is a ceiling, so it only ever rises: a kernel launched with several sizes keeps the largest
// it has been given (lowering it for a small launch would fail a later large one that found its size
// recorded).
bool smem_opt_in(const void* fn, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> ceiling;  // (kernel, device) -> bytes set
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(fn, dev);
    const auto it = ceiling.find(key);
    if (it != ceiling.end() && it->second >= bytes) return true;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
        note_launch_error(e);
        cudaGetLastError();  // not sticky: clear it so the next launch's check does not see it
        return false;
    }
    ceiling[key] = bytes;
    return true;
}
}  // namespace r97b

extern "C" uint64_t r97b_launch_count(void) { return r97b::g_launches.load(std::memory_order_relaxed); }

extern "C" int r97b_abi_version(void) { return 6; }

// The CUDA error (cudaError_t) behind the most recent R97B_ELAUNCH, and its name; 0 / "cudaSuccess" when
// none has occurred since the last read, which clears it.
extern "C" int r97b_last_launch_error(void) { return r97b::g_launch_error.exchange(0); }
extern "C" const char* r97b_launch_error_name(int code) { return cudaGetErrorName((cudaError_t)code); }

extern "C" int r97b_device_error(unsigned int* out_bits) {
    unsigned bits = r97b::gemm_error_word() | r97b::attn_error_word() | r97b::attn_fwd_error_word() |
                    r97b::gdn_error_word() | r97b::loss_error_word() | r97b::gemm_i8_error_word();
    if (out_bits) *out_bits = bits;
    return cudaGetLastError() == cudaSuccess ? R97B_OK : R97B_ELAUNCH;
}

extern "C" int r97b_gemm(const R97bGemm* g, void* stream) {
    if (!g) return R97B_EINVAL;
    return r97b::gemm_run(*g, r97b::as_stream(stream));  // gemm_run counts its launch
}

extern "C" int64_t r97b_gemm_workspace_bytes(const R97bGemm* g) {
    if (!g) return -1;
    return r97b::gemm_workspace_bytes(*g);
}

extern "C" int r97b_mem_alloc(void** out, int64_t bytes) {
    if (!out || bytes < 0) return R97B_EINVAL;
    *out = nullptr;
    if (bytes == 0) return R97B_OK;
    return cudaMalloc(out, (size_t)bytes) == cudaSuccess ? R97B_OK : R97B_EDEVICE;
}

extern "C" int r97b_mem_free(void* p) {
    if (!p) return R97B_OK;
    return cudaFree(p) == cudaSuccess ? R97B_OK : R97B_EDEVICE;
}

extern "C" int r97b_memcpy(void* dst, const void* src, int64_t bytes, int32_t kind, void* stream) {
    if (bytes < 0 || kind < 0 || kind > 2) return R97B_EINVAL;
    if (bytes == 0) return R97B_OK;
    if (!dst || !src) return R97B_EINVAL;
    static const cudaMemcpyKind kinds[3] = {cudaMemcpyHostToDevice, cudaMemcpyDeviceToHost, cudaMemcpyDeviceToDevice};
    return cudaMemcpyAsync(dst, src, (size_t)bytes, kinds[kind], r97b::as_stream(stream)) == cudaSuccess ? R97B_OK
                                                                                                         : R97B_ELAUNCH;
}

extern "C" int r97b_memset(void* dst, int32_t byte, int64_t bytes, void* stream) {
    if (bytes < 0) return R97B_EINVAL;
    if (bytes == 0) return R97B_OK;
    if (!dst) return R97B_EINVAL;
    return cudaMemsetAsync(dst, byte, (size_t)bytes, r97b::as_stream(stream)) == cudaSuccess ? R97B_OK : R97B_ELAUNCH;
}

extern "C" int r97b_stream_create(void** out) {
    if (!out) return R97B_EINVAL;
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return R97B_EDEVICE;
    *out = s;
    return R97B_OK;
}

extern "C" int r97b_stream_sync(void* stream) {
    return cudaStreamSynchronize(r97b::as_stream(stream)) == cudaSuccess ? R97B_OK : R97B_EDEVICE;
}

extern "C" const char* r97b_last_cuda_error(void) { return cudaGetErrorString(cudaPeekAtLastError()); }
