// capi.cu -- library-level entry points of libr97b200.so: the ABI version, the device error word and
// the GEMM.
#include "r97b_internal.h"

#include <atomic>

namespace r97b {
namespace {
std::atomic<unsigned long long> g_launches{0};
}
void add_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }
}  // namespace r97b

extern "C" uint64_t r97b_launch_count(void) { return r97b::g_launches.load(std::memory_order_relaxed); }

extern "C" int r97b_abi_version(void) { return 1; }

extern "C" int r97b_device_error(unsigned int* out_bits) {
    unsigned bits = r97b::gemm_error_word();
    if (out_bits) *out_bits = bits;
    return cudaGetLastError() == cudaSuccess ? R97B_OK : R97B_ELAUNCH;
}

extern "C" int r97b_gemm(const R97bGemm* g, void* stream) {
    if (!g) return R97B_EINVAL;
    return r97b::gemm_run(*g, r97b::as_stream(stream));  // gemm_run counts its launch
}
