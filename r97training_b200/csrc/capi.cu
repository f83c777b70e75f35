// capi.cu -- library-level entry points of libr97b200.so: the ABI version, the device error word and
// the GEMM.
#include "r97b_internal.h"

extern "C" int r97b_abi_version(void) { return 1; }

extern "C" int r97b_device_error(unsigned int* out_bits) {
    unsigned bits = r97b::gemm_error_word();
    if (out_bits) *out_bits = bits;
    return cudaGetLastError() == cudaSuccess ? R97B_OK : R97B_ELAUNCH;
}

extern "C" int r97b_gemm(const R97bGemm* g, void* stream) {
    if (!g) return R97B_EINVAL;
    return r97b::gemm_run(*g, r97b::as_stream(stream));
}
