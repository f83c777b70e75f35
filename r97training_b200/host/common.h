// common.h -- what every device row of the plugin shares: the record's parameters and operands, the
// process-wide stream, device buffers from the scratch allocator, and the f64 <-> device conversions
// at the row's edges.
//
// The contract every row keeps (reference include/r97/adjoint.h:73-116, docs of the reference's device
// rows): operands arrive as host f64 values; the row rounds them to the dtypes its kernels read on the
// way in, runs on the device, and ADDS its results into `dc` in f64 -- it never overwrites. A row that
// cannot serve a record returns without touching `dc`, so the walk can fall back to the host row; the
// one exception is a stored weight it cannot read, which throws std::runtime_error naming the operand.
#pragma once

#include "r97_api.h"
#include "../../include/r97b.h"

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace r97b_host {

using r97::AdjointCall;
using r97::AdValue;
using r97::OpParam;
using r97::OpRecord;

// ---- parameters and operands

bool has_param(const std::vector<OpParam>& params, const char* name);
int64_t int_param(const OpRecord& rec, const char* name, int64_t fallback);
double num_param(const OpRecord& rec, const char* name, double fallback);  // int64 or a numeric string
std::string str_param(const OpRecord& rec, const char* name, const char* fallback);
int operand_pos(const OpRecord& rec, const char* name);
int64_t numel(const std::vector<int64_t>& shape);
inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// ---- the device side

// The one stream every row of this process queues on (the reference keeps one per family; a row's
// upload, launches and download are one queue's worth of work). Throws when no stream can be made.
void* row_stream();

// Throws std::runtime_error carrying `what` and the library's status when a C-ABI call failed.
void check(int status, const char* what);

// A device buffer for the duration of one row call, from the scratch allocator.
class DevBuf {
public:
    DevBuf() = default;
    explicit DevBuf(int64_t bytes);
    ~DevBuf();
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p_(o.p_), bytes_(o.bytes_) { o.p_ = nullptr; o.bytes_ = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept;
    void* get() const { return p_; }
    template <typename T> T* as() const { return static_cast<T*>(p_); }
    int64_t bytes() const { return bytes_; }
    void zero();  // on the row stream

private:
    void* p_ = nullptr;
    int64_t bytes_ = 0;
};

// f64 -> device, rounded on the host. A [rows, cols] source is laid out with row stride `ld` (>= cols,
// padding zero); a flat one takes rows = 1.
DevBuf upload_bf16(const double* src, int64_t rows, int64_t cols, int64_t ld);
DevBuf upload_f32(const double* src, int64_t rows, int64_t cols, int64_t ld);
DevBuf upload_i32(const std::vector<int32_t>& src);
DevBuf upload_bytes(const void* src, int64_t bytes);

// device -> f64, added: dst[r * cols + c] += src[r * ld + c] (f32 or bf16 source). Synchronises the
// row stream first.
void add_f32(double* dst, const DevBuf& src, int64_t rows, int64_t cols, int64_t ld);
void add_bf16(double* dst, const DevBuf& src, int64_t rows, int64_t cols, int64_t ld);

// The bf16 bits of a double, round to nearest even through f32.
uint16_t bf16_bits(double x);

// ---- the GEMM, for the rows' products: D[M, N] (f32, row stride ldo) = or += A[M, K] B[N, K]^T with
// each operand K-major (stored [rows, K]) or MN-major (stored [K, rows]), bf16, row stride ld.
struct Opnd {
    const void* ptr;
    int64_t ld;
    bool mn_major;
};
void gemm_f32(int64_t M, int64_t N, int64_t K, Opnd a, Opnd b, float* out, int64_t ldo, bool accumulate);

// ---- trainable leaves: name of a LoRA factor's gradient (reference src/adjoint/device/lora.hip:113-123)
std::string factor_grad_name(const AdjointCall& call, const char* leaf, int64_t slot);

}  // namespace r97b_host
