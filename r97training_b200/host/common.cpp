// common.cpp -- the plugin's shared plumbing (common.h) and the device memory the rows use: the scratch
// allocator (a stream-ordered block pool with live / peak / allocation counters) and the step's gradient
// stage. The API is the reference's (src/adjoint/device/scratch.h and grad_stage.h: the calls its
// device rows allocate through); the pool behind it is this library's own.
#include "common.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <unordered_map>

namespace r97b_host {

// ------------------------------------------------------------------ parameters and operands

namespace {
const OpParam* find(const std::vector<OpParam>& params, const char* name) {
    for (const OpParam& p : params)
        if (p.first == name) return &p;
    return nullptr;
}
}  // namespace

bool has_param(const std::vector<OpParam>& params, const char* name) { return find(params, name) != nullptr; }

int64_t int_param(const OpRecord& rec, const char* name, int64_t fallback) {
    const OpParam* p = find(rec.params, name);
    if (!p) return fallback;
    if (const int64_t* v = std::get_if<int64_t>(&p->second)) return *v;
    const std::string& s = std::get<std::string>(p->second);
    char* end = nullptr;
    const long long v = std::strtoll(s.c_str(), &end, 10);
    return (end && *end == '\0' && !s.empty()) ? (int64_t)v : fallback;
}

double num_param(const OpRecord& rec, const char* name, double fallback) {
    const OpParam* p = find(rec.params, name);
    if (!p) return fallback;
    if (const int64_t* v = std::get_if<int64_t>(&p->second)) return (double)*v;
    const std::string& s = std::get<std::string>(p->second);
    char* end = nullptr;
    const double v = std::strtod(s.c_str(), &end);
    return (end && end != s.c_str()) ? v : fallback;
}

std::string str_param(const OpRecord& rec, const char* name, const char* fallback) {
    const OpParam* p = find(rec.params, name);
    if (!p) return fallback;
    if (const std::string* s = std::get_if<std::string>(&p->second)) return *s;
    return std::to_string(std::get<int64_t>(p->second));
}

int operand_pos(const OpRecord& rec, const char* name) {
    for (size_t i = 0; i < rec.operands.size(); ++i)
        if (rec.operands[i].buffer == name) return (int)i;
    return -1;
}

int64_t numel(const std::vector<int64_t>& shape) {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
}

// ------------------------------------------------------------------ device side

void check(int status, const char* what) {
    if (status == R97B_OK) return;
    throw std::runtime_error(std::string("r97b: device row: ") + what + " failed (status " +
                             std::to_string(status) + ", " + r97b_last_cuda_error() + ")");
}

void* row_stream() {
    static void* s = [] {
        void* created = nullptr;
        return r97b_stream_create(&created) == R97B_OK ? created : nullptr;
    }();
    if (!s) throw std::runtime_error("r97b: device row: no stream could be created on this device");
    return s;
}

DevBuf::DevBuf(int64_t bytes) : p_(r97::device::scratch_alloc(bytes)), bytes_(bytes) {
    if (bytes > 0 && !p_)
        throw std::runtime_error("r97b: device row: scratch allocation of " + std::to_string(bytes) +
                                 " bytes refused");
}

DevBuf::~DevBuf() { r97::device::scratch_free(p_); }

DevBuf& DevBuf::operator=(DevBuf&& o) noexcept {
    if (this != &o) {
        r97::device::scratch_free(p_);
        p_ = o.p_;
        bytes_ = o.bytes_;
        o.p_ = nullptr;
        o.bytes_ = 0;
    }
    return *this;
}

void DevBuf::zero() {
    if (p_) check(r97b_memset(p_, 0, bytes_, row_stream()), "memset");
}

uint16_t bf16_bits(double x) {
    const float f = (float)x;
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)((u >> 16) | ((u & 0xFFFFu) ? 0x40u : 0u));
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

namespace {
// Host staging is synchronous with respect to the row: each upload waits for its copy, so the host
// vector may go as soon as the call returns.
DevBuf upload_host(const void* host, int64_t bytes) {
    DevBuf d(bytes);
    if (bytes > 0) {
        check(r97b_memcpy(d.get(), host, bytes, 0, row_stream()), "upload");
        check(r97b_stream_sync(row_stream()), "upload wait");
    }
    return d;
}
}  // namespace

DevBuf upload_bf16(const double* src, int64_t rows, int64_t cols, int64_t ld) {
    std::vector<uint16_t> h((size_t)(rows * ld), 0);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) h[(size_t)(r * ld + c)] = bf16_bits(src[r * cols + c]);
    return upload_host(h.data(), (int64_t)h.size() * 2);
}

DevBuf upload_f32(const double* src, int64_t rows, int64_t cols, int64_t ld) {
    std::vector<float> h((size_t)(rows * ld), 0.0f);
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) h[(size_t)(r * ld + c)] = (float)src[r * cols + c];
    return upload_host(h.data(), (int64_t)h.size() * 4);
}

DevBuf upload_i32(const std::vector<int32_t>& src) { return upload_host(src.data(), (int64_t)src.size() * 4); }

DevBuf upload_bytes(const void* src, int64_t bytes) { return upload_host(src, bytes); }

void add_f32(double* dst, const DevBuf& src, int64_t rows, int64_t cols, int64_t ld) {
    std::vector<float> h((size_t)(rows * ld));
    check(r97b_memcpy(h.data(), src.get(), (int64_t)h.size() * 4, 1, row_stream()), "download");
    check(r97b_stream_sync(row_stream()), "download wait");
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) dst[r * cols + c] += (double)h[(size_t)(r * ld + c)];
}

void add_bf16(double* dst, const DevBuf& src, int64_t rows, int64_t cols, int64_t ld) {
    std::vector<uint16_t> h((size_t)(rows * ld));
    check(r97b_memcpy(h.data(), src.get(), (int64_t)h.size() * 2, 1, row_stream()), "download");
    check(r97b_stream_sync(row_stream()), "download wait");
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) {
            const uint32_t u = (uint32_t)h[(size_t)(r * ld + c)] << 16;
            float f;
            std::memcpy(&f, &u, 4);
            dst[r * cols + c] += (double)f;
        }
}

void gemm_f32(int64_t M, int64_t N, int64_t K, Opnd a, Opnd b, float* out, int64_t ldo, bool accumulate) {
    if (M <= 0 || N <= 0 || K <= 0) return;
    R97bGemm g{};
    g.M = M;
    g.N = N;
    g.K1 = K;
    g.K2 = 0;
    g.a1 = R97bMat{a.ptr, a.ld, a.mn_major ? 1 : 0, 0};
    g.b1 = R97bMat{b.ptr, b.ld, b.mn_major ? 1 : 0, 0};
    g.mode = accumulate ? R97B_EPI_ATOMIC_F32 : R97B_EPI_STORE_F32;
    g.splits = 1;
    g.alpha = 1.0f;
    g.beta = 0.0f;
    g.out = out;
    g.ldo = ldo;
    check(r97b_gemm(&g, row_stream()), "gemm");
}

std::string factor_grad_name(const AdjointCall& call, const char* leaf, int64_t slot) {
    const auto join = [](const char* prefix, const char* l) {
        if (!prefix || !*prefix) return std::string(l);
        return std::string(prefix) + "." + l;
    };
    if (call.fused_slots) return join(call.prefix, leaf);
    if (call.slot_prefix) return join(call.slot_prefix(slot).c_str(), leaf);
    return join(call.prefix, leaf);
}

}  // namespace r97b_host

// ====================================================================== the device memory API

namespace r97 {
namespace device {

namespace {
// The scratch allocator is a block pool rather than a ledger over raw allocations. Every row of this
// process queues on the one row stream, so a block handed back by scratch_free can serve the next
// scratch_alloc at once: the kernels that still read it are ahead of any new user in that stream's
// order. Freed blocks therefore stay with the pool (no cudaFree, which would wait for the whole
// device), sized up to a granule so near sizes share blocks, and go back to the device only when an
// allocation cannot be met or the idle total passes a cap.
class ScratchPool {
public:
    void* take(int64_t bytes) {
        const int64_t cap = granule(bytes);
        std::lock_guard<std::mutex> lock(mu_);
        void* p = reuse(cap);
        if (!p) p = fresh(cap);
        if (!p) return nullptr;
        held_[p] = Held{cap, bytes};
        counters_.live_bytes += bytes;
        counters_.peak_bytes = std::max(counters_.peak_bytes, counters_.live_bytes);
        counters_.allocations += 1;
        return p;
    }

    void give(void* p) {
        std::lock_guard<std::mutex> lock(mu_);
        auto it = held_.find(p);
        if (it == held_.end()) return;  // not one of this pool's blocks
        counters_.live_bytes -= it->second.asked;
        idle_.emplace(it->second.cap, p);
        idle_bytes_ += it->second.cap;
        held_.erase(it);
        if (idle_bytes_ > kIdleCap) shrink(kIdleCap / 2);
    }

    ScratchStats counters() {
        std::lock_guard<std::mutex> lock(mu_);
        return counters_;
    }

    void reset() {
        std::lock_guard<std::mutex> lock(mu_);
        if (!held_.empty())
            throw std::runtime_error("device scratch: reset with " + std::to_string(held_.size()) +
                                     " block(s) (" + std::to_string(counters_.live_bytes) +
                                     " bytes) still taken");
        shrink(0);
        counters_ = ScratchStats{};
    }

private:
    struct Held {
        int64_t cap;    // the block's size
        int64_t asked;  // what the caller asked for (the counters count this)
    };
    static constexpr int64_t kSmall = 1 << 20;             // below: 256-byte granules
    static constexpr int64_t kIdleCap = int64_t(1) << 30;  // idle bytes kept before blocks go back

    static int64_t granule(int64_t bytes) {
        const int64_t g = bytes < kSmall ? 256 : kSmall;
        return (bytes + g - 1) / g * g;
    }

    // The smallest idle block that fits and wastes at most half of itself.
    void* reuse(int64_t cap) {
        auto it = idle_.lower_bound(cap);
        if (it == idle_.end() || it->first > 2 * cap) return nullptr;
        void* p = it->second;
        idle_bytes_ -= it->first;
        idle_.erase(it);
        return p;
    }

    void* fresh(int64_t cap) {
        void* p = nullptr;
        if (r97b_mem_alloc(&p, cap) == R97B_OK && p) return p;
        shrink(0);  // the device may be full of idle blocks: hand them back and ask once more
        p = nullptr;
        return (r97b_mem_alloc(&p, cap) == R97B_OK) ? p : nullptr;
    }

    // Gives idle blocks back to the device, largest first, until at most `keep` idle bytes remain.
    void shrink(int64_t keep) {
        if (idle_bytes_ <= keep) return;
        r97b_stream_sync(r97b_host::row_stream());  // the last readers of an idle block may still run
        while (idle_bytes_ > keep && !idle_.empty()) {
            auto last = std::prev(idle_.end());
            idle_bytes_ -= last->first;
            r97b_mem_free(last->second);
            idle_.erase(last);
        }
    }

    std::mutex mu_;
    std::multimap<int64_t, void*> idle_;  // size -> block
    std::unordered_map<void*, Held> held_;
    int64_t idle_bytes_ = 0;
    ScratchStats counters_;
};

ScratchPool& pool() {
    static ScratchPool p;
    return p;
}

struct StageLeaf {
    std::vector<int64_t> shape;
    float* dev = nullptr;
    int64_t count = 0;
};
struct Stage {
    std::mutex mu;
    std::map<std::string, StageLeaf> leaves;  // ordered by name: the flush adds in a fixed order
    std::vector<std::string> order;           // first-ask order, the order leaves join the ParamSet
    int64_t bytes = 0;
};
Stage& stage() {
    static Stage s;
    return s;
}
}  // namespace

ScratchStats scratch_stats() { return pool().counters(); }

void scratch_reset() { pool().reset(); }

void* scratch_alloc(int64_t bytes) { return bytes > 0 ? pool().take(bytes) : nullptr; }

void scratch_free(void* p) {
    if (p) pool().give(p);
}

float* grad_stage_slot(const std::string& name, const std::vector<int64_t>& shape) {
    Stage& s = stage();
    std::lock_guard<std::mutex> lock(s.mu);
    auto it = s.leaves.find(name);
    if (it != s.leaves.end()) return it->second.dev;
    StageLeaf leaf;
    leaf.shape = shape;
    leaf.count = r97b_host::numel(shape);
    if (leaf.count <= 0) return nullptr;
    void* p = nullptr;
    if (r97b_mem_alloc(&p, leaf.count * 4) != R97B_OK || !p) return nullptr;
    if (r97b_memset(p, 0, leaf.count * 4, r97b_host::row_stream()) != R97B_OK) {
        r97b_mem_free(p);
        return nullptr;
    }
    leaf.dev = static_cast<float*>(p);
    s.bytes += leaf.count * 4;
    s.leaves.emplace(name, leaf);
    s.order.push_back(name);
    return leaf.dev;
}

int64_t grad_stage_bytes() {
    Stage& s = stage();
    std::lock_guard<std::mutex> lock(s.mu);
    return s.bytes;
}

namespace {
void release(Stage& s) {
    for (auto& kv : s.leaves) r97b_mem_free(kv.second.dev);
    s.leaves.clear();
    s.order.clear();
    s.bytes = 0;
}
}  // namespace

bool grad_stage_flush(ParamSet* grads) {
    Stage& s = stage();
    std::lock_guard<std::mutex> lock(s.mu);
    bool ok = r97b_stream_sync(r97b_host::row_stream()) == R97B_OK;
    for (const std::string& name : s.order) {
        const StageLeaf& leaf = s.leaves[name];
        std::vector<float> h((size_t)leaf.count);
        if (!ok || r97b_memcpy(h.data(), leaf.dev, leaf.count * 4, 1, r97b_host::row_stream()) != R97B_OK ||
            r97b_stream_sync(r97b_host::row_stream()) != R97B_OK) {
            ok = false;
            break;
        }
        if (!grads) continue;
        Param* dst = nullptr;
        for (Param& p : *grads)
            if (p.name == name) dst = &p;
        if (!dst) {
            grads->push_back(Param{name, leaf.shape, std::vector<float>((size_t)leaf.count, 0.0f)});
            dst = &grads->back();
        }
        const size_t n = std::min(dst->value.size(), h.size());
        for (size_t i = 0; i < n; ++i) {
            // the step's f32 total, rounded once to the bf16 grid a gradient has on the card
            const uint16_t b = r97b_host::bf16_bits((double)h[i]);
            const uint32_t u = (uint32_t)b << 16;
            float f;
            std::memcpy(&f, &u, 4);
            dst->value[i] += f;
        }
    }
    release(s);
    return ok;
}

void grad_stage_discard() {
    Stage& s = stage();
    std::lock_guard<std::mutex> lock(s.mu);
    r97b_stream_sync(r97b_host::row_stream());
    release(s);
}

}  // namespace device
}  // namespace r97
