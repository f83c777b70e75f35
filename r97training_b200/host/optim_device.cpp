// optim_device.cpp -- the reference's Optimiser (AdamW with warm-up + cosine schedule, global-norm
// clipping, gradient accumulation, per-name weight-decay exclusion, serialise / restore) over parameters
// that live in device memory, for the B200 step.
//
// Same contract as the reference's r97::Optimiser (include/r97/optim.h:26-90, src/optim.cpp:113-375):
// `step(grads)` adds the gradient into a private accumulation buffer; every accum_steps-th call the
// buffer's mean is clipped to clip_norm by its global norm, applied as one AdamW update with the
// scheduled learning rate, and cleared. The per-element arithmetic is the library's r97b_adamw_step and
// r97b_global_norm, bit-identical to the reference's f32 update and chunked f64 norm, so the serialised
// state after the same steps is the same bytes as the reference optimiser's -- the "R97OPT" checkpoint
// format of Optimiser::serialise, restorable by either.
//
// The parameters are one flat f32 device buffer laid out as the named parameters in order (the
// adapter's flat buffer); moments and the accumulation buffer are device buffers of the same length.
#include "r97b.h"
#include "r97host.h"

#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace r97b {
namespace {

void ok(int status, const char* what) {
    if (status != R97B_OK) throw std::runtime_error(std::string("r97host optimiser: ") + what + " failed");
}

class Device {
public:
    explicit Device(int64_t bytes) {
        if (bytes > 0) ok(r97b_mem_alloc(&p_, bytes), "device allocation");
    }
    ~Device() { r97b_mem_free(p_); }
    Device(const Device&) = delete;
    Device& operator=(const Device&) = delete;
    template <typename T> T* as() const { return static_cast<T*>(p_); }

private:
    void* p_ = nullptr;
};

// The learning rate of the `step`-th update (1-based): linear warm-up to lr over warmup_steps, then a
// half cosine from lr down to lr * lr_floor_frac at total_steps, flat after it; evaluated in double and
// rounded once, as the reference's schedule is (src/optim.cpp:113-126).
float schedule(const R97hostAdamW& c, int step) {
    if (step <= 0) return 0.0f;
    const double top = c.lr > 0.0f ? (double)c.lr : 0.0;
    if (c.warmup_steps > 0 && step <= c.warmup_steps) return (float)(top * ((double)step / (double)c.warmup_steps));
    if (c.total_steps <= 0 || c.total_steps <= c.warmup_steps) return c.lr;
    const double low = top * (c.lr_floor_frac >= 0.0f ? (double)c.lr_floor_frac : 0.0);
    const double span = (double)(c.total_steps - c.warmup_steps);
    const double done = std::min((double)(step - c.warmup_steps), span);
    const double half_turn = 3.14159265358979323846 * done / span;
    return (float)(low + (top - low) * 0.5 * (1.0 + std::cos(half_turn)));
}

template <typename T>
void put(std::vector<uint8_t>& out, T v) {
    uint8_t b[sizeof(T)];
    std::memcpy(b, &v, sizeof(T));
    out.insert(out.end(), b, b + sizeof(T));
}

template <typename T>
const uint8_t* take(const uint8_t* p, const uint8_t* end, T& v) {
    if (end - p < (ptrdiff_t)sizeof(T)) throw std::runtime_error("r97host optimiser restore: truncated");
    std::memcpy(&v, p, sizeof(T));
    return p + sizeof(T);
}

constexpr char kMagic[6] = {'R', '9', '7', 'O', 'P', 'T'};
constexpr uint16_t kVersion = 1;

class DeviceOptimiser {
public:
    DeviceOptimiser(const R97hostAdamW& cfg, std::vector<std::string> names, std::vector<int64_t> counts,
                    float* w, const std::vector<std::string>& no_decay, void* stream)
        : cfg_(cfg), names_(std::move(names)), counts_(std::move(counts)), w_(w), stream_(stream),
          n_(total(counts_)), m_(4 * n_), v_(4 * n_), acc_(4 * n_),
          partials_(r97b_global_norm_scratch_bytes(n_)), scal_(16) {
        if (names_.empty() || names_.size() != counts_.size() || !w_)
            throw std::invalid_argument("r97host optimiser: empty or mismatched parameter set");
        if (cfg_.accum_steps <= 0) throw std::invalid_argument("r97host optimiser: accum_steps must be >= 1");
        ok(r97b_memset(m_.as<void>(), 0, 4 * n_, stream_), "memset");
        ok(r97b_memset(v_.as<void>(), 0, 4 * n_, stream_), "memset");
        ok(r97b_memset(acc_.as<void>(), 0, 4 * n_, stream_), "memset");
        // contiguous runs of parameters that share the weight-decay flag: one update launch each
        int64_t off = 0;
        for (size_t i = 0; i < names_.size(); ++i) {
            bool decay = true;
            for (const auto& nd : no_decay)
                if (!nd.empty() && names_[i].find(nd) != std::string::npos) decay = false;
            if (!runs_.empty() && runs_.back().decay == decay && runs_.back().end == off)
                runs_.back().end += counts_[i];
            else
                runs_.push_back(Run{off, off + counts_[i], decay});
            off += counts_[i];
        }
    }

    // 1 when this call applied an update, 0 when it only accumulated.
    int step(const float* grad) {
        ok(r97b_add_f32(acc_.as<float>(), grad, n_, stream_), "accumulate");
        if (++pending_ < cfg_.accum_steps) return 0;
        const float inv_k = 1.0f / (float)pending_;
        const float* clip = nullptr;
        if (cfg_.clip_norm > 0.0f) {
            ok(r97b_global_norm(acc_.as<float>(), n_, inv_k, cfg_.clip_norm, partials_.as<double>(), scal_.as<float>(),
                                scal_.as<float>() + 1, stream_),
               "global norm");
            clip = scal_.as<float>() + 1;
        }
        const int t = step_ + 1;
        const float lr = schedule(cfg_, t);
        const float bc1 = 1.0f - std::pow(cfg_.beta1, (float)t);
        const float bc2 = 1.0f - std::pow(cfg_.beta2, (float)t);
        for (const Run& r : runs_) {
            const float wd = r.decay && cfg_.weight_decay != 0.0f ? cfg_.weight_decay : 0.0f;
            ok(r97b_adamw_step(w_ + r.begin, m_.as<float>() + r.begin, v_.as<float>() + r.begin,
                               acc_.as<float>() + r.begin, r.end - r.begin, lr, cfg_.beta1, cfg_.beta2, cfg_.eps, wd,
                               bc1, bc2, inv_k, clip, 1, stream_),
               "AdamW update");
        }
        step_ = t;
        pending_ = 0;
        return 1;
    }

    int updates_done() const { return step_; }
    int pending() const { return pending_; }

    std::vector<uint8_t> serialise() const {
        std::vector<uint8_t> out;
        out.reserve((size_t)(16 * n_ + 64 + 8 * names_.size()));
        out.insert(out.end(), kMagic, kMagic + 6);
        put(out, kVersion);
        put(out, (uint16_t)0);
        put(out, (int64_t)step_);
        put(out, (int32_t)pending_);
        put(out, (int32_t)names_.size());
        const float* src[4] = {w_, m_.as<float>(), v_.as<float>(), acc_.as<float>()};
        // the whole record is sized before any copy is queued: the buffer does not move under a copy
        size_t at = out.size();
        out.resize(at + 8 * names_.size() + 16 * (size_t)n_);
        ok(r97b_stream_sync(stream_), "stream sync");
        int64_t off = 0;
        for (size_t i = 0; i < names_.size(); ++i) {
            const int64_t c = counts_[i];
            const uint64_t cu = (uint64_t)c;
            std::memcpy(out.data() + at, &cu, 8);
            at += 8;
            for (int a = 0; a < 4; ++a) {
                ok(r97b_memcpy(out.data() + at, src[a] + off, 4 * c, 1, stream_), "copy to host");
                at += 4 * (size_t)c;
            }
            off += c;
        }
        ok(r97b_stream_sync(stream_), "stream sync");
        return out;
    }

    void restore(const uint8_t* p, int64_t size) {
        const uint8_t* end = p + size;
        for (int i = 0; i < 6; ++i) {
            uint8_t c;
            p = take(p, end, c);
            if (c != (uint8_t)kMagic[i]) throw std::runtime_error("r97host optimiser restore: bad magic");
        }
        uint16_t version, pad;
        p = take(p, end, version);
        p = take(p, end, pad);
        if (version != kVersion) throw std::runtime_error("r97host optimiser restore: unsupported version");
        int64_t step;
        int32_t pending, nparams;
        p = take(p, end, step);
        p = take(p, end, pending);
        p = take(p, end, nparams);
        if (step < 0 || pending < 0 || pending >= cfg_.accum_steps)
            throw std::runtime_error("r97host optimiser restore: bad step or accumulation count");
        if ((size_t)nparams != names_.size()) throw std::runtime_error("r97host optimiser restore: wrong parameter count");
        // check the whole record before touching device memory, so a throw leaves the state as it was
        const uint8_t* q = p;
        for (size_t i = 0; i < names_.size(); ++i) {
            uint64_t c;
            q = take(q, end, c);
            if ((int64_t)c != counts_[i]) throw std::runtime_error("r97host optimiser restore: wrong size for " + names_[i]);
            if (end - q < (ptrdiff_t)(16 * c)) throw std::runtime_error("r97host optimiser restore: truncated");
            q += 16 * c;
        }
        if (q != end) throw std::runtime_error("r97host optimiser restore: trailing bytes");
        float* dst[4] = {w_, m_.as<float>(), v_.as<float>(), acc_.as<float>()};
        int64_t off = 0;
        for (size_t i = 0; i < names_.size(); ++i) {
            p += 8;
            const int64_t c = counts_[i];
            for (int a = 0; a < 4; ++a) {
                ok(r97b_memcpy(dst[a] + off, p, 4 * c, 0, stream_), "copy to device");
                p += 4 * c;
            }
            off += c;
        }
        ok(r97b_stream_sync(stream_), "stream sync");
        step_ = (int)step;
        pending_ = pending;
    }

private:
    struct Run {
        int64_t begin, end;
        bool decay;
    };
    static int64_t total(const std::vector<int64_t>& c) {
        int64_t t = 0;
        for (int64_t x : c) {
            if (x < 0) throw std::invalid_argument("r97host optimiser: negative parameter size");
            t += x;
        }
        return t;
    }

    R97hostAdamW cfg_;
    std::vector<std::string> names_;
    std::vector<int64_t> counts_;
    float* w_;
    void* stream_;
    int64_t n_;
    Device m_, v_, acc_, partials_, scal_;
    std::vector<Run> runs_;
    int step_ = 0;
    int pending_ = 0;
};

thread_local std::string g_optim_error;

}  // namespace
}  // namespace r97b

using r97b::DeviceOptimiser;

extern "C" void* r97host_optim_create(const R97hostAdamW* cfg, int32_t nparams, const char* const* names,
                                      const int64_t* counts, float* w, const char* const* no_decay, int32_t n_no_decay,
                                      void* stream) {
    try {
        r97b::g_optim_error.clear();
        if (!cfg || nparams <= 0 || !names || !counts) throw std::invalid_argument("r97host optimiser: bad arguments");
        std::vector<std::string> nm(names, names + nparams);
        std::vector<int64_t> ct(counts, counts + nparams);
        std::vector<std::string> nd;
        for (int32_t i = 0; i < n_no_decay; ++i) nd.emplace_back(no_decay[i]);
        return new DeviceOptimiser(*cfg, std::move(nm), std::move(ct), w, nd, stream);
    } catch (const std::exception& e) {
        r97b::g_optim_error = e.what();
        return nullptr;
    }
}

extern "C" int r97host_optim_step(void* opt, const float* grad) {
    try {
        return static_cast<DeviceOptimiser*>(opt)->step(grad);
    } catch (const std::exception& e) {
        r97b::g_optim_error = e.what();
        return -1;
    }
}

extern "C" int r97host_optim_state(void* opt, int32_t* updates_done, int32_t* pending) {
    if (!opt) return 1;
    auto* o = static_cast<DeviceOptimiser*>(opt);
    if (updates_done) *updates_done = o->updates_done();
    if (pending) *pending = o->pending();
    return 0;
}

extern "C" int64_t r97host_optim_serialise(void* opt, uint8_t* out, int64_t cap) {
    try {
        const std::vector<uint8_t> b = static_cast<DeviceOptimiser*>(opt)->serialise();
        if (out && cap >= (int64_t)b.size()) std::memcpy(out, b.data(), b.size());
        return (int64_t)b.size();
    } catch (const std::exception& e) {
        r97b::g_optim_error = e.what();
        return -1;
    }
}

extern "C" int r97host_optim_restore(void* opt, const uint8_t* bytes, int64_t size) {
    try {
        static_cast<DeviceOptimiser*>(opt)->restore(bytes, size);
        return 0;
    } catch (const std::exception& e) {
        r97b::g_optim_error = e.what();
        return 1;
    }
}

extern "C" void r97host_optim_destroy(void* opt) { delete static_cast<DeviceOptimiser*>(opt); }

extern "C" const char* r97host_optim_error(void) { return r97b::g_optim_error.c_str(); }
