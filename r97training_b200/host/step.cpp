// step.cpp -- the LoRA training step of the hybrid model as C++ over libr97b200.so, and the reference's
// StepFn over it.
//
// The reference's trainer drives a step through `StepFn = std::function<StepResult(const Batch&, const
// ParamSet&, ParamSet*)>` (include/r97/step.h:18-27), which its device join builds
// (include/r97/step_device.h:164, src/step_device.cpp:355-1678). DeviceStep is that step for the B200: the
// forward (embedding, 3 GDN : 1 gated-attention blocks with SwiGLU MLPs, final norm, tied IQR head with CE in
// row chunks) and the fixed reverse walk, calling the library's kernels through its C ABI with no torch and
// no Python. It owns its device memory: persistent buffers (decoded weights, the adapter's bf16 mirrors,
// workspaces) allocated at creation, and one arena for a step's activations with stack discipline -- the
// forward pushes each layer's saved tensors, the backward pops them layer by layer -- sized by a dry pass
// of the same code with no launches. The weights (stored IQR projections, norms, GDN parameters, the head,
// the rope tables) are the caller's device buffers; the adapter is one flat f32 buffer in the layout below.
//
// The kernels, their order, shapes, tilings and split choices are those of r97training_b200.model.TrainStep,
// so the two give the same loss and gradients (up to the float atomics of the adapter-gradient GEMMs and the
// GDN adjoint, whose summation order varies from run to run).
#include "common.h"
#include "../../include/r97b_iqr.h"
#include "../../include/r97host.h"

#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace r97b_host {
namespace {

// ------------------------------------------------------------------------------------------------ memory

// One device allocation handed out by a bump pointer, with marks to pop back to. In a dry pass it hands
// out fake addresses and only records how far it reached.
class Arena {
public:
    void reserve(int64_t bytes) {
        release_all();
        if (bytes > 0 && r97b_mem_alloc(&base_, bytes) != R97B_OK)
            throw std::runtime_error("r97b step: the activation arena (" + std::to_string(bytes) +
                                     " bytes) could not be allocated");
        cap_ = bytes;
        top_ = 0;
        peak_ = 0;
    }
    void dry() {
        release_all();
        dry_ = true;
        top_ = peak_ = 0;
    }
    void* take(int64_t bytes) {
        const int64_t at = round_up(top_, 256);
        if (!dry_ && at + bytes > cap_) throw std::runtime_error("r97b step: the activation arena is too small");
        top_ = at + bytes;
        peak_ = std::max(peak_, top_);
        return dry_ ? reinterpret_cast<void*>(uintptr_t(0x10000) + uintptr_t(at)) : static_cast<char*>(base_) + at;
    }
    int64_t mark() const { return top_; }
    void pop(int64_t m) { top_ = m; }
    int64_t peak() const { return peak_; }
    int64_t capacity() const { return cap_; }
    bool is_dry() const { return dry_; }
    ~Arena() { release_all(); }

private:
    void release_all() {
        if (base_) r97b_mem_free(base_);
        base_ = nullptr;
        cap_ = 0;
        dry_ = false;
    }
    void* base_ = nullptr;
    int64_t cap_ = 0, top_ = 0, peak_ = 0;
    bool dry_ = false;
};

// A persistent device buffer for the step's lifetime.
struct Persist {
    std::vector<void*> held;
    void* take(int64_t bytes, bool zero = false) {
        void* p = nullptr;
        if (bytes <= 0) return nullptr;
        if (r97b_mem_alloc(&p, bytes) != R97B_OK || !p)
            throw std::runtime_error("r97b step: a persistent buffer of " + std::to_string(bytes) +
                                     " bytes could not be allocated");
        held.push_back(p);
        if (zero && r97b_memset(p, 0, bytes, nullptr) != R97B_OK) throw std::runtime_error("r97b step: memset");
        return p;
    }
    ~Persist() {
        for (void* p : held) r97b_mem_free(p);
    }
};

// A 2-D bf16 view: pointer, rows, columns, row stride (elements).
struct View {
    uint16_t* p = nullptr;
    int64_t rows = 0, cols = 0, ld = 0;
    View cols_from(int64_t c0, int64_t n) const { return View{p + c0, rows, n, ld}; }
    View rows_from(int64_t r0, int64_t n) const { return View{p + r0 * ld, n, cols, ld}; }
};

struct Proj {
    std::string name;  // <module>
    int64_t n;
    R97hostIqrWeight w;
};

struct Group {
    std::string name;
    int64_t k, n = 0;
    std::vector<Proj> projs;
    bool lora = true;
    int64_t a_off = 0;             // adapter offsets (f32 elements) of A_all and each B_i
    std::vector<int64_t> b_offs;
    uint16_t* a_bf = nullptr;      // [r_all * r, k]
    uint16_t* b_blk = nullptr;     // [n, r_all * r], block-diagonal
    uint16_t* w_keep = nullptr;    // the decoded weight [n, k], kept from the forward for the backward
    int64_t r_all() const { return (int64_t)projs.size(); }
};

struct Layer {
    bool gdn;
    const float *w_in, *w_post, *conv_w, *a_log, *dt_bias, *gnorm_w, *q_norm, *k_norm;
    std::vector<Group> groups;  // mixer in/qkv, mixer out/o, gate_up, down
};

// What one layer's forward keeps for its backward.
struct Saved {
    View x, n1, y, n2, y_gu, a, on, ga;
    View t[4];
    uint16_t *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;  // GDN
    float *g = nullptr, *beta = nullptr, *A = nullptr, *w = nullptr, *S = nullptr, *Vp = nullptr, *P = nullptr;
    uint16_t *qr = nullptr, *kr = nullptr, *vt = nullptr, *attn = nullptr;  // attention
    float* lse = nullptr;
    View h1;
    int64_t mark = 0;
};

}  // namespace

class DeviceStep {
public:
    DeviceStep(const R97hostStepConfig& c, const R97hostStepWeights& w) : c_(c) {
        if (c.hidden <= 0 || c.layers <= 0 || c.gdn_per_attn < 0 || c.rank <= 0 || c.seq <= 0 || c.micro_batch <= 0 ||
            c.head_k != 128 || c.seq % 128 || c.hidden % 128 || c.ffn % 128 || c.vocab <= 0)
            throw std::runtime_error("r97b step: unsupported configuration");
        T_ = (int64_t)c.seq * c.micro_batch;
        head_chunk_ = c.head_chunk > 0 ? c.head_chunk : 2048;
        scale_ = c.alpha / (float)c.rank;
        build_layers(w);
        w_final_ = w.w_final;
        head_ = w.head;
        rope_cos_ = w.rope_cos;
        rope_sin_ = w.rope_sin;
        allocate_persistent();
        // the arena: a dry pass of the whole step finds the high-water mark
        arena_.dry();
        dry_ = true;
        run_impl(nullptr, nullptr, nullptr, nullptr);
        dry_ = false;
        arena_.reserve(arena_.peak() + (1 << 20));
    }

    int64_t adapter_numel() const { return adapter_numel_; }
    const std::vector<std::string>& names() const { return names_; }
    const std::vector<std::pair<int64_t, int64_t>>& shapes() const { return shapes_; }
    const std::vector<int64_t>& offsets() const { return offsets_; }
    int64_t tokens() const { return T_; }
    int64_t arena_bytes() const { return arena_.capacity(); }

    // One step over device ids [micro_batch * seq] and targets (-1: unscored); adapter_w f32 (device), its
    // gradient added into adapter_g (device). Returns the CE summed over scored rows; `scored` their count.
    double run(const int32_t* ids_dev, const int32_t* targets_dev, int64_t n_scored, const float* adapter_w,
               float* adapter_g, void* stream) {
        std::lock_guard<std::mutex> lock(mu_);
        stream_ = stream;
        n_scored_ = n_scored;
        arena_.pop(0);
        refresh_mirrors(adapter_w);
        run_impl(ids_dev, targets_dev, adapter_w, adapter_g);
        std::vector<float> rows((size_t)T_);
        check(r97b_memcpy(rows.data(), loss_rows_, T_ * 4, 1, stream_), "loss download");
        check(r97b_stream_sync(stream_), "step wait");
        double sum = 0.0;
        for (float v : rows) sum += (double)v;
        return sum;
    }

private:
    // -------------------------------------------------------------------- set-up
    void build_layers(const R97hostStepWeights& w) {
        const int64_t d = c_.hidden, H = c_.gdn_heads, Hg = c_.gdn_qk_heads, K = c_.head_k;
        const int64_t Dh = c_.attn_head_dim, Hq = c_.attn_heads, Hkv = c_.attn_kv_heads, F = c_.ffn;
        int64_t pi = 0, off = 0;
        const int p = c_.gdn_per_attn + 1;
        for (int li = 0; li < c_.layers; ++li) {
            Layer L{};
            L.gdn = (li % p) != p - 1;
            const float* const* nv = w.norms + (size_t)li * 6;
            L.w_in = nv[0];
            L.w_post = nv[1];
            if (L.gdn) {
                L.conv_w = nv[2];
                L.a_log = nv[3];
                L.dt_bias = nv[4];
                L.gnorm_w = nv[5];
            } else {
                L.q_norm = nv[2];
                L.k_norm = nv[3];
            }
            const std::string fam = L.gdn ? "linear_attn" : "self_attn";
            const std::string pre = "model.layers." + std::to_string(li) + ".";
            struct Spec {
                const char* g;
                int64_t k;
                std::vector<std::pair<const char*, int64_t>> projs;
                bool mlp;
            };
            std::vector<Spec> specs;
            if (L.gdn) {
                specs.push_back({"in", d, {{"in_proj_qkvz", 2 * Hg * K + 2 * H * K}, {"in_proj_ba", 2 * H}}, false});
                specs.push_back({"out", H * K, {{"out_proj", d}}, false});
            } else {
                specs.push_back({"qkv", d, {{"q_proj", 2 * Hq * Dh}, {"k_proj", Hkv * Dh}, {"v_proj", Hkv * Dh}}, false});
                specs.push_back({"o", Hq * Dh, {{"o_proj", d}}, false});
            }
            specs.push_back({"gu", d, {{"gate_proj", F}, {"up_proj", F}}, true});
            specs.push_back({"down", F, {{"down_proj", d}}, true});
            for (const Spec& s : specs) {
                Group g;
                g.name = s.g;
                g.k = s.k;
                g.lora = c_.lora_mlp || !s.mlp;
                for (const auto& pr : s.projs) {
                    Proj P;
                    P.name = pre + (s.mlp ? std::string("mlp") : fam) + "." + pr.first;
                    P.n = pr.second;
                    P.w = w.proj[pi++];
                    if (P.w.rows != P.n || P.w.cols != g.k)
                        throw std::runtime_error("r97b step: stored weight " + P.name + " has the wrong shape");
                    g.n += P.n;
                    g.projs.push_back(P);
                }
                if (g.lora) {  // the adapter's flat layout: A_all = each A_i [r, k] in order, then each B_i [n_i, r]
                    const int64_t r = c_.rank;
                    g.a_off = off;
                    for (const Proj& P : g.projs) {
                        names_.push_back(P.name + ".lora_A");
                        shapes_.emplace_back(r, g.k);
                        offsets_.push_back(off);
                        off += r * g.k;
                    }
                    for (const Proj& P : g.projs) {
                        names_.push_back(P.name + ".lora_B");
                        shapes_.emplace_back(P.n, r);
                        offsets_.push_back(off);
                        g.b_offs.push_back(off);
                        off += P.n * r;
                    }
                }
                L.groups.push_back(std::move(g));
            }
            layers_.push_back(std::move(L));
        }
        adapter_numel_ = off;
    }

    void allocate_persistent() {
        const int64_t r = c_.rank;
        int64_t units = 0;
        for (Layer& L : layers_) {
            for (Group& g : L.groups) {
                g.w_keep = static_cast<uint16_t*>(per_.take(g.n * g.k * 2));
                if (!g.lora) continue;
                g.a_bf = static_cast<uint16_t*>(per_.take(g.r_all() * r * g.k * 2));
                g.b_blk = static_cast<uint16_t*>(per_.take(g.n * g.r_all() * r * 2, /*zero=*/true));
                units += g.r_all() * r * g.k / 8 + g.n * r / 8;
            }
        }
        if (r % 8) throw std::runtime_error("r97b step: the rank must be a multiple of 8");
        cast_units_ = units;
        head_w_ = static_cast<uint16_t*>(per_.take((int64_t)c_.vocab * c_.hidden * 2));
        logits_ = static_cast<uint16_t*>(per_.take((int64_t)head_chunk_ * c_.vocab * 2));
        loss_rows_ = static_cast<float*>(per_.take(T_ * 4));
        split_ws_ = per_.take(64 << 20, /*zero=*/true);
        split_ws_bytes_ = 64 << 20;
        dx_buf_[0] = static_cast<uint16_t*>(per_.take(T_ * c_.hidden * 2));
        dx_buf_[1] = static_cast<uint16_t*>(per_.take(T_ * c_.hidden * 2));
        targets_ = static_cast<int32_t*>(per_.take(T_ * 4));
        // the GDN chunk table and the sequence table
        const int32_t n_seq = c_.micro_batch;
        std::vector<int32_t> cu((size_t)n_seq + 1);
        for (int s = 0; s <= n_seq; ++s) cu[(size_t)s] = s * c_.seq;
        const int32_t n = r97b_gdn_chunk_table(cu.data(), n_seq, 64, nullptr, nullptr, nullptr);
        if (n < 0) throw std::runtime_error("r97b step: chunk table");
        std::vector<int32_t> tok0((size_t)std::max(n, 1)), len((size_t)std::max(n, 1)), sc0((size_t)n_seq + 1);
        r97b_gdn_chunk_table(cu.data(), n_seq, 64, tok0.data(), len.data(), sc0.data());
        auto up = [&](const std::vector<int32_t>& v) {
            void* p = per_.take((int64_t)v.size() * 4);
            check(r97b_memcpy(p, v.data(), (int64_t)v.size() * 4, 0, nullptr), "table upload");
            return static_cast<int32_t*>(p);
        };
        cu_dev_ = up(cu);
        tok0_dev_ = up(tok0);
        len_dev_ = up(len);
        sc0_dev_ = up(sc0);
        n_chunks_ = n;
        check(r97b_stream_sync(nullptr), "table upload wait");
        bool any_attn = false;
        for (const Layer& L : layers_) any_attn |= !L.gdn;
        if (any_attn) {
            attn_ws_bytes_ = r97b_attn_bwd_workspace_bytes(c_.micro_batch, c_.attn_heads, c_.seq);
            attn_ws_ = per_.take(attn_ws_bytes_);
        }
    }

    // The adapter's bf16 mirrors from its f32 master: every A_all and B_i block in one launch.
    void refresh_mirrors(const float* w) {
        if (w != cast_src_) {  // the table points into the caller's buffer: built for each new one
            std::vector<R97bCastSeg> segs;
            const int64_t r = c_.rank;
            int64_t unit = 0;
            for (Layer& L : layers_)
                for (Group& g : L.groups) {
                    if (!g.lora) continue;
                    segs.push_back(R97bCastSeg{w + g.a_off, g.k, g.a_bf, g.k, g.r_all() * r, g.k, unit});
                    unit += g.r_all() * r * g.k / 8;
                    int64_t row = 0;
                    for (size_t i = 0; i < g.projs.size(); ++i) {
                        segs.push_back(R97bCastSeg{w + g.b_offs[i], r, g.b_blk + row * g.r_all() * r + (int64_t)i * r,
                                                   g.r_all() * r, g.projs[i].n, r, unit});
                        unit += g.projs[i].n * r / 8;
                        row += g.projs[i].n;
                    }
                }
            if (!cast_table_) cast_table_ = per_.take((int64_t)segs.size() * (int64_t)sizeof(R97bCastSeg));
            check(r97b_memcpy(cast_table_, segs.data(), (int64_t)(segs.size() * sizeof(R97bCastSeg)), 0, stream_),
                  "cast table upload");
            check(r97b_stream_sync(stream_), "cast table wait");
            n_segs_ = (int32_t)segs.size();
            cast_src_ = w;
        }
        if (n_segs_ > 0)
            check(r97b_cast_segments(static_cast<const R97bCastSeg*>(cast_table_), n_segs_, cast_units_, stream_),
                  "cast segments");
    }

    // -------------------------------------------------------------------- launch helpers
// K(call, what): the call runs only outside the dry pass -- the dry pass hands out fake addresses, and must
// evaluate no launch at all, so this is a macro around the call rather than a function taking its status.
#define K(call, what)               \
    do {                            \
        if (!dry_) check((call), (what)); \
    } while (0)
    uint16_t* bf(int64_t rows, int64_t cols) { return static_cast<uint16_t*>(arena_.take(rows * cols * 2)); }
    float* f32(int64_t n) { return static_cast<float*>(arena_.take(n * 4)); }
    View vbf(int64_t rows, int64_t cols) { return View{bf(rows, cols), rows, cols, cols}; }

    static R97bMat mat(const void* p, int64_t ld, bool mn) { return R97bMat{p, ld, mn ? 1 : 0, 0}; }

    struct G {
        int64_t M, N;
        R97bMat a1{}, b1{}, a2{}, b2{};
        int64_t K1 = 0, K2 = 0;
        int32_t mode = R97B_EPI_STORE_BF16, splits = 1, bn = 0;
        float alpha = 1.0f, beta = 1.0f;
        void* out = nullptr;
        int64_t ldo = 0;
        const void* addend = nullptr;
        int64_t ld_add = 0;
        void* out2 = nullptr;
        int64_t ldo2 = 0;
    };
    void gemm(const G& x) {
        R97bGemm g{};
        g.M = x.M;
        g.N = x.N;
        g.K1 = x.K1;
        g.K2 = x.K2;
        g.a1 = x.a1;
        g.b1 = x.b1;
        g.a2 = x.a2;
        g.b2 = x.b2;
        g.mode = x.mode;
        g.splits = x.splits;
        g.alpha = x.alpha;
        g.beta = x.beta;
        g.bn = x.bn;
        g.out = x.out;
        g.ldo = x.ldo;
        g.addend = x.addend;
        g.ld_add = x.ld_add;
        g.out2 = x.out2;
        g.ldo2 = x.ldo2;
        if (x.mode == R97B_EPI_SPLIT_BF16) {
            g.ws = split_ws_;
            g.ws_bytes = split_ws_bytes_;
        }
        K(r97b_gemm(&g, stream_), "gemm");
    }

    // (bn, splits) rules of r97training_b200.ops: skinny_tiling for the adapter's narrow products and
    // grad_tiling for its gradient GEMMs (measured on B200 at the config-5 shapes).
    static void skinny_tiling(int64_t M, int64_t N, int64_t K, int& bn, int& splits) {
        bn = N <= 64 ? 64 : 128;
        const int64_t units = ((M + 127) / 128) * ((N + bn - 1) / bn);
        splits = (units < 100 && (N <= 64 || K >= 8192)) ? 2 : 1;
    }
    static void grad_tiling(int64_t M, int64_t N, int64_t K, int& bn, int& splits) {
        const int64_t sms = 148;
        bn = N >= 128 ? 128 : 64;
        const int64_t tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
        int best = 1;
        const int64_t top = std::max<int64_t>(1, std::min<int64_t>(8, K / 1024));
        for (int64_t s = 2; s <= top; ++s) {
            const int64_t a = (tiles * s + sms - 1) / sms * best, b = (tiles * best + sms - 1) / sms * s;
            if (a < b) best = (int)s;
        }
        splits = best;
    }

    // out = s a b^T for the adapter's narrow products (t = s x A_all^T with b K-major, dt = s dY B_blk with
    // b_mn: b stored [K, N])
    void skinny(View a, const uint16_t* b, int64_t ldb, bool b_mn, View out, int64_t K) {
        int bn, splits;
        skinny_tiling(out.rows, out.cols, K, bn, splits);
        G g{out.rows, out.cols};
        g.a1 = mat(a.p, a.ld, false);
        g.b1 = mat(b, ldb, b_mn);
        g.K1 = K;
        g.alpha = scale_;
        g.bn = bn;
        g.splits = splits;
        g.mode = splits > 1 ? R97B_EPI_SPLIT_BF16 : R97B_EPI_STORE_BF16;
        g.out = out.p;
        g.ldo = out.ld;
        gemm(g);
    }

    void decode_group(Group& grp) {
        int64_t row = 0;
        for (const Proj& P : grp.projs) {
            R97IqrDecodeDesc d{};
            d.rows_all = P.w.rows;
            d.cols = P.w.cols;
            d.row0 = 0;
            d.rows = P.w.rows;
            d.bits = P.w.bits;
            d.state_bits = P.w.state_bits;
            d.run_rows = P.w.run_rows;
            d.rb = 1;
            d.mad = 1;
            d.round_mad = 0;
            d.mad_a = P.w.mad_a;
            d.mad_b = P.w.mad_b;
            d.codes = static_cast<const uint8_t*>(P.w.codes);
            d.codes_row_bytes = P.w.cols * P.w.bits / 8;
            d.scale = reinterpret_cast<const uint8_t*>(P.w.scale);
            d.scale_dtype = 0;  // f32
            d.scale_block_cols = 128;
            d.scale_row_bytes = P.w.cols / 128 * 4;
            K(r97b_iqr_dequant_bf16(&d, grp.w_keep + row * grp.k, grp.k, stream_), "iqr dequant");
            row += P.n;
        }
    }

    // t = s x A_all^T ; out = x W^T + t B_blk^T (+ addend). Returns t. With swiglu_out the epilogue writes
    // silu(g) u there.
    View lin_fwd(Group& g, View x, View out, const uint16_t* addend, int64_t ld_add, View* swiglu_out) {
        const int64_t M = x.rows;
        G m{M, g.n};
        m.a1 = mat(x.p, x.ld, false);
        m.b1 = mat(g.w_keep, g.k, false);
        m.K1 = g.k;
        m.out = out.p;
        m.ldo = out.ld;
        if (swiglu_out) {
            m.mode = R97B_EPI_SWIGLU;
            m.out2 = swiglu_out->p;
            m.ldo2 = swiglu_out->ld;
        } else {
            m.addend = addend;
            m.ld_add = ld_add;
            m.beta = 1.0f;
        }
        View t{};
        if (g.lora) {
            const int64_t ra = g.r_all() * c_.rank;
            t = vbf(M, ra);
            skinny(x, g.a_bf, g.k, false, t, g.k);
            m.a2 = mat(t.p, t.ld, false);
            m.b2 = mat(g.b_blk, ra, false);
            m.K2 = ra;
        }
        gemm(m);
        return t;
    }

    // dt = s dY B_blk ; dX = dY W + dt A_all ; dA_all += dt^T x ; dB_i += dY_i^T t_i. With swiglu_gu (the
    // down group) dx receives SwiGLU's adjoint [dg | du].
    void lin_bwd(Group& g, View x, View t, View dy, View dx, const View* swiglu_gu, float* grad) {
        const int64_t M = dy.rows, r = c_.rank;
        G m{M, g.k};
        m.a1 = mat(dy.p, dy.ld, false);
        m.b1 = mat(g.w_keep, g.k, true);
        m.K1 = g.n;
        m.out = dx.p;
        m.ldo = dx.ld;
        if (swiglu_gu) {
            m.mode = R97B_EPI_SWIGLU_BWD;
            m.addend = swiglu_gu->p;
            m.ld_add = swiglu_gu->ld;
        }
        if (!g.lora) {
            gemm(m);
            return;
        }
        const int64_t ra = g.r_all() * r;
        View dt = vbf(M, ra);
        skinny(dy, g.b_blk, ra, true, dt, g.n);
        m.a2 = mat(dt.p, dt.ld, false);
        m.b2 = mat(g.a_bf, g.k, true);
        m.K2 = ra;
        gemm(m);
        int bn, splits;
        grad_tiling(g.k, ra, M, bn, splits);
        G ga{g.k, ra};
        ga.a1 = mat(x.p, x.ld, true);
        ga.b1 = mat(dt.p, dt.ld, true);
        ga.K1 = M;
        ga.mode = R97B_EPI_ATOMIC_F32T;
        ga.splits = splits;
        ga.bn = bn;
        ga.out = grad ? grad + g.a_off : nullptr;
        ga.ldo = g.k;
        gemm(ga);
        int64_t col = 0;
        for (size_t i = 0; i < g.projs.size(); ++i) {
            const int64_t n = g.projs[i].n;
            grad_tiling(n, r, M, bn, splits);
            G gb{n, r};
            gb.a1 = mat(dy.p + col, dy.ld, true);
            gb.b1 = mat(t.p + (int64_t)i * r, t.ld, true);
            gb.K1 = M;
            gb.mode = R97B_EPI_ATOMIC_F32;
            gb.splits = splits;
            gb.bn = bn;
            gb.out = grad ? grad + g.b_offs[i] : nullptr;
            gb.ldo = r;
            gemm(gb);
            col += n;
        }
    }

    View rmsnorm_fwd(View x, const float* w) {
        View y = vbf(x.rows, x.cols);
        K(r97b_rmsnorm_fwd(x.p, w, y.p, nullptr, x.rows, x.cols, c_.eps, 0.0f, 1.0f, stream_), "rmsnorm fwd");
        return y;
    }
    void rmsnorm_bwd(View x, const float* w, View dy, const uint16_t* addend, uint16_t* dx) {
        K(r97b_rmsnorm_bwd(x.p, w, dy.p, addend, dx, x.rows, x.cols, c_.eps, 0.0f, 1.0f, stream_), "rmsnorm bwd");
    }

    R97bGdnDims gdn_dims(int32_t flags = 0) const {
        R97bGdnDims d{};
        d.n_seq = c_.micro_batch;
        d.H = c_.gdn_heads;
        d.Hg = c_.gdn_qk_heads;
        d.n_chunks = n_chunks_;
        d.head_k = d.head_v = 128;
        d.chunk = 64;
        d.flags = flags;
        d.T = T_;
        d.scale = (float)(1.0 / std::sqrt((double)c_.head_k));  // rounded once, as the Python step passes it
        d.chunk_tok0 = tok0_dev_;
        d.chunk_len = len_dev_;
        d.seq_chunk0 = sc0_dev_;
        return d;
    }

    // -------------------------------------------------------------------- blocks
    View gdn_fwd(Layer& L, View x, Saved& s) {
        const int64_t H = c_.gdn_heads, Hg = c_.gdn_qk_heads, K = c_.head_k, T = T_;
        Group &gi = L.groups[0], &go = L.groups[1];
        const int64_t qk = Hg * K;
        s.n1 = rmsnorm_fwd(x, L.w_in);
        decode_group(gi);
        s.y = vbf(T, gi.n);
        s.t[0] = lin_fwd(gi, s.n1, s.y, nullptr, 0, nullptr);
        s.q = bf(T, qk);
        s.k = bf(T, qk);
        s.v = bf(T, H * K);
        K(r97b_conv_prep_fwd(s.y.p, s.y.ld, L.conv_w, cu_dev_, c_.micro_batch, T, (int32_t)Hg, (int32_t)H, s.q, s.k,
                             s.v, stream_),
          "conv prep fwd");
        s.g = f32(T * H);
        s.beta = f32(T * H);
        const uint16_t* ba = s.y.p + 2 * qk + 2 * H * K;
        K(r97b_gates_fwd(ba, s.y.ld, L.a_log, L.dt_bias, tok0_dev_, len_dev_, n_chunks_, (int32_t)H, s.g, s.beta,
                         stream_),
          "gates fwd");
        const int64_t nc = std::max<int32_t>(n_chunks_, 1);
        s.A = f32(T * H * 64);
        s.w = f32(T * H * 128);
        float* u = f32(T * H * 128);
        s.S = f32(nc * H * 128 * 128);
        s.Vp = f32(T * H * 128);
        s.P = f32(nc * H * 64 * 64);
        s.o = bf(T, H * K);
        R97bGdnDims dm = gdn_dims();
        R97bGdnFwd fa{s.q, s.k, s.v, s.g, s.beta, nullptr, s.A, s.w, u, s.S, s.Vp, s.P, s.o, nullptr};
        K(r97b_gdn_fwd(&dm, &fa, stream_), "gdn fwd");
        const uint16_t* z = s.y.p + 2 * qk + H * K;
        s.on = vbf(T, H * K);
        K(r97b_gated_rmsnorm_fwd(s.o, z, s.y.ld, (int32_t)H, L.gnorm_w, s.on.p, T * H, K, c_.eps, 0, stream_),
          "gated rmsnorm fwd");
        decode_group(go);
        View h1 = vbf(T, c_.hidden);
        s.t[1] = lin_fwd(go, s.on, h1, x.p, x.ld, nullptr);
        return h1;
    }

    void gdn_bwd(Layer& L, Saved& s, View dh1, uint16_t* dx_out, float* grad) {
        const int64_t H = c_.gdn_heads, Hg = c_.gdn_qk_heads, K = c_.head_k, T = T_;
        Group &gi = L.groups[0], &go = L.groups[1];
        const int64_t qk = Hg * K;
        View don = vbf(T, H * K);
        lin_bwd(go, s.on, s.t[1], dh1, don, nullptr, grad);
        View dyin = vbf(T, gi.n);
        uint16_t* dO = bf(T, H * K);
        const uint16_t* z = s.y.p + 2 * qk + H * K;
        K(r97b_gated_rmsnorm_bwd(s.o, z, s.y.ld, (int32_t)H, L.gnorm_w, don.p, dO, dyin.p + 2 * qk + H * K, T * H, K,
                                 c_.eps, 0, stream_),
          "gated rmsnorm bwd");
        const int64_t nc = std::max<int32_t>(n_chunks_, 1);
        float* dS = f32(nc * H * 128 * 128);
        float* dVp = f32(T * H * 128);
        float* dw = f32(T * H * 128);
        float* dq = f32(T * H * 128);
        float* dk = f32(T * H * 128);
        float* dv = f32(T * H * 128);
        float* dbeta = f32(T * H);
        float* dg = f32(T * H);
        R97bGdnDims dm = gdn_dims();
        R97bGdnBwd ba{};
        ba.q = s.q;
        ba.k = s.k;
        ba.v = s.v;
        ba.g = s.g;
        ba.beta = s.beta;
        ba.A = s.A;
        ba.w = s.w;
        ba.S = s.S;
        ba.Vp = s.Vp;
        ba.P = s.P;
        ba.dO = dO;
        ba.dS = dS;
        ba.dVp = dVp;
        ba.dw = dw;
        ba.dq = dq;
        ba.dk = dk;
        ba.dv = dv;
        ba.dbeta = dbeta;
        ba.dg = dg;
        K(r97b_gdn_bwd(&dm, &ba, stream_), "gdn bwd");
        // dq, dk per value head: the conv adjoint sums each key head's value heads as it reads them
        K(r97b_conv_prep_bwd(s.y.p, s.y.ld, L.conv_w, cu_dev_, c_.micro_batch, T, (int32_t)Hg, (int32_t)H, dq, dk, dv,
                             (int32_t)H, dyin.p, dyin.ld, stream_),
          "conv prep bwd");
        const uint16_t* bap = s.y.p + 2 * qk + 2 * H * K;
        K(r97b_gates_bwd(bap, s.y.ld, L.a_log, L.dt_bias, tok0_dev_, len_dev_, n_chunks_, (int32_t)H, dg, dbeta,
                         dyin.p + 2 * qk + 2 * H * K, dyin.ld, stream_),
          "gates bwd");
        View dn1 = vbf(T, c_.hidden);
        lin_bwd(gi, s.n1, s.t[0], dyin, dn1, nullptr, grad);
        rmsnorm_bwd(s.x, L.w_in, dn1, dh1.p, dx_out);
    }

    View attn_fwd(Layer& L, View x, Saved& s) {
        const int64_t T = T_, S = c_.seq, B = c_.micro_batch;
        const int64_t Hq = c_.attn_heads, Hkv = c_.attn_kv_heads, Dh = c_.attn_head_dim;
        Group &gq = L.groups[0], &go = L.groups[1];
        s.n1 = rmsnorm_fwd(x, L.w_in);
        decode_group(gq);
        s.y = vbf(T, gq.n);
        s.t[0] = lin_fwd(gq, s.n1, s.y, nullptr, 0, nullptr);
        const int64_t qn = 2 * Hq * Dh;
        s.qr = bf(B * Hq * S, Dh);
        s.kr = bf(B * Hkv * S, Dh);
        s.vt = bf(B * Hkv * S, Dh);
        K(r97b_qk_norm_rope_fwd(s.y.p, s.y.ld, (int32_t)(2 * Dh), (int32_t)Hq, (int32_t)Dh, L.q_norm, rope_cos_,
                                rope_sin_, c_.rotary_dim, T, (int32_t)S, c_.eps, s.qr, stream_),
          "q norm rope");
        K(r97b_qk_norm_rope_fwd(s.y.p + qn, s.y.ld, (int32_t)Dh, (int32_t)Hkv, (int32_t)Dh, L.k_norm, rope_cos_,
                                rope_sin_, c_.rotary_dim, T, (int32_t)S, c_.eps, s.kr, stream_),
          "k norm rope");
        K(r97b_to_bhsd(s.y.p + qn + Hkv * Dh, s.y.ld, (int32_t)Dh, (int32_t)Hkv, (int32_t)Dh, T, (int32_t)S, s.vt, 0,
                       stream_),
          "v layout");
        s.attn = bf(B * Hq * S, Dh);
        s.lse = f32(B * Hq * S);
        R97bAttnFwd af{(int32_t)B, (int32_t)Hq, (int32_t)Hkv, (int32_t)S, (int32_t)Dh, (float)(1.0 / std::sqrt((double)Dh)),
                       s.qr, s.kr, s.vt, s.attn, s.lse};
        K(r97b_attn_fwd(&af, stream_), "attention fwd");
        s.ga = vbf(T, Hq * Dh);
        K(r97b_gate_mul_fwd(s.attn, s.y.p + Dh, s.y.ld, (int32_t)(2 * Dh), (int32_t)Hq, (int32_t)Dh, T, (int32_t)S,
                            s.ga.p, stream_),
          "gate fwd");
        decode_group(go);
        View h1 = vbf(T, c_.hidden);
        s.t[1] = lin_fwd(go, s.ga, h1, x.p, x.ld, nullptr);
        return h1;
    }

    void attn_bwd(Layer& L, Saved& s, View dh1, uint16_t* dx_out, float* grad) {
        const int64_t T = T_, S = c_.seq, B = c_.micro_batch;
        const int64_t Hq = c_.attn_heads, Hkv = c_.attn_kv_heads, Dh = c_.attn_head_dim;
        Group &gq = L.groups[0], &go = L.groups[1];
        const int64_t qn = 2 * Hq * Dh;
        View dga = vbf(T, Hq * Dh);
        lin_bwd(go, s.ga, s.t[1], dh1, dga, nullptr, grad);
        View dy = vbf(T, gq.n);
        uint16_t* dattn = bf(B * Hq * S, Dh);
        K(r97b_gate_mul_bwd(s.attn, s.y.p + Dh, s.y.ld, (int32_t)(2 * Dh), (int32_t)Hq, (int32_t)Dh, T, (int32_t)S,
                            dga.p, dattn, dy.p + Dh, dy.ld, stream_),
          "gate bwd");
        uint16_t* dq = bf(B * Hq * S, Dh);
        uint16_t* dk = bf(B * Hkv * S, Dh);
        uint16_t* dv = bf(B * Hkv * S, Dh);
        R97bAttnBwd ab{(int32_t)B, (int32_t)Hq, (int32_t)Hkv, (int32_t)S, (int32_t)Dh, (float)(1.0 / std::sqrt((double)Dh)),
                       s.qr, s.kr, s.vt, s.attn, dattn, s.lse, dq, dk, dv, attn_ws_, attn_ws_bytes_};
        K(r97b_attn_bwd(&ab, stream_), "attention bwd");
        K(r97b_qk_norm_rope_bwd(s.y.p, s.y.ld, (int32_t)(2 * Dh), (int32_t)Hq, (int32_t)Dh, L.q_norm, rope_cos_,
                                rope_sin_, c_.rotary_dim, T, (int32_t)S, c_.eps, dq, dy.p, dy.ld, stream_),
          "q norm rope bwd");
        K(r97b_qk_norm_rope_bwd(s.y.p + qn, s.y.ld, (int32_t)Dh, (int32_t)Hkv, (int32_t)Dh, L.k_norm, rope_cos_,
                                rope_sin_, c_.rotary_dim, T, (int32_t)S, c_.eps, dk, dy.p + qn, dy.ld, stream_),
          "k norm rope bwd");
        K(r97b_to_bhsd(dy.p + qn + Hkv * Dh, dy.ld, (int32_t)Dh, (int32_t)Hkv, (int32_t)Dh, T, (int32_t)S, dv, 1,
                       stream_),
          "v layout bwd");
        View dn1 = vbf(T, c_.hidden);
        lin_bwd(gq, s.n1, s.t[0], dy, dn1, nullptr, grad);
        rmsnorm_bwd(s.x, L.w_in, dn1, dh1.p, dx_out);
    }

    View mlp_fwd(Layer& L, View h1, Saved& s) {
        const int64_t T = T_;
        Group &gu = L.groups[2], &gd = L.groups[3];
        s.n2 = rmsnorm_fwd(h1, L.w_post);
        decode_group(gu);
        s.y_gu = vbf(T, 2 * c_.ffn);
        s.a = vbf(T, c_.ffn);
        s.t[2] = lin_fwd(gu, s.n2, s.y_gu, nullptr, 0, &s.a);
        decode_group(gd);
        View xn = vbf(T, c_.hidden);
        s.t[3] = lin_fwd(gd, s.a, xn, h1.p, h1.ld, nullptr);
        return xn;
    }

    void mlp_bwd(Layer& L, Saved& s, View dxn, uint16_t* dh1_out, float* grad) {
        const int64_t T = T_;
        Group &gu = L.groups[2], &gd = L.groups[3];
        View dgu = vbf(T, 2 * c_.ffn);
        lin_bwd(gd, s.a, s.t[3], dxn, dgu, &s.y_gu, grad);  // SwiGLU's adjoint fused
        View dn2 = vbf(T, c_.hidden);
        lin_bwd(gu, s.n2, s.t[2], dgu, dn2, nullptr, grad);
        rmsnorm_bwd(s.h1, L.w_post, dn2, dxn.p, dh1_out);
    }

    // -------------------------------------------------------------------- the step
    void run_impl(const int32_t* ids, const int32_t* targets, const float* /*adapter_w*/, float* grad) {
        const int64_t T = T_, d = c_.hidden, V = c_.vocab;
        arena_.pop(0);
        // the tied head, decoded once for the embedding and both head products
        {
            R97IqrDecodeDesc dd{};
            dd.rows_all = head_.rows;
            dd.cols = head_.cols;
            dd.rows = head_.rows;
            dd.bits = head_.bits;
            dd.state_bits = head_.state_bits;
            dd.run_rows = head_.run_rows;
            dd.rb = 1;
            dd.mad = 1;
            dd.mad_a = head_.mad_a;
            dd.mad_b = head_.mad_b;
            dd.codes = static_cast<const uint8_t*>(head_.codes);
            dd.codes_row_bytes = head_.cols * head_.bits / 8;
            dd.scale = reinterpret_cast<const uint8_t*>(head_.scale);
            dd.scale_block_cols = 128;
            dd.scale_row_bytes = head_.cols / 128 * 4;
            K(r97b_iqr_dequant_bf16(&dd, head_w_, d, stream_), "head dequant");
        }
        View x = vbf(T, d);
        K(r97b_embed(head_w_, d, V, ids, T, d, x.p, stream_), "embed");
        std::vector<Saved> saved(layers_.size());
        for (size_t li = 0; li < layers_.size(); ++li) {
            Layer& L = layers_[li];
            Saved& s = saved[li];
            s.mark = arena_.mark();
            s.x = x;
            s.h1 = L.gdn ? gdn_fwd(L, x, s) : attn_fwd(L, x, s);
            x = mlp_fwd(L, s.h1, s);
        }
        // head: final norm, logits in chunks, CE in place, d(normed) = grad W_head
        View nf = rmsnorm_fwd(x, w_final_);
        View dnf = vbf(T, d);
        const float gscale = (float)(1.0 / (double)std::max<int64_t>(n_scored_, 1));
        for (int64_t r0 = 0; r0 < T; r0 += head_chunk_) {
            const int64_t rows = std::min<int64_t>(head_chunk_, T - r0);
            G lg{rows, V};
            lg.a1 = mat(nf.p + r0 * d, d, false);
            lg.b1 = mat(head_w_, d, false);
            lg.K1 = d;
            lg.out = logits_;
            lg.ldo = V;
            gemm(lg);
            K(r97b_ce_kld(logits_, nullptr, targets ? targets + r0 : nullptr, logits_, loss_rows_ + r0, nullptr, rows, V,
                          V, 0, gscale, 1.0f, 0.0f, stream_),
              "ce");
            G dh{rows, d};
            dh.a1 = mat(logits_, V, false);
            dh.b1 = mat(head_w_, d, true);
            dh.K1 = V;
            dh.out = dnf.p + r0 * d;
            dh.ldo = d;
            gemm(dh);
        }
        int cur = 0;
        rmsnorm_bwd(x, w_final_, dnf, nullptr, dx_buf_[cur]);
        for (size_t li = layers_.size(); li-- > 0;) {
            Layer& L = layers_[li];
            Saved& s = saved[li];
            View dx{dx_buf_[cur], T, d, d};
            View dh1{dx_buf_[cur ^ 1], T, d, d};
            mlp_bwd(L, s, dx, dh1.p, grad);
            L.gdn ? gdn_bwd(L, s, dh1, dx_buf_[cur], grad) : attn_bwd(L, s, dh1, dx_buf_[cur], grad);
            arena_.pop(s.mark);  // the layer's saved tensors and its backward's temporaries
        }
    }

    R97hostStepConfig c_;
    int64_t T_ = 0, head_chunk_ = 0;
    float scale_ = 1.0f;
    std::vector<Layer> layers_;
    const float* w_final_ = nullptr;
    R97hostIqrWeight head_{};
    const float *rope_cos_ = nullptr, *rope_sin_ = nullptr;
    std::vector<std::string> names_;
    std::vector<std::pair<int64_t, int64_t>> shapes_;
    std::vector<int64_t> offsets_;
    int64_t adapter_numel_ = 0;
    Persist per_;
    Arena arena_;
    bool dry_ = false;
    void* stream_ = nullptr;
    int64_t n_scored_ = 0;
    uint16_t* head_w_ = nullptr;
    uint16_t* logits_ = nullptr;
    float* loss_rows_ = nullptr;
    void* split_ws_ = nullptr;
    int64_t split_ws_bytes_ = 0;
    uint16_t* dx_buf_[2] = {nullptr, nullptr};
    int32_t* targets_ = nullptr;
    int32_t *cu_dev_ = nullptr, *tok0_dev_ = nullptr, *len_dev_ = nullptr, *sc0_dev_ = nullptr;
    int32_t n_chunks_ = 0;
    void* attn_ws_ = nullptr;
    int64_t attn_ws_bytes_ = 0;
    void* cast_table_ = nullptr;
    const float* cast_src_ = nullptr;
    int32_t n_segs_ = 0;
    int64_t cast_units_ = 0;
    std::mutex mu_;

    friend struct StepBinding;
};

// The reference's StepFn over a DeviceStep: the Batch's sequences become the step's token rows (each padded
// to the configured length, the padding unscored), its score masks the targets (token i scored means row
// i - 1 predicts ids[i], reference src/loss.cpp scored_rows), the ParamSet's adapter leaves the flat f32
// buffer by name, and the gradient of every leaf is added into `grads` (one entry per leaf, created when
// missing). The loss is the CE summed over the scored rows and the gradient is of the mean (scale 1 /
// scored), as the reference's CE objective defines them (src/loss.cpp CeObjective).
struct StepBinding {
    std::shared_ptr<DeviceStep> step;
    void* stream = nullptr;
    float* w_dev = nullptr;
    float* g_dev = nullptr;
    int32_t* ids_dev = nullptr;
    int32_t* tg_dev = nullptr;

    explicit StepBinding(std::shared_ptr<DeviceStep> s) : step(std::move(s)) {
        check(r97b_stream_create(&stream), "stream");
        const int64_t n = step->adapter_numel(), T = step->tokens();
        void* p = nullptr;
        check(r97b_mem_alloc(&p, n * 4), "adapter buffer");
        w_dev = static_cast<float*>(p);
        check(r97b_mem_alloc(&p, n * 4), "gradient buffer");
        g_dev = static_cast<float*>(p);
        check(r97b_mem_alloc(&p, T * 4), "ids buffer");
        ids_dev = static_cast<int32_t*>(p);
        check(r97b_mem_alloc(&p, T * 4), "targets buffer");
        tg_dev = static_cast<int32_t*>(p);
    }
    ~StepBinding() {
        r97b_mem_free(w_dev);
        r97b_mem_free(g_dev);
        r97b_mem_free(ids_dev);
        r97b_mem_free(tg_dev);
    }

    r97::StepResult operator()(const r97::Batch& batch, const r97::ParamSet& params, r97::ParamSet* grads) {
        const R97hostStepConfig& c = step->c_;
        if ((int64_t)batch.size() > c.micro_batch)  // fewer: the missing rows run unscored
            throw std::runtime_error("r97b step: the batch holds " + std::to_string(batch.size()) +
                                     " sequences, the step takes at most " + std::to_string(c.micro_batch));
        const int64_t T = step->tokens();
        std::vector<int32_t> ids((size_t)T, 0), tg((size_t)T, -1);
        int64_t scored = 0;
        for (int64_t s = 0; s < (int64_t)batch.size(); ++s) {
            const r97::TokenSeq& q = batch[(size_t)s];
            if ((int64_t)q.ids.size() > c.seq)
                throw std::runtime_error("r97b step: a sequence is longer than the step's length");
            for (size_t i = 0; i < q.ids.size(); ++i) {
                if (q.ids[i] < 0 || q.ids[i] >= c.vocab) throw std::runtime_error("r97b step: token id out of range");
                ids[(size_t)(s * c.seq) + i] = q.ids[i];
                if (i > 0 && i < q.score.size() && q.score[i] == 1) {
                    tg[(size_t)(s * c.seq) + i - 1] = q.ids[i];
                    ++scored;
                }
            }
        }
        // the adapter's leaves by name into the flat buffer
        const auto& names = step->names();
        const auto& offs = step->offsets();
        const auto& shapes = step->shapes();
        std::vector<float> w((size_t)step->adapter_numel(), 0.0f);
        for (size_t i = 0; i < names.size(); ++i) {
            const r97::Param* p = nullptr;
            for (const r97::Param& q : params)
                if (q.name == names[i]) p = &q;
            const int64_t n = shapes[i].first * shapes[i].second;
            if (!p || (int64_t)p->value.size() != n)
                throw std::runtime_error("r97b step: the parameters have no leaf " + names[i] + " of " +
                                         std::to_string(n) + " values");
            std::memcpy(w.data() + offs[i], p->value.data(), (size_t)n * 4);
        }
        check(r97b_memcpy(w_dev, w.data(), (int64_t)w.size() * 4, 0, stream), "adapter upload");
        check(r97b_memcpy(ids_dev, ids.data(), T * 4, 0, stream), "ids upload");
        check(r97b_memcpy(tg_dev, tg.data(), T * 4, 0, stream), "targets upload");
        check(r97b_memset(g_dev, 0, (int64_t)w.size() * 4, stream), "gradient clear");
        // the backward runs either way (grads == nullptr only skips the download)
        const double loss = step->run(ids_dev, tg_dev, scored, w_dev, g_dev, stream);
        if (grads) {
            std::vector<float> g(w.size());
            check(r97b_memcpy(g.data(), g_dev, (int64_t)g.size() * 4, 1, stream), "gradient download");
            check(r97b_stream_sync(stream), "gradient wait");
            for (size_t i = 0; i < names.size(); ++i) {
                const int64_t n = shapes[i].first * shapes[i].second;
                r97::Param* dst = nullptr;
                for (r97::Param& q : *grads)
                    if (q.name == names[i]) dst = &q;
                if (!dst) {
                    grads->push_back(r97::Param{names[i], {shapes[i].first, shapes[i].second},
                                                std::vector<float>((size_t)n, 0.0f)});
                    dst = &grads->back();
                }
                for (int64_t j = 0; j < n && j < (int64_t)dst->value.size(); ++j)
                    dst->value[(size_t)j] += g[(size_t)(offs[i] + j)];
            }
        }
        return r97::StepResult{loss, scored};
    }
};

r97::StepFn make_device_step(std::shared_ptr<DeviceStep> step) {
    auto b = std::make_shared<StepBinding>(std::move(step));
    return [b](const r97::Batch& batch, const r97::ParamSet& params, r97::ParamSet* grads) {
        return (*b)(batch, params, grads);
    };
}

}  // namespace r97b_host

// ==================================================================================== the C entry points

namespace {
thread_local std::string g_step_error;

struct StepHandle {
    std::shared_ptr<r97b_host::DeviceStep> step;
    r97::StepFn fn;
};
}  // namespace

extern "C" void* r97host_step_create(const R97hostStepConfig* cfg, const R97hostStepWeights* w) {
    try {
        g_step_error.clear();
        if (!cfg || !w || !w->proj || !w->norms || !w->w_final || !w->rope_cos || !w->rope_sin)
            throw std::runtime_error("r97b step: missing configuration or weights");
        auto h = new StepHandle;
        h->step = std::make_shared<r97b_host::DeviceStep>(*cfg, *w);
        return h;
    } catch (const std::exception& e) {
        g_step_error = e.what();
        return nullptr;
    }
}

extern "C" void r97host_step_destroy(void* step) { delete static_cast<StepHandle*>(step); }

extern "C" const char* r97host_step_error(void) { return g_step_error.c_str(); }

extern "C" int64_t r97host_step_adapter_numel(void* step) {
    return step ? static_cast<StepHandle*>(step)->step->adapter_numel() : -1;
}

extern "C" int32_t r97host_step_param_count(void* step) {
    return step ? (int32_t)static_cast<StepHandle*>(step)->step->names().size() : -1;
}

extern "C" const char* r97host_step_param(void* step, int32_t i, int64_t* offset, int64_t* rows, int64_t* cols) {
    if (!step) return nullptr;
    const auto& s = *static_cast<StepHandle*>(step)->step;
    if (i < 0 || i >= (int32_t)s.names().size()) return nullptr;
    if (offset) *offset = s.offsets()[(size_t)i];
    if (rows) *rows = s.shapes()[(size_t)i].first;
    if (cols) *cols = s.shapes()[(size_t)i].second;
    return s.names()[(size_t)i].c_str();
}

extern "C" int64_t r97host_step_arena_bytes(void* step) {
    return step ? static_cast<StepHandle*>(step)->step->arena_bytes() : -1;
}

extern "C" int r97host_step_run(void* step, const int32_t* ids, const int32_t* targets, int64_t n_scored,
                                const float* adapter_w, float* adapter_g, double* loss_sum, void* stream) {
    try {
        g_step_error.clear();
        if (!step || !ids || !targets || !adapter_w) throw std::runtime_error("r97b step: missing argument");
        const double l = static_cast<StepHandle*>(step)->step->run(ids, targets, n_scored, adapter_w, adapter_g, stream);
        if (loss_sum) *loss_sum = l;
        return 0;
    } catch (const std::exception& e) {
        g_step_error = e.what();
        return 1;
    }
}

// A heap copy of the step's r97::StepFn for a C++ caller that holds the reference's headers (its Trainer):
// cast the result to r97::StepFn*, copy it, and free it with r97host_step_fn_free.
extern "C" void* r97host_step_fn_new(void* step) {
    auto* h = static_cast<StepHandle*>(step);
    if (!h) return nullptr;
    if (!h->fn) h->fn = r97b_host::make_device_step(h->step);
    return new r97::StepFn(h->fn);
}

extern "C" void r97host_step_fn_free(void* fn) { delete static_cast<r97::StepFn*>(fn); }

extern "C" int r97host_step_call(void* step, int32_t n_seq, const int64_t* lengths, const int32_t* ids,
                                 const uint8_t* score, int32_t nparams, const char* const* names,
                                 const int64_t* shapes, const float* values, float* grads_out, double* loss,
                                 int64_t* scored) {
    try {
        g_step_error.clear();
        auto* h = static_cast<StepHandle*>(step);
        if (!h || n_seq < 0 || (nparams > 0 && (!names || !shapes || !values)))
            throw std::runtime_error("r97b step: missing argument");
        if (!h->fn) h->fn = r97b_host::make_device_step(h->step);
        r97::Batch batch((size_t)n_seq);
        int64_t at = 0;
        for (int32_t s = 0; s < n_seq; ++s) {
            batch[(size_t)s].ids.assign(ids + at, ids + at + lengths[s]);
            batch[(size_t)s].score.assign(score + at, score + at + lengths[s]);
            at += lengths[s];
        }
        r97::ParamSet params;
        int64_t off = 0;
        for (int32_t i = 0; i < nparams; ++i) {
            const int64_t n = shapes[2 * i] * shapes[2 * i + 1];
            params.push_back(r97::Param{names[i], {shapes[2 * i], shapes[2 * i + 1]},
                                        std::vector<float>(values + off, values + off + n)});
            off += n;
        }
        r97::ParamSet grads;
        const r97::StepResult r = h->fn(batch, params, grads_out ? &grads : nullptr);
        if (grads_out) {
            off = 0;
            for (int32_t i = 0; i < nparams; ++i) {
                const int64_t n = shapes[2 * i] * shapes[2 * i + 1];
                for (const r97::Param& g : grads)
                    if (g.name == names[i]) std::memcpy(grads_out + off, g.value.data(), (size_t)n * 4);
                off += n;
            }
        }
        if (loss) *loss = r.loss;
        if (scored) *scored = r.scored;
        return 0;
    } catch (const std::exception& e) {
        g_step_error = e.what();
        return 1;
    }
}
