// oracle/ref_shim.cpp -- TEST INFRASTRUCTURE ONLY. A flat C ABI over the reference's own host rows.
//
// This file is compiled together with the reference's radiance-free host sources (the adjoint
// registry, the host twin/adjoint rows, loss.cpp, optim.cpp, stored_weight.cpp and the header-only
// iqr_decode.h) into oracle/_ref/libr97ref.so by oracle/Makefile. Nothing of the reference is
// copied here: the shim builds the reference's own OpRecord / AdValue / AdjointCall values from flat
// arrays, looks the op up in the reference's registry (twin_find / adjoint_find, the rows registered
// by R97_REGISTER_TWIN / R97_REGISTER_ADJOINT in src/adjoint/host/*.cpp) and runs it.
//
// Only tests/, bench.py's cpu_baseline leg and __graft_entry__.smoke() load this library, and only
// as a checker or as the timed CPU baseline; the product path never does.
#include "r97/adjoint.h"
#include "r97/batcher.h"
#include "r97/loss.h"
#include "r97/optim.h"
#include "r97/trainer.h"

#include "iqr_decode.h"
#include "stored_weight.h"

#include <algorithm>
#include <cstdint>
#include <filesystem>
#include <fstream>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

namespace {

struct RefOperand {
    const char* buffer;
    const char* dtype;
    int32_t ndim;
    const int64_t* shape;
    int32_t written;
    int32_t in_place;
    // A stored IQR weight: codes [rows, cols] int8 and scale [rows, cols/128] bf16 bits. When set,
    // the AdValue carries `raw`/`enc` instead of values, the way the device join hands a stored
    // operand to a host row (reference src/stored_weight.h).
    const int8_t* stored_codes;
    const uint16_t* stored_scale;
};

struct RefParam {
    const char* name;
    int32_t is_int;
    int64_t ival;
    const char* sval;
};

thread_local std::string g_error;
r97::ParamSet g_grads;

int64_t numel(const RefOperand& o) {
    int64_t n = 1;
    for (int i = 0; i < o.ndim; ++i) n *= o.shape[i];
    return n;
}

r97::OpRecord make_record(const char* op, const RefParam* params, int nparams,
                          const RefOperand* ops, int nops) {
    r97::OpRecord rec;
    rec.op = op;
    for (int i = 0; i < nparams; ++i) {
        if (params[i].is_int)
            rec.params.emplace_back(params[i].name, std::variant<int64_t, std::string>(params[i].ival));
        else
            rec.params.emplace_back(params[i].name,
                                    std::variant<int64_t, std::string>(std::string(params[i].sval)));
    }
    for (int i = 0; i < nops; ++i) {
        r97::Operand o;
        o.buffer = ops[i].buffer;
        o.dtype = ops[i].dtype;
        o.shape.assign(ops[i].shape, ops[i].shape + ops[i].ndim);
        o.written = ops[i].written != 0;
        o.in_place = ops[i].in_place != 0;
        rec.operands.push_back(std::move(o));
    }
    return rec;
}

// One key per stored operand: the address of a static byte is a unique encoding pointer.
unsigned char g_enc_keys[64];

r97::AdValue make_value(const RefOperand& o, const double* v, int slot) {
    r97::AdValue a;
    a.dtype = o.dtype;
    a.shape.assign(o.shape, o.shape + o.ndim);
    if (o.stored_codes) {
        const int64_t rows = o.shape[0], cols = o.shape[1];
        r97::StoredWeight w;
        w.rows = rows;
        w.cols = cols;
        w.groups = cols / 128;
        w.codes.assign(o.stored_codes, o.stored_codes + rows * cols);
        w.scale.assign(o.stored_scale, o.stored_scale + rows * (cols / 128));
        const void* key = &g_enc_keys[slot & 63];
        r97::stored_weight_put(key, std::move(w));
        a.raw = key;
        a.enc = key;
        return a;
    }
    const int64_t n = numel(o);
    if (v) a.value.assign(v, v + n);
    else a.value.assign((size_t)n, 0.0);
    return a;
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

// The reference host decode, r97_iqr_decode_host (src/iqr_decode.h), on a caller-built description.
int ref_iqr_decode(const R97IqrDecodeDesc* d) { return r97_iqr_decode_host(*d); }

// Runs the twin registered for `op`. `reads` holds one value array per READ operand in schema order
// (null for a stored operand); `outs` one array per WRITTEN operand, each sized by its shape.
int ref_twin(const char* op, const RefParam* params, int nparams, const RefOperand* ops, int nops,
             const double* const* reads, double* const* outs) {
    try {
        g_error.clear();
        r97::OpRecord rec = make_record(op, params, nparams, ops, nops);
        std::string err;
        r97::TwinFn fn = r97::twin_find(rec.op, rec.params, &err);
        if (!fn) {
            g_error = err.empty() ? "no twin" : err;
            return 1;
        }
        std::vector<r97::AdValue> operands;
        int r = 0;
        for (int i = 0; i < nops; ++i) {
            if (ops[i].written && !ops[i].in_place) continue;
            operands.push_back(make_value(ops[i], reads[r], i));
            ++r;
        }
        std::vector<r97::AdValue> out;
        fn(rec, operands, &out);
        int w = 0;
        for (int i = 0; i < nops; ++i) {
            if (!ops[i].written) continue;
            if (w >= (int)out.size()) {
                g_error = "twin produced fewer outputs than the record writes";
                r97::stored_weight_clear();
                return 2;
            }
            const int64_t n = numel(ops[i]);
            if ((int64_t)out[(size_t)w].value.size() < n) {
                g_error = "twin output smaller than its shape";
                r97::stored_weight_clear();
                return 3;
            }
            std::memcpy(outs[w], out[(size_t)w].value.data(), (size_t)n * sizeof(double));
            ++w;
        }
        r97::stored_weight_clear();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        r97::stored_weight_clear();
        return 4;
    }
}

// Runs the host adjoint registered for `op`. `fwd` holds every operand's forward value in schema
// order (null for a stored one), `cots` the cotangent of each written operand in write order, and
// `dc` one array per operand (schema order, sized by its shape) that the row adds into. Gradients
// of trainable leaves land in a ParamSet read back with ref_grad_*.
int ref_adjoint_on(const char* op, const RefParam* params, int nparams, const RefOperand* ops, int nops,
                   const double* const* fwd, const double* const* cots, double* const* dc,
                   const char* prefix, int fused_slots, int side) {
    try {
        g_error.clear();
        g_grads.clear();
        r97::OpRecord rec = make_record(op, params, nparams, ops, nops);
        std::string err;
        r97::AdjointFn fn =
            r97::adjoint_find(rec.op, side ? r97::Side::device : r97::Side::host, rec.params, &err);
        if (!fn) {
            g_error = err.empty() ? "no adjoint" : err;
            return 1;
        }
        std::vector<r97::AdValue> f, c, d;
        for (int i = 0; i < nops; ++i) f.push_back(make_value(ops[i], fwd[i], i));
        int w = 0;
        for (int i = 0; i < nops; ++i) {
            if (!ops[i].written) continue;
            RefOperand plain = ops[i];
            plain.stored_codes = nullptr;
            c.push_back(make_value(plain, cots[w], 100 + i));
            ++w;
        }
        for (int i = 0; i < nops; ++i) {
            RefOperand plain = ops[i];
            plain.stored_codes = nullptr;
            d.push_back(make_value(plain, dc[i], 200 + i));
        }
        r97::AdjointCall call{rec, f, c, &d, &g_grads, prefix};
        call.fused_slots = fused_slots != 0;
        fn(call);
        for (int i = 0; i < nops; ++i) {
            if (!dc[i]) continue;
            std::memcpy(dc[i], d[(size_t)i].value.data(), d[(size_t)i].value.size() * sizeof(double));
        }
        r97::stored_weight_clear();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        r97::stored_weight_clear();
        return 4;
    }
}

// The host rows (side 0): the reference's own f64 adjoints.
int ref_adjoint(const char* op, const RefParam* params, int nparams, const RefOperand* ops, int nops,
                const double* const* fwd, const double* const* cots, double* const* dc,
                const char* prefix, int fused_slots) {
    return ref_adjoint_on(op, params, nparams, ops, nops, fwd, cots, dc, prefix, fused_slots, 0);
}

// What the registry holds for `op` (op_rows): bit 0 twin, bit 1 host adjoint, bit 2 device adjoint; the
// frozen positions of each side into the caller's arrays (up to 16 each), their counts into *n_host /
// *n_dev.
int ref_op_rows(const char* op, int* host_frozen, int* n_host, int* dev_frozen, int* n_dev) {
    const r97::OpRows r = r97::op_rows(op);
    *n_host = (int)std::min<size_t>(16, r.host_frozen.size());
    *n_dev = (int)std::min<size_t>(16, r.device_frozen.size());
    for (int i = 0; i < *n_host; ++i) host_frozen[i] = r.host_frozen[(size_t)i];
    for (int i = 0; i < *n_dev; ++i) dev_frozen[i] = r.device_frozen[(size_t)i];
    return (r.twin ? 1 : 0) | (r.host_adjoint ? 2 : 0) | (r.device_adjoint ? 4 : 0);
}

// The ParamSet the last ref_adjoint_on call's rows added to (a device row's gradients arrive there when
// the caller flushes its device stage into it).
void* ref_paramset() { return &g_grads; }

int ref_grad_count() { return (int)g_grads.size(); }
const char* ref_grad_name(int i) { return g_grads[(size_t)i].name.c_str(); }
int64_t ref_grad_numel(int i) { return (int64_t)g_grads[(size_t)i].value.size(); }
void ref_grad_copy(int i, float* out) {
    std::memcpy(out, g_grads[(size_t)i].value.data(), g_grads[(size_t)i].value.size() * sizeof(float));
}

// The reference CE of one position (src/loss.cpp ce_position): returns the loss, writes the
// gradient row when `grad` is non-null.
double ref_ce_position(const float* row, int64_t vocab, int32_t target, float* grad, double scale) {
    return r97::ce_position(row, vocab, target, grad, scale);
}

// `steps` AdamW updates of one flat parameter through the reference Optimiser (src/optim.cpp).
// `grads` holds `steps` consecutive gradient vectors of `n` floats; `w` is updated in place.
int ref_adamw(float* w, int64_t n, const float* grads, int steps, float lr, float beta1, float beta2,
              float eps, float weight_decay, float clip_norm, int warmup, int total, int threads) {
    try {
        g_error.clear();
        r97::ParamSet params;
        params.push_back(r97::Param{"adapter", {n}, std::vector<float>(w, w + n)});
        r97::AdamWConfig cfg;
        cfg.lr = lr;
        cfg.beta1 = beta1;
        cfg.beta2 = beta2;
        cfg.eps = eps;
        cfg.weight_decay = weight_decay;
        cfg.clip_norm = clip_norm;
        cfg.warmup_steps = warmup;
        cfg.total_steps = total;
        cfg.threads = threads;
        r97::Optimiser opt(params, cfg);
        for (int s = 0; s < steps; ++s) {
            r97::ParamSet g;
            g.push_back(r97::Param{"adapter", {n},
                                   std::vector<float>(grads + (int64_t)s * n, grads + (int64_t)(s + 1) * n)});
            opt.step(g);
        }
        std::memcpy(w, params[0].value.data(), (size_t)n * sizeof(float));
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 4;
    }
}

// The reference Optimiser over named parameters (initial values `w0`, concatenated), driven by `steps`
// step() calls with the concatenated gradients in `grads`; writes its serialised state (Optimiser::serialise)
// into `out` when `cap` allows and returns the byte count (-1 on a throw). The config fields mirror
// r97::AdamWConfig; `no_decay` is a list of `n_no_decay` name substrings.
int64_t ref_optim_serialised(int nparams, const char* const* names, const int64_t* counts, const float* w0,
                             const float* grads, int steps, float lr, float beta1, float beta2, float eps,
                             float weight_decay, float clip_norm, int warmup, int total, float floor_frac,
                             int accum, const char* const* no_decay, int n_no_decay, int threads, uint8_t* out,
                             int64_t cap) {
    try {
        g_error.clear();
        r97::ParamSet params;
        int64_t total_n = 0;
        for (int i = 0; i < nparams; ++i) {
            params.push_back(r97::Param{names[i], {counts[i]}, std::vector<float>(w0 + total_n, w0 + total_n + counts[i])});
            total_n += counts[i];
        }
        r97::AdamWConfig cfg;
        cfg.lr = lr;
        cfg.beta1 = beta1;
        cfg.beta2 = beta2;
        cfg.eps = eps;
        cfg.weight_decay = weight_decay;
        cfg.clip_norm = clip_norm;
        cfg.warmup_steps = warmup;
        cfg.total_steps = total;
        cfg.lr_floor_frac = floor_frac;
        cfg.accum_steps = accum;
        cfg.threads = threads;
        for (int i = 0; i < n_no_decay; ++i) cfg.no_decay.emplace_back(no_decay[i]);
        r97::Optimiser opt(params, cfg);
        for (int s = 0; s < steps; ++s) {
            r97::ParamSet g;
            int64_t off = 0;
            for (int i = 0; i < nparams; ++i) {
                const float* src = grads + (int64_t)s * total_n + off;
                g.push_back(r97::Param{names[i], {counts[i]}, std::vector<float>(src, src + counts[i])});
                off += counts[i];
            }
            opt.step(g);
        }
        const std::vector<uint8_t> b = opt.serialise();
        if (out && cap >= (int64_t)b.size()) std::memcpy(out, b.data(), b.size());
        return (int64_t)b.size();
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    }
}

float ref_scheduled_lr(float lr, int warmup, int total, float floor_frac, int step) {
    r97::AdamWConfig cfg;
    cfg.lr = lr;
    cfg.warmup_steps = warmup;
    cfg.total_steps = total;
    cfg.lr_floor_frac = floor_frac;
    return r97::scheduled_lr(cfg, step);
}

// The reference Batcher's plans of epochs [epoch0, epoch0 + epochs) over sequences of the given token counts
// (src/batcher.cpp), flattened into `out`: per epoch the step count, then per step the sub-batch count and
// per sub-batch its size and the input indices of its sequences; then the skipped indices' count and the
// indices. Each sequence carries its own index (in its ids, or in its score bytes when it has no tokens).
// Returns the number of int64 values (-1 on a throw, message in ref_last_error); writes them when cap allows.
int64_t ref_batcher_plan(const int64_t* lengths, int64_t n, int64_t budget, int devices, uint64_t seed,
                         int64_t epoch0, int epochs, int64_t* out, int64_t cap) {
    try {
        g_error.clear();
        std::vector<r97::TokenSeq> seqs((size_t)n);
        for (int64_t i = 0; i < n; ++i) {
            seqs[(size_t)i].ids.assign((size_t)lengths[i], (int32_t)i);
            if (lengths[i] == 0) {
                seqs[(size_t)i].score.resize(4);
                std::memcpy(seqs[(size_t)i].score.data(), &i, 4);
            }
        }
        r97::BatcherConfig cfg;
        cfg.token_budget = budget;
        cfg.devices = devices;
        cfg.seed = seed;
        r97::Batcher b(std::move(seqs), cfg);
        std::vector<int64_t> flat;
        auto index_of = [](const r97::TokenSeq& t) -> int64_t {
            if (!t.ids.empty()) return t.ids[0];
            int32_t i = 0;
            std::memcpy(&i, t.score.data(), 4);
            return i;
        };
        for (int64_t e = epoch0; e < epoch0 + epochs; ++e) {
            b.seek({e, 0});
            flat.push_back(b.steps_in_epoch(e));
            std::vector<r97::Batch> step;
            while (b.next(&step)) {
                flat.push_back((int64_t)step.size());
                for (const auto& sub : step) {
                    flat.push_back((int64_t)sub.size());
                    for (const auto& t : sub) flat.push_back(index_of(t));
                }
            }
        }
        flat.push_back((int64_t)b.skipped().size());
        for (size_t i : b.skipped()) flat.push_back((int64_t)i);
        if (out && cap >= (int64_t)flat.size()) std::memcpy(out, flat.data(), flat.size() * sizeof(int64_t));
        return (int64_t)flat.size();
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    }
}

}  // extern "C"

// The reference's own training loop (src/trainer.cpp: Trainer, its Optimiser, Batcher, checkpoint and resume)
// over a StepFn it is handed -- `stepfn` points at an r97::StepFn, e.g. the B200 step's from libr97host.so
// (r97host_step_fn_new). The parameters are `nparams` named leaves ([rows, cols] shapes, f32 values in and
// out); the data `nseq` sequences of `lengths[i]` token ids, every token but the first scored. Resumes from
// `resume_dir` when it is non-empty, runs `count` steps of a run of `total_steps` (checkpointing at its end),
// writes the losses of the steps it ran (StepResult.loss / scored) into `losses` and the last checkpoint's
// directory into `ckpt_out`. Returns the steps run, or -1 on a throw (message in ref_last_error).
extern "C" int64_t ref_trainer_run(void* stepfn, int nparams, const char* const* names, const int64_t* shapes, float* values,
                        int64_t nseq, const int64_t* lengths, const int32_t* ids, int64_t token_budget, double lr,
                        int64_t total_steps, int64_t count, const char* out_dir, const char* resume_dir,
                        double* losses, char* ckpt_out, int64_t ckpt_cap) {
    try {
        g_error.clear();
        r97::ParamSet params;
        int64_t off = 0;
        for (int i = 0; i < nparams; ++i) {
            const int64_t n = shapes[2 * i] * shapes[2 * i + 1];
            params.push_back(r97::Param{names[i], {shapes[2 * i], shapes[2 * i + 1]},
                                        std::vector<float>(values + off, values + off + n)});
            off += n;
        }
        std::vector<r97::TokenSeq> seqs((size_t)nseq);
        int64_t at = 0;
        for (int64_t s = 0; s < nseq; ++s) {
            seqs[(size_t)s].ids.assign(ids + at, ids + at + lengths[s]);
            seqs[(size_t)s].score.assign((size_t)lengths[s], 1);
            seqs[(size_t)s].score[0] = 0;
            at += lengths[s];
        }
        r97::Config cfg;
        cfg.out = out_dir;
        cfg.lr = lr;
        cfg.token_budget = token_budget;
        cfg.accumulation = 1;
        cfg.steps = total_steps;
        cfg.seed = 7;
        cfg.base_id = "synthetic-hybrid";
        r97::BatcherConfig bc;
        bc.token_budget = token_budget;
        bc.devices = 1;
        bc.seed = 11;
        r97::Batcher batcher(std::move(seqs), bc);
        r97::Optimiser opt(params, r97::optimiser_config(cfg));
        std::vector<double> seen;
        const r97::StepFn inner = *static_cast<const r97::StepFn*>(stepfn);
        r97::StepFn recording = [&](const r97::Batch& b, const r97::ParamSet& p, r97::ParamSet* g) {
            const r97::StepResult r = inner(b, p, g);
            seen.push_back(r.scored > 0 ? r.loss / (double)r.scored : 0.0);
            return r;
        };
        r97::TrainerOptions topt;
        topt.config = cfg;
        topt.write_adapter = [](const r97::ParamSet&, const std::string& dir) {
            std::ofstream((std::filesystem::path(dir) / "adapter.marker").string()) << "adapter\n";
        };
        r97::Trainer trainer(recording, r97::StepFn{}, params, opt, batcher, topt);
        if (resume_dir && *resume_dir) trainer.resume(resume_dir);
        const int64_t taken = trainer.run_steps(count);
        const std::string ckpt = trainer.save_checkpoint();
        if (ckpt_out && ckpt_cap > (int64_t)ckpt.size()) std::memcpy(ckpt_out, ckpt.c_str(), ckpt.size() + 1);
        for (size_t i = 0; i < seen.size(); ++i) losses[i] = seen[i];
        off = 0;
        for (const r97::Param& p : params) {
            std::memcpy(values + off, p.value.data(), p.value.size() * sizeof(float));
            off += (int64_t)p.value.size();
        }
        return taken;
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    }
}
