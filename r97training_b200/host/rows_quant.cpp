// rows_quant.cpp -- device adjoint rows of the w8a8 trunk's activation quantisers, quant_act_i8g and
// had_quant_act_i8g, on libr97b200.so's r97b_quant_act_i8g_bwd, and of its three fused producers,
// rmsnorm_had_quant_i8g, gated_had_quant_i8g and gate_had_quant_i8g, on r97b_fused_quant_i8g_bwd.
//
// The record (reference src/adjoint/host/quant.cpp:43-370): x bf16 [M, n] read, codes i8 [M, n] and scale
// f32 [M, ceil(n / group)] written; parameters n and group. The row takes the codes' cotangent straight
// through (zero where the clamp engaged, divided by the group's scale, rotated back by the same
// Walsh-Hadamard matrix) and adds dx into the call's f64 cotangent; the scale's cotangent is dropped. The
// mask is the f32 kernel's (|v (1 / s)| > 127), as the reference's device kernel computes it. A record the
// kernel does not serve (a rotation wider than 256 columns, the linearised `_ste` check rows) is left to the
// host row.
#include "common.h"

#include <cmath>
#include <cstdlib>

namespace r97b_host {
namespace {

void quant_device(const AdjointCall& call) {
    const bool rotated = call.rec.op == "had_quant_act_i8g";
    if (!rotated && call.rec.op != "quant_act_i8g") return;
    size_t reads = 0;
    for (const auto& o : call.rec.operands) reads += !o.written;
    if (reads != 1 || call.fwd.size() < 3 || call.cot.empty() || !call.dc || call.dc->empty()) return;
    const AdValue& x = call.fwd[0];
    const AdValue& scale = call.fwd[2];
    const AdValue& g = call.cot[0];
    const int64_t n = int_param(call.rec, "n", 0), group = int_param(call.rec, "group", 0);
    if (n <= 0 || x.value.empty() || (int64_t)x.value.size() % n || g.value.size() != x.value.size()) return;
    if (rotated && (group <= 0 || group > 256 || (group & (group - 1)) || n % group)) return;
    const int64_t rows = (int64_t)x.value.size() / n;
    const int64_t t = (rotated || (group > 0 && group <= n)) ? group : n;
    const int64_t ngrp = (n + t - 1) / t;
    if ((int64_t)scale.value.size() != rows * ngrp) return;
    AdValue& dx = call.dc->at(0);
    if (dx.value.size() != x.value.size()) return;
    const int64_t ld = (n + 7) / 8 * 8;  // 16-byte rows for the vector layout
    DevBuf xd = upload_bf16(x.value.data(), rows, n, ld);
    DevBuf sd = upload_f32(scale.value.data(), rows, ngrp, ngrp);
    DevBuf gd = upload_f32(g.value.data(), rows, n, ld);
    DevBuf out(rows * ld * 4);
    check(r97b_quant_act_i8g_bwd(xd.as<uint16_t>(), ld, rows, n, group, rotated ? 1 : 0, sd.as<float>(),
                                 gd.as<float>(), ld, out.as<float>(), ld, 0, row_stream()),
          "quant_act_i8g_bwd");
    add_f32(dx.value.data(), out, rows, n, ld);
}

// ------------------------------------------------------------------------------ the fused producers
// The records (reference src/adjoint/host/quant.cpp:821-1100; tests/host/adjoint_quant.cpp:724-760): the reads
// first (rmsnorm: x bf16 [rows, n], its gain w f32 [n]; gated: gate_up bf16 [rows, 2 n]; gate: a, b bf16
// [rows, n]), then the writes: the codes (i8, rank 2) and the scale (f32, rank 2), found by dtype and shape as
// the reference's rows find them, and optionally the part's value `out` beside them, whose cotangent joins the
// quantiser's. The widths are the codes' and the scale's (group = n / the scale's columns); the cotangents are
// taken by each write's index among the writes. A record with an in-place write is left to the host row.

// The reference's predicates (quant.cpp:112-147): n and group numeric, the group a power of two dividing n --
// here at most 256, the kernel's widest rotation -- and the gated parts' activation.
bool num_of(const std::vector<OpParam>& params, const char* name, double* out) {
    for (const OpParam& p : params) {
        if (p.first != name) continue;
        if (const int64_t* v = std::get_if<int64_t>(&p.second)) {
            *out = (double)*v;
            return true;
        }
        const std::string* s = std::get_if<std::string>(&p.second);
        if (!s || s->empty()) return false;
        char* end = nullptr;
        *out = std::strtod(s->c_str(), &end);
        return end && *end == '\0';
    }
    return false;
}
bool rotated_256(const std::vector<OpParam>& params) {
    double n = 0.0, group = 0.0;
    if (!num_of(params, "n", &n) || !num_of(params, "group", &group)) return false;
    if (n <= 0.0 || n != std::floor(n) || group <= 0.0 || group != std::floor(group) || group > 256.0) return false;
    const int64_t g = (int64_t)group;
    return (g & (g - 1)) == 0 && (int64_t)n % g == 0;
}
const std::string* act_of(const std::vector<OpParam>& params) {
    for (const OpParam& p : params)
        if (p.first == "act") return std::get_if<std::string>(&p.second);
    return nullptr;
}
bool serves_gated(const std::vector<OpParam>& params) {
    if (!rotated_256(params)) return false;
    for (const OpParam& p : params)
        if (p.first == "act") {
            const std::string* a = std::get_if<std::string>(&p.second);
            return a && *a == "silu";
        }
    return true;
}
bool serves_gate(const std::vector<OpParam>& params) {
    const std::string* a = act_of(params);
    return rotated_256(params) && a && *a == "sigmoid";
}

int64_t write_index(const OpRecord& rec, size_t j) {
    int64_t at = 0;
    for (size_t k = 0; k < rec.operands.size(); ++k) {
        if (!rec.operands[k].written) continue;
        if (k == j) return at;
        ++at;
    }
    return -1;
}

void fused_device(const AdjointCall& call, int part) {
    if (!call.dc || call.cot.empty()) return;
    const auto& opr = call.rec.operands;
    int64_t codes_at = -1, scale_at = -1, out_at = -1;
    size_t reads = 0;
    for (size_t j = 0; j < opr.size(); ++j) {
        if (opr[j].in_place) return;
        if (!opr[j].written) {
            if (j != reads) return;  // the reads come first
            ++reads;
            continue;
        }
        if (codes_at < 0 && opr[j].dtype == "i8" && opr[j].shape.size() == 2) codes_at = (int64_t)j;
        else if (scale_at < 0 && opr[j].dtype == "f32" && opr[j].shape.size() == 2) scale_at = (int64_t)j;
        else if (out_at < 0) out_at = (int64_t)j;
    }
    const size_t want_reads = part == R97B_PART_SILU_MUL ? 1 : 2;
    if (codes_at < 0 || scale_at < 0 || reads < (part == R97B_PART_RMSNORM ? 1 : want_reads) ||
        call.fwd.size() < opr.size() || call.dc->size() < reads)
        return;
    const auto& cshape = opr[(size_t)codes_at].shape;
    const auto& sshape = opr[(size_t)scale_at].shape;
    const int64_t rows = cshape[0], n = cshape[1];
    if (rows <= 0 || n <= 0 || sshape[0] != rows || sshape[1] <= 0 || n % sshape[1]) return;
    const int64_t group = n / sshape[1], ngrp = sshape[1];
    if (group > 256 || (group & (group - 1)) || n % 8) return;
    const AdValue& x = call.fwd[0];
    const int64_t xw = part == R97B_PART_SILU_MUL ? 2 * n : n;
    if ((int64_t)x.value.size() != rows * xw) return;
    const AdValue& scale = call.fwd[(size_t)scale_at];
    const int64_t cs = write_index(call.rec, (size_t)codes_at);
    if ((int64_t)scale.value.size() != rows * ngrp || cs < 0 || (size_t)cs >= call.cot.size() ||
        (int64_t)call.cot[(size_t)cs].value.size() != rows * n)
        return;
    for (double v : scale.value)
        if (!(v > 0.0)) return;  // a scale the forward cannot have written
    const AdValue* go = nullptr;
    if (out_at >= 0) {
        const int64_t os = write_index(call.rec, (size_t)out_at);
        if (os >= 0 && (size_t)os < call.cot.size() && (int64_t)call.cot[(size_t)os].value.size() == rows * n)
            go = &call.cot[(size_t)os];
    }
    const AdValue* w = nullptr;
    const AdValue* b = nullptr;
    if (part == R97B_PART_RMSNORM && reads >= 2 && (int64_t)call.fwd[1].value.size() >= n) w = &call.fwd[1];
    if (part == R97B_PART_SIGMOID_MUL) {
        b = &call.fwd[1];
        if ((int64_t)b->value.size() != rows * n) return;
    }
    const double eps = num_param(call.rec, "eps", 1e-6), wadd = num_param(call.rec, "wadd", 0.0),
                 mult = num_param(call.rec, "mult", 1.0);
    if (part == R97B_PART_RMSNORM && !w && wadd != 0.0) return;
    AdValue& dx = call.dc->at(0);
    if ((int64_t)dx.value.size() != rows * xw) return;
    if (b && (int64_t)call.dc->at(1).value.size() != rows * n) return;

    const int64_t ldx = round_up(xw, 8), ld = round_up(n, 8);
    DevBuf xd = upload_bf16(x.value.data(), rows, xw, ldx);
    DevBuf bd = b ? upload_bf16(b->value.data(), rows, n, ld) : DevBuf();
    DevBuf wd = w ? upload_f32(w->value.data(), 1, n, n) : DevBuf();
    DevBuf sd = upload_f32(scale.value.data(), rows, ngrp, ngrp);
    DevBuf gd = upload_f32(call.cot[(size_t)cs].value.data(), rows, n, ld);
    DevBuf god = go ? upload_f32(go->value.data(), rows, n, ld) : DevBuf();
    DevBuf d1(rows * ldx * 4), d2(b ? rows * ld * 4 : 0);
    check(r97b_fused_quant_i8g_bwd(part, xd.as<uint16_t>(), ldx, bd.as<uint16_t>(), ld, wd.as<float>(), (float)eps,
                                   (float)wadd, (float)mult, rows, n, group, sd.as<float>(), ngrp, gd.as<float>(), ld,
                                   god.as<float>(), ld, d1.as<float>(), ldx, d2.as<float>(), ld, 0, row_stream()),
          "fused_quant_i8g_bwd");
    add_f32(dx.value.data(), d1, rows, xw, ldx);
    if (b) add_f32(call.dc->at(1).value.data(), d2, rows, n, ld);
}

void rmsnorm_quant_device(const AdjointCall& call) { fused_device(call, R97B_PART_RMSNORM); }
void gated_quant_device(const AdjointCall& call) { fused_device(call, R97B_PART_SILU_MUL); }
void gate_quant_device(const AdjointCall& call) { fused_device(call, R97B_PART_SIGMOID_MUL); }

}  // namespace

// No frozen positions, as the host rows (quant.cpp registers the two ops with none).
void register_quant_rows() {
    if (!r97::adjoint_register) return;
    r97::adjoint_register("quant_act_i8g", r97::Side::device, quant_device, {}, nullptr);
    r97::adjoint_register("had_quant_act_i8g", r97::Side::device, quant_device, {}, nullptr);
    // the fused producers: the rmsnorm's gain frozen (quant.cpp:1528-1533; device quant.hip:959-961)
    r97::adjoint_register("rmsnorm_had_quant_i8g", r97::Side::device, rmsnorm_quant_device, {1}, rotated_256);
    r97::adjoint_register("gated_had_quant_i8g", r97::Side::device, gated_quant_device, {}, serves_gated);
    r97::adjoint_register("gate_had_quant_i8g", r97::Side::device, gate_quant_device, {}, serves_gate);
}

}  // namespace r97b_host
