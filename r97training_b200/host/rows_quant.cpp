// rows_quant.cpp -- device adjoint rows of the w8a8 trunk's activation quantisers, quant_act_i8g and
// had_quant_act_i8g, on libr97b200.so's r97b_quant_act_i8g_bwd.
//
// The record (reference src/adjoint/host/quant.cpp:43-370): x bf16 [M, n] read, codes i8 [M, n] and scale
// f32 [M, ceil(n / group)] written; parameters n and group. The row takes the codes' cotangent straight
// through (zero where the clamp engaged, divided by the group's scale, rotated back by the same
// Walsh-Hadamard matrix) and adds dx into the call's f64 cotangent; the scale's cotangent is dropped. The
// mask is the f32 kernel's (|v (1 / s)| > 127), as the reference's device kernel computes it. A record the
// kernel does not serve (a rotation wider than 256 columns, the linearised `_ste` check rows) is left to the
// host row.
#include "common.h"

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

}  // namespace

// No frozen positions, as the host rows (quant.cpp registers the two ops with none).
void register_quant_rows() {
    if (!r97::adjoint_register) return;
    r97::adjoint_register("quant_act_i8g", r97::Side::device, quant_device, {}, nullptr);
    r97::adjoint_register("had_quant_act_i8g", r97::Side::device, quant_device, {}, nullptr);
}

}  // namespace r97b_host
