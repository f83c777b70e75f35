// rows_norm.cpp -- device adjoint rows of the two norms: rmsnorm and gdn_gated_rmsnorm, on the
// warp-reduction kernels of libr97b200.so.
//
// rmsnorm follows the reference's host row (src/adjoint/host/elementwise.cpp:531-670): dx for the gain
// w (+ wadd) and the multiplier `mult`, eps from the record. gdn_gated_rmsnorm follows
// src/adjoint/host/gdn_prep.cpp:541-592: per row of `channels`, dx and dz for silu or sigmoid gates,
// eps 1e-6. The kernels write bf16 cotangents, which are added into the call's f64 ones.
#include "common.h"

namespace r97b_host {
namespace {

// The rank-1 gain of an rmsnorm record: the first read operand after x holding `n` values.
const AdValue* norm_gain(const AdjointCall& call, int64_t n) {
    const size_t count = std::min(call.fwd.size(), call.rec.operands.size());
    for (size_t j = 1; j < count; ++j) {
        if (call.rec.operands[j].written) continue;
        if ((int64_t)call.fwd[j].value.size() == n) return &call.fwd[j];
    }
    return nullptr;
}

void rmsnorm_device(const AdjointCall& call) {
    if (!call.dc || call.cot.empty() || call.fwd.empty() || call.dc->empty()) return;
    // a caller that proved a read set wants the two-way rule on non-finite rows: the host row's
    if (call.read_rows != nullptr) return;
    const AdValue& x = call.fwd[0];
    const AdValue& dy = call.cot[0];
    const int64_t n = int_param(call.rec, "n", x.shape.empty() ? 0 : x.shape.back());
    if (n <= 0 || x.value.empty() || (int64_t)x.value.size() % n != 0 || n % 8 != 0) return;
    const int64_t rows = (int64_t)x.value.size() / n;
    if (dy.value.size() != x.value.size()) return;
    AdValue& dx = call.dc->at(0);
    if (dx.value.size() != x.value.size()) return;
    const AdValue* w = norm_gain(call, n);
    const double wadd = num_param(call.rec, "wadd", 0.0);
    if (!w && wadd != 0.0) return;  // the host row refuses this record by name
    const double eps = num_param(call.rec, "eps", 1e-6), mult = num_param(call.rec, "mult", 1.0);
    DevBuf xd = upload_bf16(x.value.data(), rows, n, n);
    DevBuf dyd = upload_bf16(dy.value.data(), rows, n, n);
    DevBuf wd = w ? upload_f32(w->value.data(), 1, n, n) : DevBuf();
    DevBuf out(rows * n * 2);
    check(r97b_rmsnorm_bwd(xd.as<uint16_t>(), wd.as<float>(), dyd.as<uint16_t>(), nullptr, out.as<uint16_t>(), rows, n,
                           (float)eps, (float)wadd, (float)mult, row_stream()),
          "rmsnorm_bwd");
    add_bf16(dx.value.data(), out, rows, n, n);
}

void gated_rmsnorm_device(const AdjointCall& call) {
    if (!call.dc || call.cot.empty() || call.fwd.size() < 4 || call.dc->size() < 4) return;
    const AdValue& x = call.fwd[0];
    const AdValue& z = call.fwd[1];
    const AdValue& w = call.fwd[2];
    const AdValue& d_o = call.cot[0];
    const int64_t ch = int_param(call.rec, "channels", x.shape.empty() ? 0 : x.shape.back());
    if (ch <= 0 || ch % 8 != 0 || (int64_t)w.value.size() < ch || x.value.empty() || (int64_t)x.value.size() % ch)
        return;
    const int64_t rows = (int64_t)x.value.size() / ch;
    if (z.value.size() < x.value.size() || d_o.value.size() < x.value.size()) return;
    AdValue& dx = call.dc->at(0);
    AdValue& dz = call.dc->at(1);
    if (dx.value.size() < x.value.size() || dz.value.size() < x.value.size()) return;
    const bool sig = str_param(call.rec, "act", "silu") == "sigmoid";
    DevBuf xd = upload_bf16(x.value.data(), rows, ch, ch);
    DevBuf zd = upload_bf16(z.value.data(), rows, ch, ch);
    DevBuf wd = upload_f32(w.value.data(), 1, ch, ch);
    DevBuf dod = upload_bf16(d_o.value.data(), rows, ch, ch);
    DevBuf dxd(rows * ch * 2), dzd(rows * ch * 2);
    check(r97b_gated_rmsnorm_bwd(xd.as<uint16_t>(), zd.as<uint16_t>(), 0, 0, wd.as<float>(), dod.as<uint16_t>(),
                                 dxd.as<uint16_t>(), dzd.as<uint16_t>(), rows, ch, 1e-6f, sig ? 1 : 0, row_stream()),
          "gated_rmsnorm_bwd");
    add_bf16(dx.value.data(), dxd, rows, ch, ch);
    add_bf16(dz.value.data(), dzd, rows, ch, ch);
}

}  // namespace

// Frozen positions as the host rows' (elementwise.cpp:687, gdn_prep.cpp:597-600).
void register_norm_rows() {
    if (!r97::adjoint_register) return;
    r97::adjoint_register("rmsnorm", r97::Side::device, rmsnorm_device, {1}, nullptr);
    r97::adjoint_register("gdn_gated_rmsnorm", r97::Side::device, gated_rmsnorm_device, {2}, nullptr);
}

}  // namespace r97b_host
