// rows_linear.cpp -- device adjoint rows of the frozen linear and its LoRA branch: gemm_nt, gemm_nt_q (the
// int8 trunk's form at i8a8h), lora_shrink (the float-trunk form) and lora_expand / lora_expand_mm, on the
// tcgen05 GEMM of libr97b200.so.
//
// The arithmetic each row serves is the reference's host row's (src/adjoint/host/linear.cpp:193-243,
// src/adjoint/host/lora.cpp:226-523): operands are rounded to bf16 on the way in (the dtype the GEMM
// reads), products accumulate in f32, and results are added into the call's f64 cotangents. Trainable
// factors go to the step's gradient stage, as the reference's device rows send them
// (src/adjoint/device/lora.hip:125-154), under the names the host rows give them.
#include "common.h"

#include <algorithm>
#include <cmath>

namespace r97b_host {
namespace {

constexpr int64_t kPad = 8;  // bf16 elements per 16 bytes: every device row stride is a multiple

// ------------------------------------------------------------------------------------------ gemm_nt

// The weight of a gemm_nt record as a bf16 [N, ldK] device operand: the values the tape carried, or the
// stored (codes, scale) pair the join decoded for it (reference src/stored_weight.h), which is looked
// up by the operand's encoding and dequantised on the device.
DevBuf weight_operand(const AdjointCall& call, int ib, int64_t N, int64_t K, int64_t ldK) {
    const AdValue& b = call.fwd[(size_t)ib];
    if (b.raw == nullptr) {
        if ((int64_t)b.value.size() != N * K) return DevBuf();
        return upload_bf16(b.value.data(), N, K, ldK);
    }
    const r97::StoredWeight* w =
        r97::stored_weight_find ? r97::stored_weight_find(b.enc, N, K) : nullptr;
    if (w == nullptr || w->rows != N || w->cols != K || w->groups <= 0 || (int64_t)w->codes.size() != N * K ||
        (int64_t)w->scale.size() != N * w->groups)
        throw std::runtime_error("r97b: gemm_nt device row: op '" + call.rec.op + "': operand '" +
                                 call.rec.operands[(size_t)ib].buffer +
                                 "' is stored in an encoding this row cannot read (no decoded codes/scale pair "
                                 "for it in the stored-weight table)");
    DevBuf codes = upload_bytes(w->codes.data(), N * K);
    DevBuf scale = upload_bytes(w->scale.data(), N * w->groups * 2);
    DevBuf out(N * ldK * 2);
    out.zero();
    check(r97b_codes_dequant_bf16(codes.as<int8_t>(), scale.as<uint16_t>(), N, K, (K + w->groups - 1) / w->groups,
                                  out.as<uint16_t>(), ldK, row_stream()),
          "codes dequant");
    return out;
}

// dX[M, K] += dY[M, N] W[N, K] (reference linear.cpp:230-243).
void gemm_nt_device(const AdjointCall& call) {
    if (!call.dc || call.cot.empty()) return;
    const int ia = operand_pos(call.rec, "a"), ib = operand_pos(call.rec, "b");
    if (ia < 0 || ib < 0 || (size_t)ia >= call.dc->size()) return;
    const AdValue& a = call.fwd[(size_t)ia];
    const AdValue& b = call.fwd[(size_t)ib];
    const AdValue& dy = call.cot[0];
    const int64_t K = int_param(call.rec, "K", a.shape.size() >= 2 ? a.shape[1] : 0);
    const int64_t N = int_param(call.rec, "N", b.shape.size() >= 2 ? b.shape[0] : 0);
    const int64_t M = a.shape.empty() ? int_param(call.rec, "M", 0) : a.shape[0];
    AdValue& dx = (*call.dc)[(size_t)ia];
    if (M <= 0 || N <= 0 || K <= 0 || (int64_t)dy.value.size() != M * N || (int64_t)dx.value.size() != M * K) return;
    const int64_t ldN = round_up(N, kPad), ldK = round_up(K, kPad);
    DevBuf w = weight_operand(call, ib, N, K, ldK);
    if (!w.get()) return;
    DevBuf d = upload_bf16(dy.value.data(), M, N, ldN);
    DevBuf out(M * ldK * 4);
    // D[M, K] = dY[M, N] . W^T where the GEMM's B operand is W read MN-major ([N, K] = [reduction, cols])
    gemm_f32(M, K, N, Opnd{d.get(), ldN, false}, Opnd{w.get(), ldK, true}, out.as<float>(), ldK, false);
    add_f32(dx.value.data(), out, M, K, ldK);
}

// ------------------------------------------------------------------------------------------ gemm_nt_q

// The group scale of `rows` rows over `groups` K blocks as a dense [rows, groups] array, by the host rows'
// rule for reading one (reference linear.cpp:101-111 scale_at): per (row, block), per block, per row, one
// for the whole operand, or 1 when absent. An index selection only.
std::vector<double> dense_scale(const AdValue* s, int64_t rows, int64_t groups) {
    std::vector<double> out((size_t)(rows * groups), 1.0);
    if (s == nullptr || s->value.empty()) return out;
    const int64_t n = (int64_t)s->value.size();
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t g = 0; g < groups; ++g) {
            int64_t at;
            if (n == 1) at = 0;
            else if (n == rows * groups) at = r * groups + g;
            else if (n == groups) at = g;
            else if (n == rows) at = r;
            else at = std::min<int64_t>(r * groups + g, n - 1);
            out[(size_t)(r * groups + g)] = s->value[(size_t)at];
        }
    return out;
}

// The int8 trunk's linear at dtype i8a8h with the device's K block of 128 (reference
// src/adjoint/device/linear.hip:748-751 serves_i8a8h).
bool serves_i8a8h(const std::vector<OpParam>& params) {
    bool dtype = false, group = false;
    for (const OpParam& p : params) {
        if (p.first == "dtype") {
            const auto* d = std::get_if<std::string>(&p.second);
            dtype = d && *d == "i8a8h";
        } else if (p.first == "group") {
            const auto* g = std::get_if<int64_t>(&p.second);
            group = g && *g == 128;
        }
    }
    return dtype && group;
}

// dX[M, K] += s_a[m, k / 128] (dY W)[m, k], W[n, k] = b[n, k] s_b[n, k / 128] -- the cotangent in the codes'
// activation basis that the upstream quantiser consumes (reference linear.cpp:286-317 gemm_nt_q_adjoint; the
// device row linear.hip:461-665). The weight is dequantised on the device: a stored one from its decoded
// codes and bf16 scale, a values one from the tape's codes and b_scale; dY enters as bf16, the product
// accumulates in f32 and the activation's group scale is applied to it before the f64 add.
void gemm_nt_q_device(const AdjointCall& call) {
    if (!call.dc || call.cot.empty()) return;
    const int ia = operand_pos(call.rec, "a"), ib = operand_pos(call.rec, "b");
    const int ias = operand_pos(call.rec, "a_scale"), ibs = operand_pos(call.rec, "b_scale");
    if (ia < 0 || ib < 0 || (size_t)ia >= call.dc->size()) return;
    const AdValue& a = call.fwd[(size_t)ia];
    const AdValue& b = call.fwd[(size_t)ib];
    const AdValue* as = ias >= 0 ? &call.fwd[(size_t)ias] : nullptr;
    const AdValue* bs = ibs >= 0 ? &call.fwd[(size_t)ibs] : nullptr;
    const AdValue& dy = call.cot[0];
    const int64_t K = int_param(call.rec, "K", a.shape.size() >= 2 ? a.shape[1] : 0);
    const int64_t N = int_param(call.rec, "N", b.shape.size() >= 2 ? b.shape[0] : 0);
    const int64_t M = a.shape.empty() ? int_param(call.rec, "M", 0) : a.shape[0];
    const int64_t group = int_param(call.rec, "group", 128);
    AdValue& dx = (*call.dc)[(size_t)ia];
    if (M <= 0 || N <= 0 || K <= 0 || group != 128 || (int64_t)dy.value.size() != M * N ||
        (int64_t)dx.value.size() != M * K)
        return;
    const int64_t G = (K + group - 1) / group;
    const int64_t ldN = round_up(N, kPad), ldK = round_up(K, kPad);
    DevBuf w;
    if (b.raw != nullptr) {
        w = weight_operand(call, ib, N, K, ldK);
    } else {
        if ((int64_t)b.value.size() != N * K) return;
        DevBuf codes = upload_f32(b.value.data(), N, K, ldK);
        const std::vector<double> sb = dense_scale(bs, N, G);
        DevBuf sbd = upload_f32(sb.data(), N, G, G);
        w = DevBuf(N * ldK * 2);
        w.zero();
        check(r97b_group_scale(codes.as<float>(), ldK, N, K, group, sbd.as<float>(), G, w.get(), ldK, 1,
                               row_stream()),
              "weight group scale");
    }
    if (!w.get()) return;
    DevBuf d = upload_bf16(dy.value.data(), M, N, ldN);
    DevBuf out(M * ldK * 4);
    gemm_f32(M, K, N, Opnd{d.get(), ldN, false}, Opnd{w.get(), ldK, true}, out.as<float>(), ldK, false);
    const std::vector<double> sa = dense_scale(as, M, G);
    DevBuf sad = upload_f32(sa.data(), M, G, G);
    check(r97b_group_scale(out.as<float>(), ldK, M, K, group, sad.as<float>(), G, out.get(), ldK, 0, row_stream()),
          "activation group scale");
    add_f32(dx.value.data(), out, M, K, ldK);
}

// ------------------------------------------------------------------------------------------ LoRA

// The rows of the record that belong to each adapter slot; rows whose slot is outside [0, S) are base
// rows that neither op reads or writes (reference lora.cpp:9-11).
std::vector<std::vector<int64_t>> rows_by_slot(const AdValue& slot, int64_t M, int64_t S) {
    std::vector<std::vector<int64_t>> out((size_t)S);
    for (int64_t m = 0; m < M; ++m) {
        const double v = slot.value[(size_t)m];
        if (!(v >= 0.0)) continue;
        const int64_t s = (int64_t)v;
        if (s < S) out[(size_t)s].push_back(m);
    }
    return out;
}

// Gathers rows `idx` of a row-major [*, cols] f64 array, each scaled by f(col) when given.
std::vector<double> gather(const std::vector<double>& src, const std::vector<int64_t>& idx, int64_t cols,
                           const double* col_scale = nullptr) {
    std::vector<double> out((size_t)idx.size() * (size_t)cols);
    for (size_t i = 0; i < idx.size(); ++i)
        for (int64_t c = 0; c < cols; ++c)
            out[i * (size_t)cols + (size_t)c] =
                src[(size_t)(idx[i] * cols + c)] * (col_scale ? col_scale[c] : 1.0);
    return out;
}

// Whether the shrink's activation is a code stream (the coded trunk, with a real a_scale): that form is
// not this row's -- the B200 path trains over the bf16 trunk -- and the walk runs the host row for it.
bool coded_act(const std::vector<OpParam>& params) {
    for (const OpParam& p : params) {
        if (p.first != "dtype") continue;
        const auto* d = std::get_if<std::string>(&p.second);
        return d && (*d == "i8" || *d == "fp8_e4m3" || *d == "fp8_e5m2");
    }
    return false;
}

bool float_act(const std::vector<OpParam>& params) { return !coded_act(params); }

// lora_shrink (a, a_scale absent, slot, lora_a, t): dx[m] += dt[m] A_s, dA_s += dt_s^T x_s.
void lora_shrink_device(const AdjointCall& call) {
    if (!call.dc || call.cot.empty() || call.fwd.size() < 5 || call.dc->size() < 5) return;
    if (coded_act(call.rec.params)) return;
    const AdValue& x = call.fwd[0];
    const AdValue& held = call.fwd[1];
    const AdValue& slot = call.fwd[2];
    const AdValue& la = call.fwd[3];
    const AdValue& dt = call.cot[0];
    if (held.dtype != "invalid" || x.shape.size() != 2 || slot.shape.size() != 1 || la.shape.size() != 3) return;
    const int64_t M = x.shape[0], K = x.shape[1], S = la.shape[0], R = la.shape[1];
    if (M <= 0 || K <= 0 || S <= 0 || R <= 0 || la.shape[2] != K || slot.shape[0] != M) return;
    if ((int64_t)x.value.size() != M * K || (int64_t)slot.value.size() != M || (int64_t)la.value.size() != S * R * K ||
        (int64_t)dt.value.size() != M * R)
        return;
    AdValue& dx = (*call.dc)[0];
    if ((int64_t)dx.value.size() != M * K) return;
    const auto rows = rows_by_slot(slot, M, S);
    const int64_t ldK = round_up(K, kPad), ldR = round_up(R, kPad);
    // the step's accumulators, one per slot the record's rows name (reference lora.hip:125-154)
    std::vector<float*> dA((size_t)S, nullptr);
    if (call.grads) {
        const std::vector<int64_t> shape =
            call.fused_slots ? std::vector<int64_t>{S * R, K} : std::vector<int64_t>{R, K};
        for (int64_t s = 0; s < S; ++s) {
            if (rows[(size_t)s].empty()) continue;
            float* base = r97::device::grad_stage_slot(factor_grad_name(call, "lora_A", s), shape);
            if (!base) throw std::runtime_error("r97b: lora_shrink device row: the gradient stage refused lora_A");
            dA[(size_t)s] = call.fused_slots ? base + s * R * K : base;
        }
    }
    for (int64_t s = 0; s < S; ++s) {
        const std::vector<int64_t>& idx = rows[(size_t)s];
        const int64_t Ms = (int64_t)idx.size();
        if (Ms == 0) continue;
        const std::vector<double> xs = gather(x.value, idx, K), ts = gather(dt.value, idx, R);
        DevBuf xd = upload_bf16(xs.data(), Ms, K, ldK);
        DevBuf td = upload_bf16(ts.data(), Ms, R, ldR);
        DevBuf ad = upload_bf16(la.value.data() + s * R * K, R, K, ldK);
        // dx_s[Ms, K] = dt_s[Ms, R] A_s[R, K]: B operand A_s read MN-major
        DevBuf out(Ms * ldK * 4);
        gemm_f32(Ms, K, R, Opnd{td.get(), ldR, false}, Opnd{ad.get(), ldK, true}, out.as<float>(), ldK, false);
        std::vector<double> part((size_t)(Ms * K), 0.0);
        add_f32(part.data(), out, Ms, K, ldK);
        for (int64_t i = 0; i < Ms; ++i)
            for (int64_t k = 0; k < K; ++k) dx.value[(size_t)(idx[(size_t)i] * K + k)] += part[(size_t)(i * K + k)];
        // dA_s[R, K] += dt_s^T x_s: both operands read MN-major ([Ms, R] and [Ms, K])
        if (dA[(size_t)s])
            gemm_f32(R, K, Ms, Opnd{td.get(), ldR, true}, Opnd{xd.get(), ldK, true}, dA[(size_t)s], K, true);
    }
}

// lora_expand / lora_expand_mm (t, slot, lora_b, [scale], y): dt[m] += (dy[m] . scale_s) B_s,
// dB_s += (dy_s . scale_s)^T t_s, and an in-place y's old value takes dy back unchanged.
void lora_expand_device(const AdjointCall& call) {
    if (!call.dc || call.cot.empty()) return;
    const size_t n = call.fwd.size();
    if (n != 4u && n != 5u) return;
    const AdValue& t = call.fwd[0];
    const AdValue& slot = call.fwd[1];
    const AdValue& lb = call.fwd[2];
    const bool has_scale = n == 5u || !call.rec.operands[3].written;
    const AdValue* sc = has_scale ? &call.fwd[3] : nullptr;
    if (t.shape.size() != 2 || slot.shape.size() != 1 || lb.shape.size() != 3) return;
    const int64_t M = t.shape[0], R = t.shape[1], S = lb.shape[0], N = lb.shape[1];
    if (M <= 0 || N <= 0 || R <= 0 || S <= 0 || lb.shape[2] != R || slot.shape[0] != M) return;
    if ((int64_t)t.value.size() != M * R || (int64_t)slot.value.size() != M || (int64_t)lb.value.size() != S * N * R)
        return;
    if (sc && (int64_t)sc->value.size() != S * N) return;
    const AdValue& dy = call.cot[0];
    if ((int64_t)dy.value.size() != M * N || call.dc->empty()) return;
    AdValue& dt = call.dc->at(0);
    if ((int64_t)dt.value.size() != M * R) return;
    for (size_t i = 0; i < call.rec.operands.size(); ++i)
        if (call.rec.operands[i].written && call.rec.operands[i].in_place && i < call.dc->size()) {
            AdValue& d_base = call.dc->at(i);
            if (d_base.value.size() == dy.value.size())
                for (size_t e = 0; e < dy.value.size(); ++e) d_base.value[e] += dy.value[e];
        }
    const auto rows = rows_by_slot(slot, M, S);
    const int64_t ldN = round_up(N, kPad), ldR = round_up(R, kPad);
    std::vector<float*> dB((size_t)S, nullptr);
    const int64_t cols = call.fused_slots ? S * R : R;
    if (call.grads) {
        const std::vector<int64_t> shape{N, cols};
        for (int64_t s = 0; s < S; ++s) {
            if (rows[(size_t)s].empty()) continue;
            float* base = r97::device::grad_stage_slot(factor_grad_name(call, "lora_B", s), shape);
            if (!base) throw std::runtime_error("r97b: lora_expand device row: the gradient stage refused lora_B");
            dB[(size_t)s] = call.fused_slots ? base + s * R : base;
        }
    }
    for (int64_t s = 0; s < S; ++s) {
        const std::vector<int64_t>& idx = rows[(size_t)s];
        const int64_t Ms = (int64_t)idx.size();
        if (Ms == 0) continue;
        const std::vector<double> ys = gather(dy.value, idx, N, sc ? sc->value.data() + s * N : nullptr);
        const std::vector<double> ts = gather(t.value, idx, R);
        DevBuf yd = upload_bf16(ys.data(), Ms, N, ldN);
        DevBuf td = upload_bf16(ts.data(), Ms, R, ldR);
        DevBuf bd = upload_bf16(lb.value.data() + s * N * R, N, R, ldR);
        // dt_s[Ms, R] = dys[Ms, N] B_s[N, R]: B operand B_s read MN-major
        DevBuf out(Ms * ldR * 4);
        gemm_f32(Ms, R, N, Opnd{yd.get(), ldN, false}, Opnd{bd.get(), ldR, true}, out.as<float>(), ldR, false);
        std::vector<double> part((size_t)(Ms * R), 0.0);
        add_f32(part.data(), out, Ms, R, ldR);
        for (int64_t i = 0; i < Ms; ++i)
            for (int64_t j = 0; j < R; ++j) dt.value[(size_t)(idx[(size_t)i] * R + j)] += part[(size_t)(i * R + j)];
        // dB_s[N, R] += dys^T t_s: both read MN-major; the fused factor's rows are N long at stride cols
        if (dB[(size_t)s])
            gemm_f32(N, R, Ms, Opnd{yd.get(), ldN, true}, Opnd{td.get(), ldR, true}, dB[(size_t)s], cols, true);
    }
}

}  // namespace

// The frozen positions are the host rows' (reference linear.cpp:444-457, lora.cpp:534-538).
void register_linear_rows() {
    if (!r97::adjoint_register) return;
    r97::adjoint_register("gemm_nt", r97::Side::device, gemm_nt_device, {1}, nullptr);
    r97::adjoint_register("gemm_nt_q", r97::Side::device, gemm_nt_q_device, {1, 2, 3}, serves_i8a8h);
    // the float-trunk form only: a coded record finds no device row here and the walk runs the host's
    r97::adjoint_register("lora_shrink", r97::Side::device, lora_shrink_device, {1, 2, 3}, float_act);
    r97::adjoint_register("lora_expand", r97::Side::device, lora_expand_device, {1, 2, 3}, nullptr);
    r97::adjoint_register("lora_expand_mm", r97::Side::device, lora_expand_device, {1, 2, 3}, nullptr);
}

}  // namespace r97b_host
