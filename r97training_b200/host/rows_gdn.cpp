// rows_gdn.cpp -- device adjoint rows of the chunked GatedDeltaNet as the reference splits it:
// gdn_kkt_solve (A = (I + M)^-1 per chunk) and gdn_chunk_scan (the state pass that reads A), on the
// tensor-core GDN kernels of libr97b200.so.
//
// The fused layer (r97b_gdn_fwd / r97b_gdn_bwd) solves for A itself and folds the solve's adjoint into
// its backward; the two flags of R97bGdnDims split it back into the reference's two ops: the scan row
// runs the forward on the record's own A (R97B_GDN_A_GIVEN) and the backward with the solve's adjoint
// left out and the scan's dA written (R97B_GDN_SPLIT_KKT); the solve row runs r97b_gdn_kkt_bwd on the
// cotangent the walk hands it. Records follow the host rows' schemas (src/adjoint/host/gdn_kkt.cpp:221-355,
// gdn_scan.cpp:36-60 and 487-584). The kernels take head_k = head_v = 128 and chunk = 64; a record of
// another geometry is left to the host row.
#include "common.h"

#include <cmath>

namespace r97b_host {
namespace {

constexpr int64_t kD = 128;
constexpr int64_t kChunk = 64;

// A ragged batch's chunk table on the device, and the dims the kernels read.
struct Geometry {
    R97bGdnDims dims{};
    DevBuf tok0, len, seq_c0;
};

bool make_geometry(const AdValue& cu, int64_t H, int64_t Hg, double scale, int32_t flags, Geometry* g) {
    const int64_t N = (int64_t)cu.value.size() - 1;
    if (N <= 0) return false;
    std::vector<int32_t> cuh((size_t)(N + 1));
    for (int64_t i = 0; i <= N; ++i) cuh[(size_t)i] = (int32_t)cu.value[(size_t)i];
    const int32_t n = r97b_gdn_chunk_table(cuh.data(), (int32_t)N, (int32_t)kChunk, nullptr, nullptr, nullptr);
    if (n < 0) return false;
    std::vector<int32_t> tok0((size_t)std::max(n, 1), 0), len((size_t)std::max(n, 1), 0), sc0((size_t)(N + 1), 0);
    r97b_gdn_chunk_table(cuh.data(), (int32_t)N, (int32_t)kChunk, tok0.data(), len.data(), sc0.data());
    g->tok0 = upload_i32(tok0);
    g->len = upload_i32(len);
    g->seq_c0 = upload_i32(sc0);
    R97bGdnDims& d = g->dims;
    d.n_seq = (int32_t)N;
    d.H = (int32_t)H;
    d.Hg = (int32_t)Hg;
    d.n_chunks = n;
    d.head_k = (int32_t)kD;
    d.head_v = (int32_t)kD;
    d.chunk = (int32_t)kChunk;
    d.flags = flags;
    d.T = (int64_t)cuh.back();
    d.scale = (float)scale;
    d.chunk_tok0 = g->tok0.as<int32_t>();
    d.chunk_len = g->len.as<int32_t>();
    d.seq_chunk0 = g->seq_c0.as<int32_t>();
    return true;
}

// [T, H, 128] f32 per value head -> [T, Hg, 128], summing the heads that share a key head.
DevBuf sum_heads(const DevBuf& src, int64_t T, int64_t H, int64_t Hg) {
    DevBuf out(T * Hg * kD * 4);
    check(r97b_gdn_sum_heads(src.as<float>(), out.as<float>(), T, (int32_t)H, (int32_t)Hg, row_stream()), "sum_heads");
    return out;
}

// ------------------------------------------------------------------------------------ gdn_kkt_solve
// Operands: k [T, Hg, K] bf16, beta [T, H] f32, g [T, H] f32, cu_seqlens [S+1], A [T, H, chunk] (written).

void kkt_device(const AdjointCall& call) {
    if (!call.dc || call.cot.empty() || call.fwd.size() < 5 || call.dc->size() < 3) return;
    const AdValue& k = call.fwd[0];
    const AdValue& beta = call.fwd[1];
    const AdValue& g = call.fwd[2];
    const AdValue& cu = call.fwd[3];
    const AdValue& A = call.fwd[4];
    const AdValue& dA = call.cot[0];
    const int64_t chunk = int_param(call.rec, "chunk", kChunk), K = int_param(call.rec, "head_k", kD);
    if (chunk != kChunk || K != kD || cu.value.size() < 2) return;
    const int64_t T = (int64_t)cu.value.back();
    if (T <= 0 || (int64_t)k.value.size() % (T * kD) || (int64_t)beta.value.size() % T) return;
    const int64_t Hg = (int64_t)k.value.size() / (T * kD), H = (int64_t)beta.value.size() / T;
    if (Hg <= 0 || H <= 0 || H % Hg || (int64_t)g.value.size() != T * H) return;
    if ((int64_t)A.value.size() != T * H * kChunk || (int64_t)dA.value.size() != T * H * kChunk) return;
    AdValue& dk = call.dc->at(0);
    AdValue& dbeta = call.dc->at(1);
    AdValue& dg = call.dc->at(2);
    if (dk.value.size() != k.value.size() || dbeta.value.size() != beta.value.size() || dg.value.size() != g.value.size())
        return;
    Geometry geo;
    if (!make_geometry(cu, H, Hg, 1.0 / std::sqrt((double)K), 0, &geo)) return;
    DevBuf kd = upload_bf16(k.value.data(), 1, T * Hg * kD, T * Hg * kD);
    DevBuf gd = upload_f32(g.value.data(), 1, T * H, T * H);
    DevBuf bd = upload_f32(beta.value.data(), 1, T * H, T * H);
    DevBuf Ad = upload_f32(A.value.data(), 1, T * H * kChunk, T * H * kChunk);
    DevBuf dAd = upload_f32(dA.value.data(), 1, T * H * kChunk, T * H * kChunk);
    DevBuf dkh(T * H * kD * 4), dbd(T * H * 4), dgd(T * H * 4);
    check(r97b_gdn_kkt_bwd(&geo.dims, kd.as<uint16_t>(), gd.as<float>(), bd.as<float>(), Ad.as<float>(), dAd.as<float>(),
                           dkh.as<float>(), dbd.as<float>(), dgd.as<float>(), row_stream()),
          "gdn_kkt_bwd");
    DevBuf dkg = sum_heads(dkh, T, H, Hg);
    add_f32(dk.value.data(), dkg, 1, T * Hg * kD, T * Hg * kD);
    add_f32(dbeta.value.data(), dbd, 1, T * H, T * H);
    add_f32(dg.value.data(), dgd, 1, T * H, T * H);
}

// ------------------------------------------------------------------------------------ gdn_chunk_scan

enum : int { kQ = 0, kK = 1, kV = 2, kA = 3, kG = 4, kBeta = 5, kH0 = 6, kCu = 7, kO = 8, kHt = 9, kSidx = 10 };

void scan_device(const AdjointCall& call) {
    const std::vector<AdValue>& f = call.fwd;
    if (!call.dc || call.cot.size() < 2 || f.size() < (size_t)kHt + 1 || call.dc->size() < (size_t)kBeta + 1) return;
    const int64_t K = int_param(call.rec, "head_k", kD), V = int_param(call.rec, "head_v", kD);
    const int64_t chunk = int_param(call.rec, "chunk", kChunk);
    if (K != kD || V != kD || chunk != kChunk) return;
    const double scale = num_param(call.rec, "scale", 1.0 / std::sqrt((double)K));
    const AdValue& cu = f[kCu];
    const int64_t N = (int64_t)cu.value.size() - 1;
    if (N <= 0) return;
    const int64_t T = (int64_t)cu.value.back();
    if (T <= 0 || (int64_t)f[kQ].value.size() % (T * kD) || (int64_t)f[kV].value.size() % (T * kD)) return;
    const int64_t Hg = (int64_t)f[kQ].value.size() / (T * kD), H = (int64_t)f[kV].value.size() / (T * kD);
    if (Hg <= 0 || H <= 0 || H % Hg) return;
    if ((int64_t)f[kK].value.size() != T * Hg * kD || (int64_t)f[kA].value.size() != T * H * kChunk ||
        (int64_t)f[kG].value.size() != T * H || (int64_t)f[kBeta].value.size() != T * H)
        return;
    const AdValue& d_o = call.cot[0];
    const AdValue& d_ht = call.cot[1];
    if ((int64_t)d_o.value.size() != T * H * kD) return;
    // the state slot each sequence owns; two sequences on one slot are left to the host row
    const std::vector<int64_t>& h0s = call.rec.operands[kH0].shape;
    const int64_t slots = h0s.empty() ? N : h0s.front();
    const int64_t per = H * kD * kD;
    std::vector<int64_t> slot_of((size_t)N, -1);
    for (int64_t n = 0; n < N; ++n) {
        if (cu.value[(size_t)(n + 1)] <= cu.value[(size_t)n]) continue;
        int64_t s = n;
        if (f.size() > (size_t)kSidx && (int64_t)f[kSidx].value.size() > n) s = (int64_t)f[kSidx].value[(size_t)n];
        if (s >= 0 && s < slots) slot_of[(size_t)n] = s;
    }
    for (int64_t a = 0; a < N; ++a)
        for (int64_t b = a + 1; b < N; ++b)
            if (slot_of[(size_t)a] >= 0 && slot_of[(size_t)a] == slot_of[(size_t)b]) return;
    std::vector<double> h0((size_t)(N * per), 0.0), dht((size_t)(N * per), 0.0);
    for (int64_t n = 0; n < N; ++n) {
        const int64_t s = slot_of[(size_t)n];
        if (s < 0) continue;
        if ((int64_t)f[kH0].value.size() >= (s + 1) * per)
            std::copy(f[kH0].value.begin() + s * per, f[kH0].value.begin() + (s + 1) * per, h0.begin() + n * per);
        if ((int64_t)d_ht.value.size() >= (s + 1) * per)
            std::copy(d_ht.value.begin() + s * per, d_ht.value.begin() + (s + 1) * per, dht.begin() + n * per);
    }
    AdValue& dq = call.dc->at(kQ);
    AdValue& dk = call.dc->at(kK);
    AdValue& dv = call.dc->at(kV);
    AdValue& dA = call.dc->at(kA);
    AdValue& dg = call.dc->at(kG);
    AdValue& dbeta = call.dc->at(kBeta);
    if (dq.value.size() != f[kQ].value.size() || dk.value.size() != f[kK].value.size() ||
        dv.value.size() != f[kV].value.size() || dA.value.size() != f[kA].value.size() ||
        dg.value.size() != f[kG].value.size() || dbeta.value.size() != f[kBeta].value.size())
        return;

    Geometry geo;
    if (!make_geometry(cu, H, Hg, scale, R97B_GDN_A_GIVEN | R97B_GDN_SPLIT_KKT, &geo)) return;
    const int64_t n_chunks = std::max<int64_t>(geo.dims.n_chunks, 1);
    DevBuf q = upload_bf16(f[kQ].value.data(), 1, T * Hg * kD, T * Hg * kD);
    DevBuf k = upload_bf16(f[kK].value.data(), 1, T * Hg * kD, T * Hg * kD);
    DevBuf v = upload_bf16(f[kV].value.data(), 1, T * H * kD, T * H * kD);
    DevBuf g = upload_f32(f[kG].value.data(), 1, T * H, T * H);
    DevBuf beta = upload_f32(f[kBeta].value.data(), 1, T * H, T * H);
    DevBuf A = upload_f32(f[kA].value.data(), 1, T * H * kChunk, T * H * kChunk);
    DevBuf h0d = upload_f32(h0.data(), 1, N * per, N * per);
    DevBuf w(T * H * kD * 4), u(T * H * kD * 4), S(n_chunks * H * kD * kD * 4), Vp(T * H * kD * 4);
    DevBuf P(n_chunks * H * kChunk * kChunk * 4), o(T * H * kD * 2);
    R97bGdnFwd fa{};
    fa.q = q.as<uint16_t>();
    fa.k = k.as<uint16_t>();
    fa.v = v.as<uint16_t>();
    fa.g = g.as<float>();
    fa.beta = beta.as<float>();
    fa.h0 = h0d.as<float>();
    fa.A = A.as<float>();
    fa.w = w.as<float>();
    fa.u = u.as<float>();
    fa.S = S.as<float>();
    fa.Vp = Vp.as<float>();
    fa.P = P.as<float>();
    fa.o = o.as<uint16_t>();
    fa.ht = nullptr;
    check(r97b_gdn_fwd(&geo.dims, &fa, row_stream()), "gdn_fwd");

    DevBuf dOd = upload_bf16(d_o.value.data(), 1, T * H * kD, T * H * kD);
    DevBuf dhtd = upload_f32(dht.data(), 1, N * per, N * per);
    DevBuf dS(n_chunks * H * kD * kD * 4), dVp(T * H * kD * 4), dw(T * H * kD * 4);
    DevBuf dqh(T * H * kD * 4), dkh(T * H * kD * 4), dvd(T * H * kD * 4);
    DevBuf dbd(T * H * 4), dgd(T * H * 4), dAd(T * H * kChunk * 4);
    dAd.zero();
    R97bGdnBwd ba{};
    ba.q = fa.q;
    ba.k = fa.k;
    ba.v = fa.v;
    ba.g = fa.g;
    ba.beta = fa.beta;
    ba.A = fa.A;
    ba.w = fa.w;
    ba.S = fa.S;
    ba.Vp = fa.Vp;
    ba.P = fa.P;
    ba.dO = dOd.as<uint16_t>();
    ba.dht = dhtd.as<float>();
    ba.dS = dS.as<float>();
    ba.dVp = dVp.as<float>();
    ba.dw = dw.as<float>();
    ba.dq = dqh.as<float>();
    ba.dk = dkh.as<float>();
    ba.dv = dvd.as<float>();
    ba.dbeta = dbd.as<float>();
    ba.dg = dgd.as<float>();
    ba.dh0 = nullptr;  // h0 is frozen
    ba.dA = dAd.as<float>();
    check(r97b_gdn_bwd(&geo.dims, &ba, row_stream()), "gdn_bwd");
    DevBuf dqg = sum_heads(dqh, T, H, Hg), dkg = sum_heads(dkh, T, H, Hg);
    add_f32(dq.value.data(), dqg, 1, T * Hg * kD, T * Hg * kD);
    add_f32(dk.value.data(), dkg, 1, T * Hg * kD, T * Hg * kD);
    add_f32(dv.value.data(), dvd, 1, T * H * kD, T * H * kD);
    add_f32(dA.value.data(), dAd, 1, T * H * kChunk, T * H * kChunk);
    add_f32(dg.value.data(), dgd, 1, T * H, T * H);
    add_f32(dbeta.value.data(), dbd, 1, T * H, T * H);
}

}  // namespace

// Frozen positions as the host rows' (gdn_kkt.cpp:355: cu_seqlens; gdn_scan.cpp:584: h0, cu_seqlens,
// state_idx).
void register_gdn_rows() {
    if (!r97::adjoint_register) return;
    r97::adjoint_register("gdn_kkt_solve", r97::Side::device, kkt_device, {3}, nullptr);
    r97::adjoint_register("gdn_chunk_scan", r97::Side::device, scan_device, {kH0, kCu, kSidx}, nullptr);
}

}  // namespace r97b_host
