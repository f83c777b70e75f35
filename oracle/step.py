"""TEST INFRASTRUCTURE -- the whole LoRA training step of the hybrid model composed from the reference's OWN
host rows (oracle/_ref/libr97ref.so), in f64: the forward through the registered twins and the reverse walk
through the registered host adjoints, op by op in the step's order. This is the reference's own
`reference_step.cpp` pattern (src/reference_step.cpp:1040-1078: replay the recorded ops through
`twin_record` in f64, then `backward_block` over the same records with the host adjoints), applied to the
op program of one hybrid block as the reference's container records it (tests/fixtures/programs/oracle.json:
rmsnorm, gemm_nt + lora_shrink / lora_expand per projection, gdn_conv_prep, gdn_kkt_solve, gdn_chunk_scan,
gdn_gated_rmsnorm, add; rmsnorm on the q / k heads, rope, attn_paged, sigmoid, mul; rmsnorm, gemm_nt,
silu_mul, gemm_nt, add; the final rmsnorm, the head product and ce_position).

Only tests/ use this, as the checker of the B200 step (r97training_b200.model.TrainStep).

The model is handed in as plain numpy: every projection's stored weight as the decoded (int8 codes, bf16
scale bits) pair the reference's stored-weight rows read, the norms' gains, the GDN parameters, the LoRA
factors by their reference names (`<module>.lora_A` [r, k], `<module>.lora_B` [n, r]).
"""
from __future__ import annotations

import numpy as np

from . import Operand, ref_adjoint, ref_lib, ref_twin
from . import rows as R


def _exact(x):
    return x


# What a stored activation keeps: the identity (the exact f64 step), or R.f64_to_bf16 when the step is
# replayed with the B200 step's storage precision (reference_step's `bf16_store`).
_store = _exact


def _set_store(fn):
    global _store
    _store = fn


def _weight_operand(n, K, codes, sbits):
    """A projection's weight operand: the stored IQR weight the reference's rows decode themselves
    (code x bf16 scale in f64), or, with the B200 storage precision, the bf16 weight its GEMMs read."""
    if _store is _exact:
        return Operand("b", "iqr", (n, K), stored=(codes, sbits)), None
    return Operand("b", "bf16", (n, K)), _store(R.dequant_value(codes, sbits))


def _linear_fwd(x, projs, lora, scale):
    """One fused projection group: for each projection (prefix, n, codes, sbits) the base product
    gemm_nt over its stored weight, plus lora_expand(lora_shrink(x)). Returns the outputs side by side
    and what the adjoint reads."""
    M, K = x.shape
    outs, saved = [], []
    slot = np.zeros(M)
    for prefix, n, codes, sbits in projs:
        b_op, b_val = _weight_operand(n, K, codes, sbits)
        g_ops = [Operand("a", "bf16", (M, K)), b_op, Operand("y", "bf16", (M, n), written=True)]
        g_par = {"M": M, "N": n, "K": K}
        y = ref_twin("gemm_nt", g_par, g_ops, {"a": x, "b": b_val})["y"]
        if prefix + ".lora_A" not in lora:  # a projection without an adapter
            outs.append(y)
            saved.append((prefix, g_ops, g_par, dict(a=x, b=b_val, y=y), None, None, None, None))
            continue
        # the GEMMs read the factors' bf16 mirrors
        A, B = _store(lora[prefix + ".lora_A"]), _store(lora[prefix + ".lora_B"])
        r = A.shape[0]
        sh_ops = [Operand("a", "bf16", (M, K)), Operand("none:1", "invalid", (0,)), Operand("slot", "i32", (M,)),
                  Operand("lora_a", "f32", (1, r, K)), Operand("t", "f32", (M, r), written=True)]
        sh_fwd = {"a": x, "none:1": None, "slot": slot, "lora_a": A[None]}
        t = _store(ref_twin("lora_shrink", {}, sh_ops, sh_fwd)["t"])
        ex_ops = [Operand("t", "f32", (M, r)), Operand("slot", "i32", (M,)), Operand("lora_b", "f32", (1, n, r)),
                  Operand("scale", "f32", (1, n)), Operand("y", "bf16", (M, n), written=True)]
        ex_fwd = {"t": t, "slot": slot, "lora_b": B[None], "scale": np.full((1, n), scale)}
        yl = ref_twin("lora_expand", {}, ex_ops, ex_fwd)["y"]
        outs.append(y + yl)
        saved.append((prefix, g_ops, g_par, dict(a=x, b=b_val, y=y), sh_ops, dict(sh_fwd, t=t), ex_ops,
                      dict(ex_fwd, y=yl)))
    return np.concatenate(outs, axis=1), saved


def _linear_bwd(saved, dy, grads):
    """The group's reverse: per projection the lora_expand, lora_shrink and gemm_nt host adjoints; the
    factors' gradients land in `grads` under the reference's names, dX is returned."""
    dx, col = None, 0
    for prefix, g_ops, g_par, g_fwd, sh_ops, sh_fwd, ex_ops, ex_fwd in saved:
        n = g_ops[1].shape[0]
        d = dy[:, col:col + n]
        col += n
        if sh_ops is None:
            part = ref_adjoint("gemm_nt", g_par, g_ops, g_fwd, {"y": d})[0]["a"]
            dx = part if dx is None else dx + part
            continue
        dc_ex, gr = ref_adjoint("lora_expand", {}, ex_ops, ex_fwd, {"y": d}, prefix=prefix)
        grads.update(gr)
        dc_sh, gr = ref_adjoint("lora_shrink", {}, sh_ops, sh_fwd, {"t": _store(dc_ex["t"])}, prefix=prefix)
        grads.update(gr)
        dc_g, _ = ref_adjoint("gemm_nt", g_par, g_ops, g_fwd, {"y": d})
        part = dc_g["a"] + dc_sh["a"]
        dx = part if dx is None else dx + part
    return dx


def _rmsnorm(x, w, eps):
    rows, n = x.shape
    ops = [Operand("x", "bf16", (rows, n)), Operand("w", "f32", (n,)), Operand("y", "bf16", (rows, n), written=True)]
    par = {"eps": repr(float(eps)), "n": n}
    y = ref_twin("rmsnorm", par, ops, {"x": x, "w": w})["y"]
    return _store(y), (par, ops, {"x": x, "w": w, "y": y})


def _rmsnorm_bwd(saved, dy):
    par, ops, fwd = saved
    return ref_adjoint("rmsnorm", par, ops, fwd, {"y": dy})[0]["x"]


def _gdn_fwd(blk, x, cfg, cu, lora):
    T = x.shape[0]
    H, Hg, K, S = cfg["gdn_heads"], cfg["gdn_qk_heads"], cfg["head_k"], len(cu) - 1
    C = (2 * Hg + H) * K
    sv = {}
    n1, sv["n1"] = _rmsnorm(x, blk["w_in"], cfg["eps"])
    y_in, sv["in"] = _linear_fwd(n1, blk["groups"][0], lora, cfg["scale"])
    y_in = _store(y_in)
    z = y_in[:, C:C + H * K]
    ba = y_in[:, C + H * K:]
    cp_ops = [Operand("x", "bf16", (T, C)), Operand("w", "bf16", (C, 4)), Operand("b", "bf16", (C,)),
              Operand("A_log", "f32", (H,)), Operand("dt_bias", "f32", (H,)),
              Operand("conv_state", "bf16", (S, C, 3), written=True), Operand("cu", "i32", (S + 1,)),
              Operand("a", "bf16", (T, H)), Operand("b_gate", "bf16", (T, H)), Operand("cache_idx", "i32", (S,)),
              Operand("has_init", "i32", (S,)), Operand("q", "bf16", (T, Hg, K), written=True),
              Operand("k", "bf16", (T, Hg, K), written=True), Operand("v", "bf16", (T, H, K), written=True),
              Operand("g", "f32", (T, H), written=True), Operand("beta", "f32", (T, H), written=True)]
    cp_par = {"head_k": K, "head_v": K, "chunk": 64, "conv_width": 4}
    cp_reads = {"x": y_in[:, :C], "w": blk["conv_w"], "b": np.zeros(C), "A_log": blk["a_log"],
                "dt_bias": blk["dt_bias"], "cu": cu, "a": ba[:, H:], "b_gate": ba[:, :H],
                "cache_idx": np.arange(S), "has_init": np.zeros(S)}
    cp = ref_twin("gdn_conv_prep", cp_par, cp_ops, cp_reads)
    for key in ("q", "k", "v"):
        cp[key] = _store(cp[key])
    q, k, v, g, beta = cp["q"], cp["k"], cp["v"], cp["g"], cp["beta"]
    kk_ops = [Operand("k", "bf16", (T, Hg, K)), Operand("beta", "f32", (T, H)), Operand("g", "f32", (T, H)),
              Operand("cu_seqlens", "i32", (S + 1,)), Operand("A", "bf16", (T, H, 64), written=True)]
    kk_par = {"chunk": 64, "head_k": K}
    kk_reads = {"k": k, "beta": beta, "g": g, "cu_seqlens": cu}
    A = ref_twin("gdn_kkt_solve", kk_par, kk_ops, kk_reads)["A"]
    sc_ops = [Operand("q", "bf16", (T, Hg, K)), Operand("k", "bf16", (T, Hg, K)), Operand("v", "bf16", (T, H, K)),
              Operand("A", "bf16", (T, H, 64)), Operand("g", "f32", (T, H)), Operand("beta", "f32", (T, H)),
              Operand("h0", "f32", (S, H, K, K)), Operand("cu_seqlens", "i32", (S + 1,)),
              Operand("o", "bf16", (T, H, K), written=True), Operand("ht", "f32", (S, H, K, K), written=True),
              Operand("state_idx", "i32", (S,))]
    sc_par = {"head_k": K, "head_v": K, "chunk": 64, "scale": repr(1.0 / np.sqrt(K))}
    sc_reads = {"q": q, "k": k, "v": v, "A": A, "g": g, "beta": beta, "h0": np.zeros((S, H, K, K)),
                "cu_seqlens": cu, "state_idx": np.arange(S)}
    sc = ref_twin("gdn_chunk_scan", sc_par, sc_ops, sc_reads)
    o = sc["o"] = _store(sc["o"])
    gn_ops = [Operand("x", "bf16", (T * H, K)), Operand("z", "bf16", (T * H, K)), Operand("w", "f32", (K,)),
              Operand("o", "bf16", (T * H, K), written=True)]
    gn_reads = {"x": o.reshape(T * H, K), "z": z.reshape(T * H, K), "w": blk["gnorm_w"]}
    on = _store(ref_twin("gdn_gated_rmsnorm", {"channels": K}, gn_ops, gn_reads)["o"])
    h, sv["out"] = _linear_fwd(on.reshape(T, H * K), blk["groups"][1], lora, cfg["scale"])
    sv.update(C=C, cp=(cp_par, cp_ops, dict(cp_reads, **cp)), kk=(kk_par, kk_ops, dict(kk_reads, A=A)),
              sc=(sc_par, sc_ops, dict(sc_reads, **sc)), gn=(gn_ops, dict(gn_reads, o=on)), shape=(T, H, K, S))
    return _store(x + h), sv


def _gdn_bwd(sv, dh1, grads):
    T, H, K, S = sv["shape"]
    C = sv["C"]
    don = _store(_linear_bwd(sv["out"], dh1, grads))
    gn_ops, gn_fwd = sv["gn"]
    dgn = ref_adjoint("gdn_gated_rmsnorm", {"channels": K}, gn_ops, gn_fwd, {"o": don.reshape(T * H, K)})[0]
    dgn = {key: _store(val) for key, val in dgn.items()}
    sc_par, sc_ops, sc_fwd = sv["sc"]
    dsc = ref_adjoint("gdn_chunk_scan", sc_par, sc_ops, sc_fwd,
                      {"o": dgn["x"].reshape(T, H, K), "ht": np.zeros((S, H, K, K))})[0]
    kk_par, kk_ops, kk_fwd = sv["kk"]
    dkk = ref_adjoint("gdn_kkt_solve", kk_par, kk_ops, kk_fwd, {"A": dsc["A"]})[0]
    cp_par, cp_ops, cp_fwd = sv["cp"]
    cots = {"conv_state": np.zeros((S, C, 3)), "q": dsc["q"], "k": dsc["k"] + dkk["k"], "v": dsc["v"],
            "g": dsc["g"] + dkk["g"], "beta": dsc["beta"] + dkk["beta"]}
    dcp = ref_adjoint("gdn_conv_prep", cp_par, cp_ops, cp_fwd, cots)[0]
    d_yin = _store(np.concatenate([dcp["x"], dgn["z"].reshape(T, H * K), dcp["b_gate"], dcp["a"]], axis=1))
    dn1 = _store(_linear_bwd(sv["in"], d_yin, grads))
    return _store(_rmsnorm_bwd(sv["n1"], dn1) + dh1)


def _attn_fwd(blk, x, cfg, cu, lora):
    T = x.shape[0]
    Hq, Hkv, Dh, rot = cfg["attn_heads"], cfg["attn_kv_heads"], cfg["attn_head_dim"], cfg["rotary_dim"]
    S, seq = len(cu) - 1, cfg["seq"]
    sv = {}
    n1, sv["n1"] = _rmsnorm(x, blk["w_in"], cfg["eps"])
    y, sv["qkv"] = _linear_fwd(n1, blk["groups"][0], lora, cfg["scale"])
    y = _store(y)
    qg = y[:, :2 * Hq * Dh].reshape(T, Hq, 2, Dh)
    qpre, gate = qg[:, :, 0], qg[:, :, 1].reshape(T, Hq * Dh)
    kpre = y[:, 2 * Hq * Dh:(2 * Hq + Hkv) * Dh].reshape(T, Hkv, Dh)
    v = y[:, (2 * Hq + Hkv) * Dh:].reshape(T, Hkv, Dh)
    # the q / k norm and the rotation are one kernel on the B200 side: the normed rows are not stored
    saved_store = _store
    _set_store(_exact)
    qn, sv["qn"] = _rmsnorm(qpre.reshape(T * Hq, Dh), blk["q_norm"], cfg["eps"])
    kn, sv["kn"] = _rmsnorm(kpre.reshape(T * Hkv, Dh), blk["k_norm"], cfg["eps"])
    _set_store(saved_store)
    pos = np.concatenate([np.arange(cu[s + 1] - cu[s]) for s in range(S)])

    def rope(xr, heads):
        ops = [Operand("x", "bf16", (T, heads * Dh), written=True, in_place=True), Operand("pos", "i32", (T,))]
        par = {"M": seq, "head_dim": Dh, "rotary_dim": rot, "n_head": heads, "n_head_kv": 0,
               "theta": repr(float(cfg["rope_theta"])), "scale": "1"}
        return ref_twin("rope", par, ops, {"x": xr, "pos": pos})["x"], (par, ops, {"x": xr, "pos": pos})

    qr, sv["rq"] = rope(qn.reshape(T, Hq * Dh), Hq)
    kr, sv["rk"] = rope(kn.reshape(T, Hkv * Dh), Hkv)
    qr, kr = _store(qr.reshape(T, Hq, Dh)), _store(kr.reshape(T, Hkv, Dh))
    blkn = int(max(cu[s + 1] - cu[s] for s in range(S)))
    kv = np.zeros((S, Hkv, blkn, 2 * Dh))
    for s in range(S):
        a, b = cu[s], cu[s + 1]
        kv[s, :, :b - a, :Dh] = kr[a:b].transpose(1, 0, 2)
        kv[s, :, :b - a, Dh:] = v[a:b].transpose(1, 0, 2)
    at_ops = [Operand("q", "bf16", (T, Hq, Dh)), Operand("kv", "bf16", (S, Hkv, blkn, 2 * Dh)),
              Operand("block_table", "i32", (S, 1)), Operand("seqused", "i32", (S,)),
              Operand("none:4", "invalid", ()), Operand("none:5", "invalid", ()),
              Operand("cu_seqlens", "i32", (S + 1,)), Operand("out", "bf16", (T, Hq, Dh), written=True)]
    at_reads = {"q": qr, "kv": kv, "block_table": np.arange(S)[:, None], "seqused": np.diff(cu),
                "none:4": None, "none:5": None, "cu_seqlens": cu}
    att = _store(ref_twin("attn_paged", {}, at_ops, at_reads)["out"].reshape(T, Hq * Dh))
    n = Hq * Dh
    sg_ops = [Operand("gate", "bf16", (T, n)), Operand("sg", "bf16", (T, n), written=True)]
    sg = ref_twin("sigmoid", {"M": T, "n": n}, sg_ops, {"gate": gate})["sg"]
    mul_ops = [Operand("o", "bf16", (T, n)), Operand("sg", "bf16", (T, n)), Operand("y", "bf16", (T, n), written=True)]
    ga = _store(ref_twin("mul", {"M": T, "n": n}, mul_ops, {"o": att, "sg": sg})["y"])
    h, sv["o"] = _linear_fwd(ga, blk["groups"][1], lora, cfg["scale"])
    sv.update(at=(at_ops, dict(at_reads, out=att.reshape(T, Hq, Dh))), sg=(sg_ops, {"gate": gate, "sg": sg}),
              mul=(mul_ops, {"o": att, "sg": sg, "y": ga}), shape=(T, Hq, Hkv, Dh, S, blkn))
    return _store(x + h), sv


def _attn_bwd(sv, dh1, grads):
    T, Hq, Hkv, Dh, S, blkn = sv["shape"]
    n = Hq * Dh
    dga = _store(_linear_bwd(sv["o"], dh1, grads))
    mul_ops, mul_fwd = sv["mul"]
    dmul = ref_adjoint("mul", {"M": T, "n": n}, mul_ops, mul_fwd, {"y": dga})[0]
    sg_ops, sg_fwd = sv["sg"]
    dgate = _store(ref_adjoint("sigmoid", {"M": T, "n": n}, sg_ops, sg_fwd, {"sg": dmul["sg"]})[0]["gate"])
    at_ops, at_fwd = sv["at"]
    dat = ref_adjoint("attn_paged", {}, at_ops, at_fwd, {"out": _store(dmul["o"]).reshape(T, Hq, Dh)})[0]
    dat = {key: _store(val) for key, val in dat.items()}
    cu = at_fwd["cu_seqlens"]
    dkr = np.zeros((T, Hkv, Dh))
    dv = np.zeros((T, Hkv, Dh))
    for s in range(S):
        a, b = cu[s], cu[s + 1]
        dkr[a:b] = dat["kv"][s, :, :b - a, :Dh].transpose(1, 0, 2)
        dv[a:b] = dat["kv"][s, :, :b - a, Dh:].transpose(1, 0, 2)

    def rope_bwd(saved, d):
        par, ops, fwd = saved
        return ref_adjoint("rope", par, ops, fwd, {"x": d})[0]["x"]

    dqn = rope_bwd(sv["rq"], dat["q"].reshape(T, n))
    dkn = rope_bwd(sv["rk"], dkr.reshape(T, Hkv * Dh))
    dqpre = _rmsnorm_bwd(sv["qn"], dqn.reshape(T * Hq, Dh)).reshape(T, Hq, 1, Dh)
    dkpre = _rmsnorm_bwd(sv["kn"], dkn.reshape(T * Hkv, Dh)).reshape(T, Hkv * Dh)
    dqg = np.concatenate([dqpre, dgate.reshape(T, Hq, 1, Dh)], axis=2).reshape(T, 2 * n)
    dy = _store(np.concatenate([dqg, dkpre, dv.reshape(T, Hkv * Dh)], axis=1))
    dn1 = _store(_linear_bwd(sv["qkv"], dy, grads))
    return _store(_rmsnorm_bwd(sv["n1"], dn1) + dh1)


def _mlp_fwd(blk, h1, cfg, lora):
    T = h1.shape[0]
    F = cfg["ffn"]
    sv = {}
    n2, sv["n2"] = _rmsnorm(h1, blk["w_post"], cfg["eps"])
    gu, sv["gu"] = _linear_fwd(n2, blk["groups"][2], lora, cfg["scale"])
    gu = _store(gu)
    sm_ops = [Operand("gu", "bf16", (T, 2 * F)), Operand("a", "bf16", (T, F), written=True)]
    a = _store(ref_twin("silu_mul", {"M": T, "n": F}, sm_ops, {"gu": gu})["a"])
    d, sv["down"] = _linear_fwd(a, blk["groups"][3], lora, cfg["scale"])
    sv["sm"] = (sm_ops, {"gu": gu, "a": a}, T, F)
    return _store(h1 + d), sv


def _mlp_bwd(sv, dxn, grads):
    da = _linear_bwd(sv["down"], dxn, grads)
    sm_ops, sm_fwd, T, F = sv["sm"]
    dgu = _store(ref_adjoint("silu_mul", {"M": T, "n": F}, sm_ops, sm_fwd, {"a": da})[0]["gu"])
    dn2 = _store(_linear_bwd(sv["gu"], dgu, grads))
    return _store(_rmsnorm_bwd(sv["n2"], dn2) + dxn)


def reference_step(model: dict, ids: np.ndarray, targets: np.ndarray, backward: bool = True,
                   f64_loss: bool = False, bf16_store: bool = False):
    """The loss (mean CE over the scored rows, targets < 0 unscored) and every LoRA factor's gradient
    {name: f32 array} of one step over token ids [micro_batch, seq], composed from the reference's rows.
    backward=False returns (loss, None). f64_loss takes the CE in f64 (oracle.rows.ce_rows, pinned to
    ce_position) instead of ce_position over f32 logit rows, for finite differences of the loss.
    bf16_store replays the same rows with every activation, cotangent and weight that the B200 step keeps
    in bf16 rounded to bf16 where that step stores it (the op outputs, the LoRA factors' bf16 mirrors, the
    decoded weights, the logits and their gradient), so that what is left between the two is arithmetic
    order and f32 against f64.

    ``model``: {"cfg": {...}, "blocks": [...], "w_final", "head": (codes, sbits), "lora": {name: array}};
    each block {"kind", "w_in", "w_post", "groups": [[(prefix, n, codes, sbits), ...] x 4], and the GDN's
    "conv_w", "a_log", "dt_bias", "gnorm_w" or the attention's "q_norm", "k_norm"}."""
    _set_store(R.f64_to_bf16 if bf16_store else _exact)
    try:
        return _reference_step(model, ids, targets, backward, f64_loss)
    finally:
        _set_store(_exact)


def _reference_step(model: dict, ids: np.ndarray, targets: np.ndarray, backward: bool, f64_loss: bool):
    cfg, lora = model["cfg"], model["lora"]
    mb, seq = ids.shape
    T = mb * seq
    cu = np.arange(0, T + 1, seq)
    head_codes, head_sbits = model["head"]
    W_head = _store(R.dequant_value(head_codes, head_sbits))
    x = W_head[ids.reshape(-1)]  # the tied head's rows (frozen: no cotangent is needed)
    saved = []
    for blk in model["blocks"]:
        if blk["kind"] == "gdn":
            h1, sm = _gdn_fwd(blk, x, cfg, cu, lora)
        else:
            h1, sm = _attn_fwd(blk, x, cfg, cu, lora)
        x, sp = _mlp_fwd(blk, h1, cfg, lora)
        saved.append((blk["kind"], sm, sp))
    nf, s_nf = _rmsnorm(x, model["w_final"], cfg["eps"])
    V = W_head.shape[0]
    hb_op, hb_val = _weight_operand(V, nf.shape[1], head_codes, head_sbits)
    h_ops = [Operand("a", "bf16", (T, nf.shape[1])), hb_op, Operand("y", "f32", (T, V), written=True)]
    h_par = {"M": T, "N": V, "K": nf.shape[1]}
    logits = _store(ref_twin("gemm_nt", h_par, h_ops, {"a": nf, "b": hb_val})["y"])
    tg = targets.reshape(-1)
    scored = int((tg >= 0).sum())
    scale = 1.0 / max(scored, 1)
    if f64_loss:
        lr, dlog = R.ce_rows(logits, tg, grad_scale=scale)
        loss = float(lr.sum()) * scale
    else:
        lib = ref_lib()
        dlog = np.zeros((T, V), np.float32)
        loss = 0.0
        for r in range(T):
            if tg[r] < 0:
                continue
            row = np.ascontiguousarray(logits[r], np.float32)
            loss += lib.ref_ce_position(row.ctypes.data, V, int(tg[r]), dlog[r].ctypes.data, scale)
        loss *= scale
    if not backward:
        return loss, None
    dlog = _store(dlog.astype(np.float64))
    dnf = _store(ref_adjoint("gemm_nt", h_par, h_ops, {"a": nf, "b": hb_val, "y": logits}, {"y": dlog})[0]["a"])
    dx = _store(_rmsnorm_bwd(s_nf, dnf))
    grads = {}
    for kind, sm, sp in reversed(saved):
        dh1 = _mlp_bwd(sp, dx, grads)
        dx = _gdn_bwd(sm, dh1, grads) if kind == "gdn" else _attn_bwd(sm, dh1, grads)
    return loss, grads


def model_from_torch(model, lora: dict) -> dict:
    """The numpy model reference_step takes, from an r97training_b200.model.HybridModel (any device): every
    stored weight decoded on the CPU by this oracle's C restatement of the IQR decode (bit-exact to the
    reference's r97_iqr_decode_host) into the (int8 codes, bf16 scale bits) pair the stored-weight rows
    read. ``lora`` maps each factor's reference name to its f32 value."""
    c = model.cfg

    def stored(w):
        form = R.trunk_form(w.codes.cpu().numpy(), w.scale.cpu().numpy(), w.mad_a, w.mad_b, w.cols)
        return R.iqr_decode(form)

    def f64(t):
        return t.detach().cpu().double().numpy()

    from r97training_b200.model import module_path
    blocks = []
    for li, blk in enumerate(model.blocks):
        b = {"kind": blk["kind"], "w_in": f64(blk["w_in"]), "w_post": f64(blk["w_post"]), "groups": []}
        for g in blk["groups"]:
            projs = []
            for (pname, n), w in zip(g.projs, g.iqr):
                codes, sbits = stored(w)
                projs.append((module_path(li, blk["kind"], pname), n, codes, sbits))
            b["groups"].append(projs)
        for key in ("conv_w", "a_log", "dt_bias", "gnorm_w", "q_norm", "k_norm"):
            if key in blk:
                b[key] = f64(blk[key])
        blocks.append(b)
    cfg = dict(hidden=c.hidden, gdn_heads=c.gdn_heads, gdn_qk_heads=c.gdn_qk_heads, head_k=c.head_k,
               attn_heads=c.attn_heads, attn_kv_heads=c.attn_kv_heads, attn_head_dim=c.attn_head_dim,
               rotary_dim=c.rotary_dim, rope_theta=c.rope_theta, ffn=c.ffn, eps=c.eps, seq=c.seq,
               scale=c.alpha / c.rank)
    return {"cfg": cfg, "blocks": blocks, "w_final": f64(model.w_final), "head": stored(model.head),
            "lora": {k: np.asarray(v, np.float64) for k, v in lora.items()}}
