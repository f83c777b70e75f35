"""The oracle's restatements pinned against the reference's OWN host code (oracle/_ref/libr97ref.so,
compiled in place from the reference tree): the IQR decode bit for bit over every stored form, the
f64 linear/LoRA/norm rows to rounding, CE, and AdamW bit for bit. CPU only."""
import numpy as np
import pytest

import oracle
from oracle import Operand, ref_adjoint, ref_twin
from oracle import rows as R
from tests.iqr_forms import FORMS, make_form

ref = pytest.importorskip  # noqa: keep the name free


def _ref():
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")
    return oracle.ref_lib()


@pytest.mark.parametrize("kw", FORMS, ids=[str(i) for i in range(len(FORMS))])
def test_iqr_decode_bit_exact_vs_reference(kw):
    lib = _ref()
    form = make_form(**kw)
    c0, s0 = R.iqr_decode(form)
    c1, s1 = R.iqr_decode(form, lib=lib)
    assert np.array_equal(c0, c1)
    assert np.array_equal(s0, s1)


def test_iqr_decode_chunk_equals_whole():
    form = make_form(rows=768)
    c, s = R.iqr_decode(form)
    c2, s2 = R.iqr_decode(form, row0=256, rows=512)
    assert np.array_equal(c[256:], c2) and np.array_equal(s[256:], s2)


def test_iqr_validate_rejects():
    form = make_form()
    with pytest.raises(ValueError):
        R.iqr_decode(form, row0=100, rows=100)  # not a run boundary


def _stored_weight(n, k, seed):
    rs = np.random.RandomState(seed)
    codes = rs.randint(-126, 127, size=(n, k)).astype(np.int8)
    sc = np.abs(rs.normal(0, 0.02, size=(n, k // 128))).astype(np.float32)
    bits = ((sc.view(np.uint32) + 0x7FFF + ((sc.view(np.uint32) >> 16) & 1)) >> 16).astype(np.uint16)
    return codes, bits


def test_gemm_nt_stored_twin_and_adjoint():
    _ref()
    M, N, K = 8, 256, 256
    rs = np.random.RandomState(1)
    x = rs.normal(size=(M, K))
    dy = rs.normal(size=(M, N)) * 1e-2
    codes, sbits = _stored_weight(N, K, 2)
    ops = [Operand("a", "bf16", (M, K)), Operand("b", "iqr", (N, K), stored=(codes, sbits)),
           Operand("y", "bf16", (M, N), written=True)]
    params = {"M": M, "N": N, "K": K}
    y = ref_twin("gemm_nt", params, ops, {"a": x, "b": None})["y"]
    W = R.dequant_value(codes, sbits)
    np.testing.assert_allclose(y, R.gemm_nt(x, W), rtol=1e-12, atol=1e-12)
    dc, _ = ref_adjoint("gemm_nt", params, ops, {"a": x, "b": None, "y": y}, {"y": dy})
    np.testing.assert_allclose(dc["a"], R.gemm_nt_dx(dy, W), rtol=1e-12, atol=1e-12)


def test_lora_shrink_expand_twins_and_adjoints():
    _ref()
    M, K, N, r = 16, 128, 96, 4
    rs = np.random.RandomState(3)
    x = rs.normal(size=(M, K))
    A = rs.normal(size=(1, r, K)) / 4
    B = rs.normal(size=(1, N, r)) * 0.01
    scale = np.full((1, N), 2.0)
    slot = np.zeros(M)
    sh_ops = [Operand("a", "bf16", (M, K)), Operand("none:1", "invalid", (0,)), Operand("slot", "i32", (M,)),
              Operand("lora_a", "f32", (1, r, K)), Operand("t", "f32", (M, r), written=True)]
    t = ref_twin("lora_shrink", {}, sh_ops, {"a": x, "none:1": None, "slot": slot, "lora_a": A})["t"]
    np.testing.assert_allclose(t, x @ A[0].T, rtol=1e-12)
    ex_ops = [Operand("t", "f32", (M, r)), Operand("slot", "i32", (M,)), Operand("lora_b", "f32", (1, N, r)),
              Operand("scale", "f32", (1, N)), Operand("y", "bf16", (M, N), written=True)]
    y = ref_twin("lora_expand", {}, ex_ops, {"t": t, "slot": slot, "lora_b": B, "scale": scale})["y"]
    np.testing.assert_allclose(y, 2.0 * t @ B[0].T, rtol=1e-12)
    dy = rs.normal(size=(M, N)) * 1e-2
    dc, grads = ref_adjoint("lora_expand", {}, ex_ops, {"t": t, "slot": slot, "lora_b": B, "scale": scale, "y": y},
                            {"y": dy}, prefix="m")
    W0 = np.zeros((N, K))
    dx, dA, dB, dt = R.lora_bwd(x, W0, A[0], B[0], 2.0, t, dy)
    np.testing.assert_allclose(dc["t"], dt, rtol=1e-12, atol=1e-15)
    np.testing.assert_allclose(grads["m.lora_B"].reshape(N, r), dB, rtol=1e-5, atol=1e-9)
    dc2, grads2 = ref_adjoint("lora_shrink", {}, sh_ops,
                              {"a": x, "none:1": None, "slot": slot, "lora_a": A, "t": t}, {"t": dt}, prefix="m")
    np.testing.assert_allclose(dc2["a"], dt @ A[0], rtol=1e-12, atol=1e-15)
    np.testing.assert_allclose(grads2["m.lora_A"].reshape(r, K), dA, rtol=1e-5, atol=1e-9)


def test_rmsnorm_rows():
    _ref()
    rows, n = 6, 64
    rs = np.random.RandomState(4)
    x = rs.normal(size=(rows, n))
    w = rs.normal(size=(n,))
    dy = rs.normal(size=(rows, n))
    ops = [Operand("x", "bf16", (rows, n)), Operand("w", "f32", (n,)), Operand("y", "bf16", (rows, n), written=True)]
    params = {"eps": "1e-06"}
    y = ref_twin("rmsnorm", params, ops, {"x": x, "w": w})["y"]
    np.testing.assert_allclose(y, R.rmsnorm_fwd(x, w), rtol=1e-12)
    dc, _ = ref_adjoint("rmsnorm", params, ops, {"x": x, "w": w, "y": y}, {"y": dy})
    np.testing.assert_allclose(dc["x"], R.rmsnorm_bwd(x, w, dy), rtol=1e-10, atol=1e-12)


def test_gated_rmsnorm_rows():
    _ref()
    rows, n = 12, 128
    rs = np.random.RandomState(5)
    x, z, do = rs.normal(size=(rows, n)), rs.normal(size=(rows, n)), rs.normal(size=(rows, n))
    w = rs.normal(size=(n,))
    ops = [Operand("x", "bf16", (rows, n)), Operand("z", "bf16", (rows, n)), Operand("w", "f32", (n,)),
           Operand("o", "bf16", (rows, n), written=True)]
    o = ref_twin("gdn_gated_rmsnorm", {"channels": n}, ops, {"x": x, "z": z, "w": w})["o"]
    np.testing.assert_allclose(o, R.gated_rmsnorm_fwd(x, z, w), rtol=1e-12)
    dc, _ = ref_adjoint("gdn_gated_rmsnorm", {"channels": n}, ops, {"x": x, "z": z, "w": w, "o": o}, {"o": do})
    dx, dz = R.gated_rmsnorm_bwd(x, z, w, do)
    np.testing.assert_allclose(dc["x"], dx, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dc["z"], dz, rtol=1e-10, atol=1e-12)


def test_ce_position_vs_reference():
    import ctypes
    lib = _ref()
    rs = np.random.RandomState(6)
    vocab = 1000
    x = rs.normal(size=(3, vocab)).astype(np.float32) * 3
    tg = np.array([5, 999, 0], np.int32)
    loss, grad = R.ce_rows(x.astype(np.float64), tg, grad_scale=0.25)
    for i in range(3):
        g = np.zeros(vocab, np.float32)
        row = np.ascontiguousarray(x[i])
        l = lib.ref_ce_position(row.ctypes.data, vocab, int(tg[i]), g.ctypes.data, 0.25)
        assert abs(l - loss[i]) < 1e-12
        np.testing.assert_allclose(g, grad[i].astype(np.float32), rtol=1e-6, atol=1e-9)


def test_adamw_bit_exact_vs_reference():
    lib = _ref()
    rs = np.random.RandomState(7)
    n, steps = 5000, 3
    w0 = rs.normal(size=n).astype(np.float32)
    gs = (rs.normal(size=(steps, n)) * 1e-2).astype(np.float32)
    cfg = dict(lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01)
    wr = w0.copy()
    rc = lib.ref_adamw(wr.ctypes.data, n, gs.ctypes.data, steps, cfg["lr"], cfg["beta1"], cfg["beta2"], cfg["eps"],
                       cfg["weight_decay"], 0.0, 0, 0, 1)
    assert rc == 0
    w, m, v = w0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    for t in range(1, steps + 1):
        lr = R.scheduled_lr(cfg["lr"], 0, 0, 0.1, t)
        R.adamw_update(w, m, v, gs[t - 1], lr, cfg["beta1"], cfg["beta2"], cfg["eps"], cfg["weight_decay"], t)
    assert np.array_equal(w.view(np.uint32), wr.view(np.uint32))


def test_scheduled_lr_vs_reference():
    lib = _ref()
    for step in (1, 5, 10, 11, 50, 100, 200):
        a = lib.ref_scheduled_lr(1e-3, 10, 100, 0.1, step)
        b = R.scheduled_lr(1e-3, 10, 100, 0.1, step)
        assert np.float32(a) == b


def _conv_record(T, S, Hg, H, K, W=4):
    C = 2 * Hg * K + H * K
    ops = [Operand("x", "bf16", (T, C)), Operand("w", "bf16", (C, W)), Operand("b", "bf16", (C,)),
           Operand("A_log", "f32", (H,)), Operand("dt_bias", "f32", (H,)),
           Operand("conv_state", "bf16", (S, C, W - 1), written=True), Operand("cu", "i32", (S + 1,)),
           Operand("a", "bf16", (T, H)), Operand("b_gate", "bf16", (T, H)), Operand("cache_idx", "i32", (S,)),
           Operand("has_init", "i32", (S,)), Operand("q", "bf16", (T, Hg, K), written=True),
           Operand("k", "bf16", (T, Hg, K), written=True), Operand("v", "bf16", (T, H, K), written=True),
           Operand("g", "f32", (T, H), written=True), Operand("beta", "f32", (T, H), written=True)]
    return ops, {"head_k": K, "head_v": K, "chunk": 64, "conv_width": W}


def test_conv_prep_and_gates_vs_reference():
    _ref()
    rs = np.random.RandomState(21)
    lens, Hg, H, K = (70, 5, 130), 2, 4, 16
    T, S = sum(lens), len(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    C = 2 * Hg * K + H * K
    x = rs.normal(size=(T, C))
    w = rs.normal(size=(C, 4)) * 0.5
    a, bg = rs.normal(size=(T, H)), rs.normal(size=(T, H))
    a_log, dt_bias = np.log(rs.uniform(1, 16, size=H)), rs.normal(size=H) * 0.1
    ops, params = _conv_record(T, S, Hg, H, K)
    reads = {"x": x, "w": w, "b": np.zeros(C), "A_log": a_log, "dt_bias": dt_bias, "cu": cu, "a": a, "b_gate": bg,
             "cache_idx": np.arange(S), "has_init": np.zeros(S)}
    out = ref_twin("gdn_conv_prep", params, ops, reads)
    q, k, v = R.conv_prep_fwd(x, w, cu, Hg, H, K)
    g, beta = R.gates_fwd(a, bg, a_log, dt_bias, cu)
    np.testing.assert_allclose(q, out["q"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(k, out["k"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(v, out["v"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(g, out["g"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(beta, out["beta"], rtol=1e-10, atol=1e-12)
    dq, dk, dv = rs.normal(size=q.shape), rs.normal(size=k.shape), rs.normal(size=v.shape)
    dg, db = rs.normal(size=g.shape), rs.normal(size=beta.shape)
    fwd = dict(reads, conv_state=out["conv_state"], q=out["q"], k=out["k"], v=out["v"], g=out["g"], beta=out["beta"])
    cots = {"conv_state": np.zeros_like(out["conv_state"]), "q": dq, "k": dk, "v": dv, "g": dg, "beta": db}
    dc, _ = ref_adjoint("gdn_conv_prep", params, ops, fwd, cots)
    np.testing.assert_allclose(R.conv_prep_bwd(x, w, cu, Hg, H, dq, dk, dv, K), dc["x"], rtol=1e-9, atol=1e-11)
    da, dbg = R.gates_bwd(a, bg, a_log, dt_bias, cu, dg, db)
    np.testing.assert_allclose(da, dc["a"], rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(dbg, dc["b_gate"], rtol=1e-9, atol=1e-11)
