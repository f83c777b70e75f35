"""The numpy GDN restatement (oracle/gdn.py) pinned against the reference's own compiled
gdn_kkt_solve / gdn_chunk_scan twins and host adjoints, on ragged sequences with a short last chunk,
grouped heads (H = 2 Hg) and a non-zero initial state. CPU only."""
import numpy as np
import pytest

import oracle
from oracle import Operand, ref_adjoint, ref_twin
from oracle import gdn as G


def _need_ref():
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")


def _case(seed=0, K=32, V=32, chunk=16, H=4, Hg=2, lens=(40, 16, 7)):
    d = G.synth_inputs(list(lens), H, Hg, K, V, seed=seed)
    # re-accumulate g within chunks of `chunk` (synth_inputs accumulates over 64)
    rs = np.random.RandomState(seed + 1)
    inc = -np.log1p(np.exp(rs.normal(size=d["g"].shape)))
    cu = d["cu"]
    for s in range(len(lens)):
        for c0 in range(0, lens[s], chunk):
            r = slice(cu[s] + c0, cu[s] + min(lens[s], c0 + chunk))
            d["g"][r] = np.cumsum(inc[r], axis=0)
    d["h0"] = rs.normal(size=(len(lens), H, V, K)) * 0.1
    d["dht"] = rs.normal(size=(len(lens), H, V, K)) * 0.01
    return d, dict(K=K, V=V, chunk=chunk, H=H, Hg=Hg)


def _kkt_ops(T, H, Hg, K, chunk, S):
    return [Operand("k", "bf16", (T, Hg, K)), Operand("beta", "f32", (T, H)), Operand("g", "f32", (T, H)),
            Operand("cu_seqlens", "i32", (S + 1,)), Operand("A", "bf16", (T, H, chunk), written=True)]


def _scan_ops(T, H, Hg, K, V, chunk, S):
    return [Operand("q", "bf16", (T, Hg, K)), Operand("k", "bf16", (T, Hg, K)), Operand("v", "bf16", (T, H, V)),
            Operand("A", "bf16", (T, H, chunk)), Operand("g", "f32", (T, H)), Operand("beta", "f32", (T, H)),
            Operand("h0", "f32", (S, H, V, K)), Operand("cu_seqlens", "i32", (S + 1,)),
            Operand("o", "bf16", (T, H, V), written=True), Operand("ht", "f32", (S, H, V, K), written=True),
            Operand("state_idx", "i32", (S,))]


def test_kkt_twin_and_adjoint_vs_reference():
    _need_ref()
    d, p = _case()
    T, S = d["q"].shape[0], len(d["cu"]) - 1
    ops = _kkt_ops(T, p["H"], p["Hg"], p["K"], p["chunk"], S)
    params = {"chunk": p["chunk"], "head_k": p["K"]}
    A_ref = ref_twin("gdn_kkt_solve", params, ops, {"k": d["k"], "beta": d["beta"], "g": d["g"],
                                                   "cu_seqlens": d["cu"]})["A"]
    A = G.kkt_fwd(d["k"], d["beta"], d["g"], d["cu"], p["chunk"])
    np.testing.assert_allclose(A, A_ref, rtol=1e-10, atol=1e-12)
    dA = np.random.RandomState(3).normal(size=A.shape)
    dc, _ = ref_adjoint("gdn_kkt_solve", params, ops, {"k": d["k"], "beta": d["beta"], "g": d["g"],
                                                       "cu_seqlens": d["cu"], "A": A_ref}, {"A": dA})
    dk, db, dg = G.kkt_bwd(d["k"], d["beta"], d["g"], d["cu"], A, dA, p["chunk"])
    np.testing.assert_allclose(dk, dc["k"], rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(db, dc["beta"], rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(dg, dc["g"], rtol=1e-9, atol=1e-11)


def test_scan_twin_and_adjoint_vs_reference():
    _need_ref()
    d, p = _case(seed=5)
    T, S = d["q"].shape[0], len(d["cu"]) - 1
    K, V, H, Hg, chunk = p["K"], p["V"], p["H"], p["Hg"], p["chunk"]
    A = G.kkt_fwd(d["k"], d["beta"], d["g"], d["cu"], chunk)
    ops = _scan_ops(T, H, Hg, K, V, chunk, S)
    scale = 1.0 / np.sqrt(K)
    params = {"head_k": K, "head_v": V, "chunk": chunk, "scale": repr(scale)}
    sidx = np.arange(S)
    reads = {"q": d["q"], "k": d["k"], "v": d["v"], "A": A, "g": d["g"], "beta": d["beta"], "h0": d["h0"],
             "cu_seqlens": d["cu"], "state_idx": sidx}
    out = ref_twin("gdn_chunk_scan", params, ops, reads)
    o, ht = G.scan_fwd(d["q"], d["k"], d["v"], A, d["g"], d["beta"], d["cu"], d["h0"], scale, chunk)
    np.testing.assert_allclose(o, out["o"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(ht, out["ht"], rtol=1e-9, atol=1e-12)
    fwd = dict(reads, o=out["o"], ht=out["ht"])
    dc, _ = ref_adjoint("gdn_chunk_scan", params, ops, fwd, {"o": d["do"], "ht": d["dht"]})
    dq, dk, dv, dA, dg, db, dh0 = G.scan_bwd(d["q"], d["k"], d["v"], A, d["g"], d["beta"], d["cu"], d["do"],
                                             d["dht"], d["h0"], scale, chunk)
    for name, mine in (("q", dq), ("k", dk), ("v", dv), ("A", dA), ("g", dg), ("beta", db)):
        np.testing.assert_allclose(mine, dc[name], rtol=1e-8, atol=1e-11, err_msg=name)


def test_scan_finite_difference():
    """The composed adjoint against central differences of the composed twin (f64)."""
    d, p = _case(seed=9, K=8, V=8, chunk=4, H=2, Hg=1, lens=(6, 3))
    chunk = p["chunk"]
    d["h0"] = None
    res = G.layer_fwd_bwd(d["q"], d["k"], d["v"], d["g"], d["beta"], d["cu"], d["do"], chunk=chunk)

    def loss(q, k, v, g, beta):
        A = G.kkt_fwd(k, beta, g, d["cu"], chunk)
        o, _ = G.scan_fwd(q, k, v, A, g, beta, d["cu"], None, None, chunk)
        return float((o * d["do"]).sum())

    args = dict(q=d["q"], k=d["k"], v=d["v"], g=d["g"], beta=d["beta"])
    rs = np.random.RandomState(0)
    for name, key in (("q", "dq"), ("k", "dk"), ("v", "dv"), ("g", "dg"), ("beta", "dbeta")):
        x = args[name]
        for _ in range(3):
            idx = tuple(rs.randint(0, s) for s in x.shape)
            eps = 1e-6
            xp, xm = x.copy(), x.copy()
            xp[idx] += eps
            xm[idx] -= eps
            a1 = dict(args, **{name: xp})
            a2 = dict(args, **{name: xm})
            fd = (loss(**a1) - loss(**a2)) / (2 * eps)
            assert abs(fd - res[key][idx]) <= 1e-6 + 1e-5 * abs(fd), (name, idx, fd, res[key][idx])
