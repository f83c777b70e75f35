"""The gated-attention restatements (oracle/rows.py: attention_fwd/_bwd, rope_fwd/_bwd, gate_fwd/_bwd and
the per-head q/k RMSNorm) pinned against the reference's own compiled rows: the `attn_paged` twin and host
adjoint (src/adjoint/host/attention.cpp) over a pool that holds each sequence's keys at their positions
(one block per sequence), the `rope` twin and adjoint (rope.cpp over qk.cpp's table and rotation), the
`rmsnorm` row on head-wide rows and the `sigmoid` / `mul` rows of the output gate. CPU only."""
import numpy as np
import pytest

import oracle
from oracle import Operand, ref_adjoint, ref_twin
from oracle import rows as R


def _need_ref():
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")


def _attn_record(lens, Hq, Hkv, D, with_cu=True):
    S, T, blk = len(lens), sum(lens), max(lens)
    ops = [Operand("q", "bf16", (T, Hq, D)), Operand("kv", "bf16", (S, Hkv, blk, 2 * D)),
           Operand("block_table", "i32", (S, 1)), Operand("seqused", "i32", (S,)),
           Operand("none:4", "invalid", ()), Operand("none:5", "invalid", ())]
    ops.append(Operand("cu_seqlens", "i32", (S + 1,)) if with_cu else Operand("none:6", "invalid", ()))
    ops.append(Operand("out", "bf16", (T, Hq, D), written=True))
    return ops


def _pool(k, v, lens):
    """The paged pool [sequence block, kv head, slot, k | v] with sequence s's key j at slot j of block s."""
    S, blk, Hkv, D = len(lens), max(lens), k.shape[1], k.shape[2]
    kv = np.zeros((S, Hkv, blk, 2 * D))
    cu = np.concatenate([[0], np.cumsum(lens)])
    for s in range(S):
        a, b = cu[s], cu[s + 1]
        kv[s, :, :b - a, :D] = k[a:b].transpose(1, 0, 2)
        kv[s, :, :b - a, D:] = v[a:b].transpose(1, 0, 2)
    return kv, cu


@pytest.mark.parametrize("lens,Hq,Hkv,D", [((37, 64, 5), 4, 2, 32), ((48,), 2, 2, 16), ((20, 33), 6, 1, 24)])
def test_attention_twin_and_adjoint_vs_reference(lens, Hq, Hkv, D):
    _need_ref()
    rs = np.random.RandomState(sum(lens) + Hq)
    T = sum(lens)
    q, k, v = rs.normal(size=(T, Hq, D)), rs.normal(size=(T, Hkv, D)), rs.normal(size=(T, Hkv, D))
    dy = rs.normal(size=(T, Hq, D)) * 0.1
    kv, cu = _pool(k, v, lens)
    S = len(lens)
    reads = {"q": q, "kv": kv, "block_table": np.arange(S)[:, None], "seqused": np.array(lens),
             "none:4": None, "none:5": None, "cu_seqlens": cu}
    ops = _attn_record(lens, Hq, Hkv, D)
    out = ref_twin("attn_paged", {}, ops, reads)["out"]
    np.testing.assert_allclose(R.attention_fwd(q, k, v, cu=cu), out, rtol=1e-10, atol=1e-12)
    dc, _ = ref_adjoint("attn_paged", {}, ops, dict(reads, out=out), {"out": dy})
    dq, dk, dv = R.attention_bwd(q, k, v, dy, cu=cu)
    np.testing.assert_allclose(dq, dc["q"], rtol=1e-9, atol=1e-12)
    dkv, _ = _pool(dk, dv, lens)
    np.testing.assert_allclose(dkv, dc["kv"], rtol=1e-9, atol=1e-12)


def test_attention_equal_lengths_without_cu_seqlens():
    """Sequences of one length need no cu_seqlens: rows are split evenly (attention.cpp Call::row_of)."""
    _need_ref()
    lens, Hq, Hkv, D = (40, 40), 4, 1, 16
    rs = np.random.RandomState(3)
    T = sum(lens)
    q, k, v = rs.normal(size=(T, Hq, D)), rs.normal(size=(T, Hkv, D)), rs.normal(size=(T, Hkv, D))
    kv, cu = _pool(k, v, lens)
    reads = {"q": q, "kv": kv, "block_table": np.arange(2)[:, None], "seqused": np.array(lens),
             "none:4": None, "none:5": None, "none:6": None}
    out = ref_twin("attn_paged", {}, _attn_record(lens, Hq, Hkv, D, with_cu=False), reads)["out"]
    np.testing.assert_allclose(R.attention_fwd(q, k, v, cu=cu), out, rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("heads,D,rot,theta", [(4, 32, 16, 1e4), (2, 64, 64, 1e7), (3, 256, 64, 1e7)])
def test_rope_twin_and_adjoint_vs_reference(heads, D, rot, theta):
    _need_ref()
    rs = np.random.RandomState(heads * D + rot)
    T = 50
    pos = np.concatenate([np.arange(30), np.arange(20)])  # two sequences, positions restart
    x = rs.normal(size=(T, heads * D))
    dy = rs.normal(size=(T, heads * D))
    ops = [Operand("x", "bf16", (T, heads * D), written=True, in_place=True), Operand("pos", "i32", (T,))]
    params = {"M": 64, "head_dim": D, "rotary_dim": rot, "n_head": heads, "n_head_kv": 0, "theta": repr(theta),
              "scale": "1"}
    y = ref_twin("rope", params, ops, {"x": x, "pos": pos})["x"]
    np.testing.assert_allclose(R.rope_fwd(x, pos, rot, theta, D), y, rtol=1e-12, atol=1e-12)
    dc, _ = ref_adjoint("rope", params, ops, {"x": x, "pos": pos}, {"x": dy})
    np.testing.assert_allclose(R.rope_bwd(dy, pos, rot, theta, D), dc["x"], rtol=1e-12, atol=1e-12)


def test_qk_head_rmsnorm_vs_reference():
    """The q/k norm: the rmsnorm row over head-wide rows [T * heads, D] with one gain of D."""
    _need_ref()
    rs = np.random.RandomState(8)
    rows, D = 3 * 4, 64
    x, w, dy = rs.normal(size=(rows, D)), 1 + 0.1 * rs.normal(size=D), rs.normal(size=(rows, D))
    ops = [Operand("x", "bf16", (rows, D)), Operand("w", "f32", (D,)), Operand("y", "bf16", (rows, D), written=True)]
    params = {"eps": "1e-06", "n": D}
    y = ref_twin("rmsnorm", params, ops, {"x": x, "w": w})["y"]
    np.testing.assert_allclose(R.rmsnorm_fwd(x, w), y, rtol=1e-12)
    dc, _ = ref_adjoint("rmsnorm", params, ops, {"x": x, "w": w, "y": y}, {"y": dy})
    np.testing.assert_allclose(R.rmsnorm_bwd(x, w, dy), dc["x"], rtol=1e-10, atol=1e-12)


def test_output_gate_vs_reference():
    """sigmoid(gate) then mul: the gated attention's output gate, forward and both cotangents."""
    _need_ref()
    rs = np.random.RandomState(9)
    M, n = 24, 48
    o, gate, dy = rs.normal(size=(M, n)), rs.normal(size=(M, n)) * 2, rs.normal(size=(M, n))
    sg_ops = [Operand("gate", "bf16", (M, n)), Operand("sg", "bf16", (M, n), written=True)]
    sg = ref_twin("sigmoid", {"M": M, "n": n}, sg_ops, {"gate": gate})["sg"]
    mul_ops = [Operand("o", "bf16", (M, n)), Operand("sg", "bf16", (M, n)), Operand("y", "bf16", (M, n), written=True)]
    y = ref_twin("mul", {"M": M, "n": n}, mul_ops, {"o": o, "sg": sg})["y"]
    np.testing.assert_allclose(R.gate_fwd(o, gate), y, rtol=1e-12)
    dc, _ = ref_adjoint("mul", {"M": M, "n": n}, mul_ops, {"o": o, "sg": sg, "y": y}, {"y": dy})
    dc2, _ = ref_adjoint("sigmoid", {"M": M, "n": n}, sg_ops, {"gate": gate, "sg": sg}, {"sg": dc["sg"]})
    do, dgate = R.gate_bwd(o, gate, dy)
    np.testing.assert_allclose(do, dc["o"], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(dgate, dc2["gate"], rtol=1e-10, atol=1e-14)


def test_ce_large_offset_row_vs_reference():
    """A logit row whose maximum is large: the loss keeps log(s) (computed as log(s) - (x_t - m))."""
    import ctypes  # noqa: F401
    lib = oracle.ref_lib() if oracle.ref_available() else pytest.skip("no reference")
    rs = np.random.RandomState(10)
    vocab = 4096
    x = (rs.normal(size=vocab) * 0.01 + 3.0e4).astype(np.float32)
    tgt = 17
    loss, _ = R.ce_rows(x[None].astype(np.float64), np.array([tgt]))
    g = np.zeros(vocab, np.float32)
    want = lib.ref_ce_position(x.ctypes.data, vocab, tgt, g.ctypes.data, 1.0)
    assert abs(loss[0] - want) <= 1e-9 * abs(want), (loss[0], want)
