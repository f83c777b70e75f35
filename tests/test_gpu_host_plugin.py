"""The drop-in boundary on the GPU: every device adjoint row the plugin (libr97host.so) registers into the
reference's own registry, run through that registry exactly as the reference's walk would find it
(adjoint_find(op, Side::device)), against the reference's own f64 host row for the same record. The bar is
the north star's: per-tensor relative L2 <= 1e-2 and cosine >= 0.999 for every cotangent and gradient
(gemm_nt_q at i8a8h included).
Also the plugin's HeadCeKernel against the reference's ce_position."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from oracle import Operand, ref_adjoint, ref_twin
from oracle import gdn as G
from oracle import rows as R
from tests.plugin_util import assert_parity, flush, plugin

pytestmark = pytest.mark.gpu


def bf16_round(x):
    """Values on the bf16 grid (round to nearest even), as a tape holds a bf16 operand."""
    f = np.ascontiguousarray(x, np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32).astype(np.float64).reshape(np.shape(x))


def both(op, params, ops, fwd, cots, **kw):
    plugin()
    host = ref_adjoint(op, params, ops, fwd, cots, side="host", **kw)
    dev = ref_adjoint(op, params, ops, fwd, cots, side="device", flush=flush, **kw)
    assert plugin().r97host_sync() == 0
    return host, dev


def _stored_weight(n, k, seed):
    rs = np.random.RandomState(seed)
    codes = rs.randint(-126, 127, size=(n, k)).astype(np.int8)
    sc = np.abs(rs.normal(0, 0.02, size=(n, k // 128))).astype(np.float32)
    bits = ((sc.view(np.uint32) + 0x7FFF + ((sc.view(np.uint32) >> 16) & 1)) >> 16).astype(np.uint16)
    return codes, bits


@pytest.mark.parametrize("stored", [True, False])
def test_gemm_nt_device_row(cuda, stored):
    M, N, K = 96, 384, 256
    rs = np.random.RandomState(1)
    x = bf16_round(rs.normal(size=(M, K)))
    dy = bf16_round(rs.normal(size=(M, N)) * 1e-2)
    codes, sbits = _stored_weight(N, K, 2)
    W = R.dequant_value(codes, sbits)
    b = Operand("b", "iqr", (N, K), stored=(codes, sbits)) if stored else Operand("b", "bf16", (N, K))
    ops = [Operand("a", "bf16", (M, K)), b, Operand("y", "bf16", (M, N), written=True)]
    params = {"M": M, "N": N, "K": K}
    fwd = {"a": x, "b": None if stored else bf16_round(W), "y": np.zeros((M, N))}
    (hdc, _), (ddc, _) = both("gemm_nt", params, ops, fwd, {"y": dy})
    assert np.abs(hdc["a"]).max() > 0
    assert_parity(ddc["a"], hdc["a"], "gemm_nt dX")


@pytest.mark.parametrize("stored", [False, True])
def test_gemm_nt_q_device_row(cuda, stored):
    """The int8 trunk's linear at i8a8h: dX = s_a (dY W) with W the codes times their group scale -- the
    tape's b_scale for a values weight, the stored plane's own bf16 scale for a stored one."""
    M, N, K = 96, 384, 384
    G = K // 128
    rs = np.random.RandomState(4)
    a = rs.randint(-127, 128, size=(M, K)).astype(np.float64)
    sa = np.abs(rs.normal(size=(M, G))) * 0.01 + 1e-4
    dy = bf16_round(rs.normal(size=(M, N)) * 1e-2)
    codes, sbits = _stored_weight(N, K, 5)
    sb = R.bf16_bits_to_f64(sbits) if stored else np.abs(rs.normal(size=(N, G))) * 0.002 + 1e-5
    b = Operand("b", "iqr", (N, K), stored=(codes, sbits)) if stored else Operand("b", "i8", (N, K))
    ops = [Operand("a", "i8", (M, K)), Operand("a_scale", "f32", (M, G)), b, Operand("b_scale", "f32", (N, G)),
           Operand("y", "bf16", (M, N), written=True)]
    params = {"M": M, "N": N, "K": K, "group": 128, "dtype": "i8a8h"}
    fwd = {"a": a, "a_scale": sa, "b": None if stored else codes.astype(np.float64), "b_scale": sb,
           "y": np.zeros((M, N))}
    (hdc, _), (ddc, _) = both("gemm_nt_q", params, ops, fwd, {"y": dy})
    assert np.abs(hdc["a"]).max() > 0
    assert_parity(ddc["a"], hdc["a"], "gemm_nt_q dX")


@pytest.mark.parametrize("part", ["rmsnorm", "silu_mul", "sigmoid_mul"])
def test_fused_quant_device_rows(cuda, part):
    """The int8 trunk's fused producers (rmsnorm_had_quant_i8g, gated_had_quant_i8g, gate_had_quant_i8g) on the
    records the reference's own quant test builds, with the `out` write's cotangent beside the codes'."""
    from tests.test_gpu_quant_fused import OPS, _near_clamp, _record
    rows, n, group = 24, 512, 128
    params, ops = _record(part, rows, n, group, 1 if part == "rmsnorm" else 0)
    rs = np.random.RandomState(9)
    if part == "rmsnorm":
        host = {"x": bf16_round(rs.normal(size=(rows, n))), "w": rs.normal(size=n) * 0.1}
    elif part == "silu_mul":
        host = {"gate_up": bf16_round(rs.normal(size=(rows, 2 * n)) * 2.0)}
    else:
        host = {"a": bf16_round(rs.normal(size=(rows, n)) * 2.0), "b": bf16_round(rs.normal(size=(rows, n)))}
    want = ref_twin(OPS[part], params, ops, host)
    fwd = dict(host)
    fwd.update({"codes": want["codes"], "scale": want["scale"], "out": want["out"]})
    g = rs.normal(size=(rows, n))
    g[_near_clamp(want["out"], want["scale"], group)] = 0.0  # the f32 and f64 masks may differ only there
    cots = {"codes": g, "scale": np.zeros_like(want["scale"]), "out": rs.normal(size=(rows, n)) * 0.1}
    (hdc, _), (ddc, _) = both(OPS[part], params, ops, fwd, cots)
    for name in ([r.buffer for r in ops if not r.written][:1 if part != "sigmoid_mul" else 2]):
        assert np.abs(hdc[name]).max() > 0
        assert_parity(ddc[name], hdc[name], f"{OPS[part]} d{name}")
    if part == "rmsnorm":
        assert not np.abs(ddc["w"]).any()  # the gain is frozen


@pytest.mark.parametrize("fused", [False, True])
def test_lora_device_rows(cuda, fused):
    M, K, N, r, S = 80, 256, 192, 16, 2
    rs = np.random.RandomState(3)
    x = bf16_round(rs.normal(size=(M, K)))
    A = rs.normal(size=(S, r, K)) / 4
    B = rs.normal(size=(S, N, r)) * 0.1
    scale = np.stack([np.full(N, 2.0), np.full(N, 0.5)])
    slot = rs.randint(-1, S, size=M).astype(np.float64)  # -1: base rows neither op touches
    sh_ops = [Operand("a", "bf16", (M, K)), Operand("none:1", "invalid", (0,)), Operand("slot", "i32", (M,)),
              Operand("lora_a", "f32", (S, r, K)), Operand("t", "f32", (M, r), written=True)]
    t = ref_twin("lora_shrink", {}, sh_ops, {"a": x, "none:1": None, "slot": slot, "lora_a": A})["t"]
    ex_ops = [Operand("t", "f32", (M, r)), Operand("slot", "i32", (M,)), Operand("lora_b", "f32", (S, N, r)),
              Operand("scale", "f32", (S, N)), Operand("y", "bf16", (M, N), written=True)]
    dy = bf16_round(rs.normal(size=(M, N)) * 1e-2)
    fwd = {"t": t, "slot": slot, "lora_b": B, "scale": scale, "y": np.zeros((M, N))}
    (hdc, hg), (ddc, dg) = both("lora_expand", {}, ex_ops, fwd, {"y": dy}, prefix="m", fused_slots=fused)
    assert_parity(ddc["t"], hdc["t"], "lora_expand dt")
    assert sorted(hg) == sorted(dg), (sorted(hg), sorted(dg))
    for name in hg:
        assert_parity(dg[name], hg[name], f"lora_expand {name}")
    dt = hdc["t"]
    fwd = {"a": x, "none:1": None, "slot": slot, "lora_a": A, "t": t}
    (hdc, hg), (ddc, dg) = both("lora_shrink", {}, sh_ops, fwd, {"t": dt}, prefix="m", fused_slots=fused)
    assert_parity(ddc["a"], hdc["a"], "lora_shrink dx")
    base = slot < 0
    assert np.all(ddc["a"][base] == 0) and np.all(hdc["a"][base] == 0)
    assert sorted(hg) == sorted(dg)
    for name in hg:
        assert_parity(dg[name], hg[name], f"lora_shrink {name}")


@pytest.mark.parametrize("wadd,mult", [(0.0, 1.0), (1.0, 0.5)])
def test_rmsnorm_device_row(cuda, wadd, mult):
    rows, n = 64, 512
    rs = np.random.RandomState(4)
    x = bf16_round(rs.normal(size=(rows, n)))
    w = rs.normal(size=(n,)) * 0.1
    dy = bf16_round(rs.normal(size=(rows, n)))
    ops = [Operand("x", "bf16", (rows, n)), Operand("w", "f32", (n,)), Operand("y", "bf16", (rows, n), written=True)]
    params = {"eps": "1e-06", "wadd": repr(wadd), "mult": repr(mult)}
    (hdc, _), (ddc, _) = both("rmsnorm", params, ops, {"x": x, "w": w, "y": np.zeros((rows, n))}, {"y": dy})
    assert_parity(ddc["x"], hdc["x"], "rmsnorm dx")


@pytest.mark.parametrize("act", ["silu", "sigmoid"])
def test_gated_rmsnorm_device_row(cuda, act):
    rows, n = 96, 128
    rs = np.random.RandomState(5)
    x, z, do = (bf16_round(rs.normal(size=(rows, n))) for _ in range(3))
    w = rs.normal(size=(n,))
    ops = [Operand("x", "bf16", (rows, n)), Operand("z", "bf16", (rows, n)), Operand("w", "f32", (n,)),
           Operand("o", "bf16", (rows, n), written=True)]
    params = {"channels": n, "act": act}
    fwd = {"x": x, "z": z, "w": w, "o": np.zeros((rows, n))}
    (hdc, _), (ddc, _) = both("gdn_gated_rmsnorm", params, ops, fwd, {"o": do})
    assert_parity(ddc["x"], hdc["x"], "gated dx")
    assert_parity(ddc["z"], hdc["z"], "gated dz")


def _gdn_case(seed, lens=(100, 64, 30), H=4, Hg=2):
    d = G.synth_inputs(list(lens), H, Hg, 128, 128, seed=seed)
    for key in ("q", "k", "v"):
        d[key] = bf16_round(d[key])
    return d


def test_gdn_kkt_device_row(cuda):
    d = _gdn_case(11)
    T, H, Hg, S = d["q"].shape[0], 4, 2, len(d["cu"]) - 1
    ops = [Operand("k", "bf16", (T, Hg, 128)), Operand("beta", "f32", (T, H)), Operand("g", "f32", (T, H)),
           Operand("cu_seqlens", "i32", (S + 1,)), Operand("A", "bf16", (T, H, 64), written=True)]
    params = {"chunk": 64, "head_k": 128}
    reads = {"k": d["k"], "beta": d["beta"], "g": d["g"], "cu_seqlens": d["cu"]}
    A = ref_twin("gdn_kkt_solve", params, ops, reads)["A"]
    dA = np.tril(np.random.RandomState(12).normal(size=A.shape)) * 0.1
    (hdc, _), (ddc, _) = both("gdn_kkt_solve", params, ops, dict(reads, A=A), {"A": dA})
    for name in ("k", "beta", "g"):
        assert_parity(ddc[name], hdc[name], f"kkt d{name}")


def test_gdn_chunk_scan_device_row(cuda):
    d = _gdn_case(21)
    T, H, Hg, S = d["q"].shape[0], 4, 2, len(d["cu"]) - 1
    rs = np.random.RandomState(22)
    slots = S + 1
    h0 = rs.normal(size=(slots, H, 128, 128)) * 0.05
    dht = rs.normal(size=(slots, H, 128, 128)) * 1e-3
    sidx = np.array([2, 0, 3][:S], dtype=np.float64)  # sequences own permuted state slots
    A = ref_twin("gdn_kkt_solve", {"chunk": 64, "head_k": 128},
                 [Operand("k", "bf16", (T, Hg, 128)), Operand("beta", "f32", (T, H)), Operand("g", "f32", (T, H)),
                  Operand("cu_seqlens", "i32", (S + 1,)), Operand("A", "bf16", (T, H, 64), written=True)],
                 {"k": d["k"], "beta": d["beta"], "g": d["g"], "cu_seqlens": d["cu"]})["A"]
    A = bf16_round(A)
    ops = [Operand("q", "bf16", (T, Hg, 128)), Operand("k", "bf16", (T, Hg, 128)), Operand("v", "bf16", (T, H, 128)),
           Operand("A", "bf16", (T, H, 64)), Operand("g", "f32", (T, H)), Operand("beta", "f32", (T, H)),
           Operand("h0", "f32", (slots, H, 128, 128)), Operand("cu_seqlens", "i32", (S + 1,)),
           Operand("o", "bf16", (T, H, 128), written=True), Operand("ht", "f32", (slots, H, 128, 128), written=True),
           Operand("state_idx", "i32", (S,))]
    params = {"head_k": 128, "head_v": 128, "chunk": 64, "scale": repr(1.0 / np.sqrt(128))}
    reads = {"q": d["q"], "k": d["k"], "v": d["v"], "A": A, "g": d["g"], "beta": d["beta"], "h0": h0,
             "cu_seqlens": d["cu"], "state_idx": sidx}
    out = ref_twin("gdn_chunk_scan", params, ops, reads)
    fwd = dict(reads, o=out["o"], ht=out["ht"])
    do = bf16_round(d["do"])
    (hdc, _), (ddc, _) = both("gdn_chunk_scan", params, ops, fwd, {"o": do, "ht": dht})
    for name in ("q", "k", "v", "A", "g", "beta"):
        assert np.abs(hdc[name]).max() > 0, name
        assert_parity(ddc[name], hdc[name], f"scan d{name}")


class HeadChunk(ctypes.Structure):
    """The reference's r97::HeadChunk (include/r97/head.h:35-44)."""
    _fields_ = [("logits", ctypes.c_void_p), ("grad", ctypes.c_void_p), ("loss", ctypes.c_void_p),
                ("ids", ctypes.c_void_p), ("positions", ctypes.c_int64), ("vocab", ctypes.c_int64),
                ("grad_scale", ctypes.c_float), ("stream", ctypes.c_void_p)]


@pytest.mark.parametrize("vocab", [1024, 1003])
def test_head_ce_kernel(cuda, vocab):
    rows = 40
    g = torch.Generator().manual_seed(7)
    logits = (torch.randn(rows, vocab, generator=g) * 2).bfloat16()
    ids = torch.randint(0, vocab, (rows,), generator=g, dtype=torch.int32)
    ids[::5] = -1
    x = logits.to(cuda)
    grad = torch.empty_like(x)
    loss = torch.empty(rows, device=cuda)
    idd = ids.to(cuda)
    chunk = HeadChunk(x.data_ptr(), grad.data_ptr(), loss.data_ptr(), idd.data_ptr(), rows, vocab, 1.0 / 32,
                      torch.cuda.current_stream().cuda_stream)
    err = ctypes.c_char_p()
    assert plugin().r97host_head_ce(ctypes.byref(chunk), ctypes.byref(err)) == 0, err.value
    torch.cuda.synchronize()
    lib = oracle.ref_lib()
    xs = logits.float().numpy()
    ref_loss = np.zeros(rows)
    ref_grad = np.zeros((rows, vocab), np.float32)
    for r in range(rows):
        if ids[r] < 0:
            continue
        row = np.ascontiguousarray(xs[r])
        gr = np.zeros(vocab, np.float32)
        ref_loss[r] = lib.ref_ce_position(row.ctypes.data, vocab, int(ids[r]), gr.ctypes.data, 1.0 / 32)
        ref_grad[r] = gr
    np.testing.assert_allclose(loss.cpu().numpy(), ref_loss, rtol=1e-4, atol=1e-4)
    assert_parity(grad.float().cpu().numpy(), ref_grad, "head CE grad")
    assert np.all(grad.float().cpu().numpy()[ids.numpy() < 0] == 0)
