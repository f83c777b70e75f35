"""The int8 trunk's fused producers (r97b_fused_quant_i8g / _bwd, csrc/quant.cu) against the reference's own
host rows, compiled into oracle/_ref: rmsnorm_had_quant_i8g, gated_had_quant_i8g and gate_had_quant_i8g
(src/adjoint/host/quant.cpp:821-1100, the records of tests/host/adjoint_quant.cpp:724-760: the reads, then the
codes, the scale and the part's `out`).

Bars. Forward: the scales within 1e-5 of the f64 twin's (the f32 part and its f32 rotation); codes identical
except one apart at a rounding tie (v / s within 2e-3 of a half-integer), at most 1 in 1000; `out` within one
bf16 step of the twin's intermediate. Adjoint: rel L2 <= 1e-5 against the host row, twice: with the scale
raised 1 % above the forward's (no code sits on the clamp, in the f32 kernel or the f64 row, and the
straight-through map is the whole adjoint), and with the forward's own scale and the codes' cotangent zero at
the elements within 1e-4 of the clamp (a group's amax element lands on |v / s| = 127 to a few ulps, and the
f32 kernel and the f64 row decide its mask differently -- as the reference's own f32 device kernel does; a
zero cotangent there makes the decision immaterial)."""
import numpy as np
import pytest
import torch

import oracle
from oracle import Operand, ref_adjoint, ref_twin
from r97training_b200 import ops

pytestmark = pytest.mark.gpu


def _need_ref():
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")


def _bf(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16)


OPS = {"rmsnorm": "rmsnorm_had_quant_i8g", "silu_mul": "gated_had_quant_i8g", "sigmoid_mul": "gate_had_quant_i8g"}


def _record(part, rows, n, group, wadd):
    ngrp = n // group
    params = {"M": rows, "n": n, "group": group, "dtype": "bf16"}
    if part == "rmsnorm":
        params.update({"eps": "1e-6", "wadd": wadd})
        reads = [Operand("x", "bf16", (rows, n)), Operand("w", "f32", (n,))]
    elif part == "silu_mul":
        params["act"] = "silu"
        reads = [Operand("gate_up", "bf16", (rows, 2 * n))]
    else:
        params["act"] = "sigmoid"
        reads = [Operand("a", "bf16", (rows, n)), Operand("b", "bf16", (rows, n))]
    writes = [Operand("codes", "i8", (rows, n), written=True), Operand("scale", "f32", (rows, ngrp), written=True),
              Operand("out", "bf16", (rows, n), written=True)]
    return params, reads + writes


def _inputs(part, rows, n, seed, cuda):
    """(host f64 reads by buffer, device tensors: x, x2, w)."""
    rs = np.random.RandomState(seed)
    if part == "rmsnorm":
        x = _bf(rs.normal(size=(rows, n)))
        x[:, 3] *= 8.0
        w = torch.from_numpy((rs.normal(size=n) * 0.1).astype(np.float32))
        return {"x": x.double().numpy(), "w": w.double().numpy()}, (x.to(cuda), None, w.to(cuda))
    if part == "silu_mul":
        gu = _bf(rs.normal(size=(rows, 2 * n)) * 2.0)
        return {"gate_up": gu.double().numpy()}, (gu.to(cuda), None, None)
    a, b = _bf(rs.normal(size=(rows, n)) * 2.0), _bf(rs.normal(size=(rows, n)))
    return {"a": a.double().numpy(), "b": b.double().numpy()}, (a.to(cuda), b.to(cuda), None)


def _fwht(v, t):
    v = v.copy()
    g = v.reshape(-1, t)
    h = 1
    while h < t:
        blk = g.reshape(g.shape[0], t // (2 * h), 2, h)
        x0, x1 = blk[:, :, 0, :].copy(), blk[:, :, 1, :].copy()
        blk[:, :, 0, :] = x0 + x1
        blk[:, :, 1, :] = x0 - x1
        h *= 2
    return g.reshape(v.shape)


CASES = [("rmsnorm", 4, 256, 128, 1), ("rmsnorm", 9, 1024, 64, 0), ("rmsnorm", 3, 4096, 128, 1),
         ("silu_mul", 5, 512, 128, 0), ("silu_mul", 2, 768, 256, 0), ("sigmoid_mul", 6, 256, 32, 0),
         ("sigmoid_mul", 3, 1024, 128, 0)]
IDS = [f"{p}-{r}x{n}g{t}" for p, r, n, t, _ in CASES]


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_fused_forward_matches_reference_twin(cuda, case):
    _need_ref()
    part, rows, n, group, wadd = case
    params, ops_ = _record(part, rows, n, group, wadd)
    host, (x, x2, w) = _inputs(part, rows, n, rows * 31 + n, cuda)
    want = ref_twin(OPS[part], params, ops_, host)
    codes, scale, out = ops.fused_quant_i8g(part, x, group, x2=x2, w=w, wadd=float(wadd))
    torch.cuda.synchronize()
    got_s = scale.cpu().numpy().astype(np.float64)
    assert np.max(np.abs(got_s / want["scale"] - 1)) < 1e-5
    y = want["out"]
    ref_b = _bf(y).float().numpy()
    tol = np.abs(ref_b) * 2.0 ** -7 + 1e-6 * np.abs(y).max()
    assert np.all(np.abs(out.float().cpu().numpy() - ref_b) <= tol)
    wc, gc = want["codes"].astype(np.int64), codes.cpu().numpy().astype(np.int64)
    bad = gc != wc
    if bad.any():
        u = _fwht(y, group) / np.repeat(want["scale"], group, axis=1)
        frac = np.abs(np.abs(u[bad]) - np.floor(np.abs(u[bad])) - 0.5)
        assert np.all(np.abs(gc[bad] - wc[bad]) == 1) and np.all(frac < 2e-3), \
            f"{bad.sum()} codes differ away from a rounding tie"
    assert bad.sum() <= max(2, bad.size // 1000)


def _near_clamp(y, scale, group):
    """Where |W y / s| lies within 1e-4 of 127: the elements whose mask the f32 and f64 forms may decide
    differently."""
    u = _fwht(y, group) / np.repeat(scale, group, axis=1)
    return np.abs(u) > 127.0 * (1 - 1e-4)


def _adjoint(part, rows, n, group, wadd, cuda, raise_scale):
    params, ops_ = _record(part, rows, n, group, wadd)
    host, (x, x2, w) = _inputs(part, rows, n, rows * 17 + n + 1, cuda)
    want = ref_twin(OPS[part], params, ops_, host)
    scale = want["scale"] * (1.01 if raise_scale else 1.0)
    rs = np.random.RandomState(n + rows)
    g = rs.normal(size=(rows, n))
    if not raise_scale:
        g[_near_clamp(want["out"], scale, group)] = 0.0
    go = rs.normal(size=(rows, n)) * 0.1
    fwd = dict(host)
    fwd.update({"codes": want["codes"], "scale": scale, "out": want["out"]})
    dc, _ = ref_adjoint(OPS[part], params, ops_, fwd, {"codes": g, "scale": np.zeros_like(scale), "out": go})
    sd = torch.from_numpy(scale.astype(np.float32)).to(cuda)
    gd = torch.from_numpy(g.astype(np.float32)).to(cuda)
    god = torch.from_numpy(go.astype(np.float32)).to(cuda)
    dx, dx2 = ops.fused_quant_i8g_bwd(part, x, group, sd, gd, g_out=god, x2=x2, w=w, wadd=float(wadd))
    torch.cuda.synchronize()
    got = {"rmsnorm": {"x": dx}, "silu_mul": {"gate_up": dx}, "sigmoid_mul": {"a": dx, "b": dx2}}[part]
    return {k: (v.cpu().numpy().astype(np.float64), dc[k]) for k, v in got.items()}


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_fused_adjoint_matches_reference_row(cuda, case):
    _need_ref()
    part, rows, n, group, wadd = case
    for raise_scale in (True, False):
        for name, (mine, ref) in _adjoint(part, rows, n, group, wadd, cuda, raise_scale).items():
            assert np.abs(ref).max() > 0
            err = np.linalg.norm(mine - ref) / np.linalg.norm(ref)
            assert err <= 1e-5, f"{name} (scale {'raised' if raise_scale else 'as written'}): rel L2 {err:.3g}"
