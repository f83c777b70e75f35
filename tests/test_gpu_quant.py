"""The w8a8 trunk's activation quantisers (r97b_quant_act_i8g / _bwd, csrc/quant.cu) against the
reference's own host rows of the quant family (src/adjoint/host/quant.cpp, compiled into oracle/_ref):
had_quant_act_i8g (rotated by the order-t Walsh-Hadamard matrix) and quant_act_i8g (plain), forward twin and
straight-through adjoint, at the shapes the reference's adjoint_quant test uses and at a trunk-sized case.

Bars (the reference's own, docs/adjoints/quant.md s2): scales within 2 bf16 ulps of the f64 twin (they
agree to f32 rounding); codes identical except at a rounding tie -- where v / s lies within 1e-4 of a
half-integer the f32 kernel and the f64 twin may round one code apart. The adjoint: rel L2 <= 1e-6 of the
host row's dx over every group whose clamp mask the f32 kernel and the f64 row agree on (the mask is |v / s|
> 127 at the amax element, which only the last bit of the reciprocal decides), and over every group against
W (m . g / s) under the kernel's own mask."""
import numpy as np
import pytest
import torch

import oracle
from oracle import Operand, ref_adjoint, ref_twin
from r97training_b200 import ops
from r97training_b200._lib import R97bError

pytestmark = pytest.mark.gpu


def _need_ref():
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")


def _fwht(v, t):
    """Unnormalised Walsh-Hadamard transform of every t-wide group of the last axis, the reference's loop
    order (ascending h, lower index = a + b), in v's own dtype."""
    v = v.copy()
    shp = v.shape
    g = v.reshape(-1, t)
    h = 1
    while h < t:
        blk = g.reshape(g.shape[0], t // (2 * h), 2, h)
        a, b = blk[:, :, 0, :].copy(), blk[:, :, 1, :].copy()
        blk[:, :, 0, :] = a + b
        blk[:, :, 1, :] = a - b
        h *= 2
    return g.reshape(shp)


def _ops(M, n, ngrp):
    return [Operand("x", "bf16", (M, n)), Operand("codes", "i8", (M, n), written=True),
            Operand("scale", "f32", (M, ngrp), written=True)]


def _params(M, n, t):
    return {"M": M, "n": n, "group": t, "dtype": "bf16"}


def _x(rs, M, n, dev):
    x = torch.from_numpy(rs.normal(size=(M, n)).astype(np.float32)).to(torch.bfloat16)
    x[:, 5 % n] *= 9.0  # one outlier column, the case the rotation exists for
    return x, x.float().numpy().astype(np.float64), x.to(dev)


CASES = [  # (rows, n, group, rotated): the reference test's shapes, group 0, a short last group, 256 wide
    (1, 64, 4, True), (2, 96, 32, True), (3, 128, 128, True), (4, 256, 64, True), (5, 128, 16, True),
    (8, 256, 256, True), (3, 64, 32, False), (1, 48, 16, False), (5, 128, 128, False), (2, 48, 32, False),
    (4, 96, 0, False), (6, 100, 7, False), (64, 4096, 128, True),
]


@pytest.mark.parametrize("case", CASES, ids=[f"{m}x{n}g{t}{'h' if r else 'p'}" for m, n, t, r in CASES])
def test_quant_forward_matches_reference_twin(cuda, case):
    _need_ref()
    M, n, t, rot = case
    op = "had_quant_act_i8g" if rot else "quant_act_i8g"
    te = t if (rot or 0 < t <= n) else n
    ngrp = -(-n // te)
    rs = np.random.RandomState(M * 1000 + n + t)
    x, x64, xd = _x(rs, M, n, cuda)
    want = ref_twin(op, _params(M, n, t), _ops(M, n, ngrp), {"x": x64})
    codes, scale = ops.quant_act_i8g(xd, t, rotate=rot)
    torch.cuda.synchronize()
    got_c, got_s = codes.cpu().numpy().astype(np.int64), scale.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(got_s, want["scale"], rtol=2.0 / 256, atol=0)
    assert np.max(np.abs(got_s / want["scale"] - 1)) < 1e-6  # in fact f32 rounding of the same value
    wc = want["codes"].astype(np.int64)
    bad = got_c != wc
    if bad.any():
        v = _fwht(x64, te) if rot else x64
        u = v / np.repeat(want["scale"], te, axis=1)[:, :n]
        frac = np.abs(np.abs(u[bad]) - np.floor(np.abs(u[bad])) - 0.5)
        assert np.all(np.abs(got_c[bad] - wc[bad]) == 1) and np.all(frac < 1e-4), \
            f"{bad.sum()} codes differ away from a rounding tie"
    assert bad.sum() <= max(2, bad.size // 1000)


def _mask32(x, scale, te, rot):
    v = _fwht(x.astype(np.float32), te) if rot else x.astype(np.float32)
    s = np.repeat(scale.astype(np.float32), te, axis=1)[:, :x.shape[1]]
    return np.abs(v * (np.float32(1.0) / s)) > np.float32(127.0)


@pytest.mark.parametrize("case", CASES, ids=[f"{m}x{n}g{t}{'h' if r else 'p'}" for m, n, t, r in CASES])
def test_quant_adjoint_matches_reference_row(cuda, case):
    _need_ref()
    M, n, t, rot = case
    op = "had_quant_act_i8g" if rot else "quant_act_i8g"
    te = t if (rot or 0 < t <= n) else n
    ngrp = -(-n // te)
    rs = np.random.RandomState(M * 7 + n + t)
    x, x64, xd = _x(rs, M, n, cuda)
    codes, scale = ops.quant_act_i8g(xd, t, rotate=rot)
    g = rs.normal(size=(M, n)).astype(np.float32)
    gd = torch.from_numpy(g).to(cuda)
    dx = ops.quant_act_i8g_bwd(xd, t, scale, gd, rotate=rot)
    prev = torch.from_numpy(rs.normal(size=(M, n)).astype(np.float32)).to(cuda)
    acc = ops.quant_act_i8g_bwd(xd, t, scale, gd, rotate=rot, dx=prev.clone(), accumulate=True)
    torch.cuda.synchronize()
    # the host row on the f64 twin's own forward (its scale), as the reference's walk runs it
    s_twin = ref_twin(op, _params(M, n, t), _ops(M, n, ngrp), {"x": x64})["scale"]
    dc, _ = ref_adjoint(op, _params(M, n, t), _ops(M, n, ngrp),
                        {"x": x64, "codes": codes.cpu().numpy().astype(np.float64), "scale": s_twin},
                        {"codes": g.astype(np.float64), "scale": rs.normal(size=(M, ngrp))})
    want = dc["x"]
    got = dx.cpu().numpy().astype(np.float64)
    # the clamp mask: the f64 row's, and the f32 kernel's (u = v * (1 / s) in f32 rounds outward at about a
    # fifth of the groups' amax elements, docs/adjoints/quant.md s1: 14 of 64 candidates; a few groups
    # sample that widely)
    v64 = _fwht(x64, te) if rot else x64
    m64 = np.abs(v64 * (1.0 / np.repeat(s_twin, te, axis=1)[:, :n])) > 127.0
    s32 = scale.cpu().numpy()
    m32 = _mask32(x.float().numpy(), s32, te, rot)
    diff_grp = np.zeros((M, ngrp), bool)
    for j in range(ngrp):
        diff_grp[:, j] = (m64[:, j * te:(j + 1) * te] != m32[:, j * te:(j + 1) * te]).any(axis=1)
    keep = ~np.repeat(diff_grp, te, axis=1)[:, :n]
    assert diff_grp.size < 32 or diff_grp.mean() <= 0.5
    if keep.any():
        err = np.linalg.norm((got - want)[keep]) / max(np.linalg.norm(want[keep]), 1e-30)
        assert err <= 1e-6, f"rel L2 {err:.3g} against the host row"
    # every group, against the same formula under the kernel's own mask
    d = np.where(m32, 0.0, g.astype(np.float64) / np.repeat(s32.astype(np.float64), te, axis=1)[:, :n])
    full = _fwht(d, te) if rot else d
    err = np.linalg.norm(got - full) / max(np.linalg.norm(full), 1e-30)
    assert err <= 1e-6, f"rel L2 {err:.3g} against W (m32 . g / s)"
    np.testing.assert_allclose(acc.cpu().numpy(), dx.cpu().numpy() + prev.cpu().numpy(), rtol=1e-6, atol=1e-6)


def test_quant_adjoint_is_the_rotation(cuda):
    """With scale 1 and nothing clamped, a cotangent at a group's first code comes back as W e0 (all ones),
    and a cotangent of one everywhere as (t, 0, ..., 0): W itself, not its transpose over t (quant.md s3)."""
    for t in (4, 32, 128, 256):
        n = 2 * t
        x = torch.zeros((1, n), dtype=torch.bfloat16, device=cuda)
        scale = torch.ones((1, 2), dtype=torch.float32, device=cuda)
        g = torch.zeros((1, n), dtype=torch.float32, device=cuda)
        g[0, 0] = 1.0
        g[0, t:] = 1.0
        dx = ops.quant_act_i8g_bwd(x, t, scale, g, rotate=True).cpu().numpy()[0]
        assert np.array_equal(dx[:t], np.ones(t, np.float32))
        want = np.zeros(t, np.float32)
        want[0] = t
        assert np.array_equal(dx[t:], want)


def test_quant_zero_group_and_clamp_mask(cuda):
    """An all-zero group has scale 1 and zero codes; the adjoint zeroes a clamped code's cotangent."""
    x = torch.zeros((2, 128), dtype=torch.bfloat16, device=cuda)
    x[1] = torch.linspace(-3, 3, 128, device=cuda).to(torch.bfloat16)
    codes, scale = ops.quant_act_i8g(x, 128, rotate=True)
    assert scale[0, 0].item() == 1.0 and not codes[0].any()
    assert int(codes[1].abs().max().item()) == 127
    # a scale a little below the true amax / 127 clamps the amax element: its cotangent is dropped
    s = scale.clone()
    s[1, 0] *= 0.999
    g = torch.zeros((2, 128), dtype=torch.float32, device=cuda)
    v = torch.from_numpy(_fwht(x.float().cpu().numpy(), 128)).to(cuda)
    j = int(v[1].abs().argmax().item())
    g[1, j] = 1.0
    dx = ops.quant_act_i8g_bwd(x, 128, s, g, rotate=True)
    assert not dx[1].any()


def test_quant_trunk_size_properties(cuda):
    """At a trunk activation's size (8192 tokens x 4096, groups of 128): every dequantised value lies within
    half a scale step of the rotated activation, and rotating the dequantised groups back (W q / t)
    recovers x to the quantiser's resolution."""
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn((8192, 4096), generator=g, device=cuda).to(torch.bfloat16)
    codes, scale = ops.quant_act_i8g(x, 128, rotate=True)
    torch.cuda.synchronize()
    xs = x[:512].float().cpu().numpy()
    v = _fwht(xs, 128)
    s = np.repeat(scale[:512].cpu().numpy(), 128, axis=1)
    q = codes[:512].cpu().numpy().astype(np.float32) * s
    assert np.all(np.abs(q - v) <= 0.5 * s * (1 + 1e-5))
    back = _fwht(q, 128) / 128.0
    err = np.linalg.norm(back - xs) / np.linalg.norm(xs)
    assert err < 0.02, err
    assert scale.min().item() > 0 and int(codes.abs().max().item()) == 127


def test_quant_rejects_bad_groups(cuda):
    x = torch.zeros((2, 96), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(R97bError):
        ops.quant_act_i8g(x, 64, rotate=True)   # 64 does not divide 96
    with pytest.raises(R97bError):
        ops.quant_act_i8g(x, 24, rotate=True)   # not a power of two
    with pytest.raises(R97bError):
        ops.quant_act_i8g(torch.zeros((1, 1024), dtype=torch.bfloat16, device=cuda), 512, rotate=True)


def test_quant_four_column_layout(cuda):
    """Rows whose pitch allows only 8-byte loads take the four-columns-a-lane layout; it agrees with the
    eight-column one bit for bit (same transform order, same arithmetic)."""
    rs = np.random.RandomState(11)
    M, n = 6, 256
    base = torch.from_numpy(rs.normal(size=(M, n + 4)).astype(np.float32)).to(torch.bfloat16).to(cuda)
    x4 = base[:, :n]                      # pitch n + 4: 8-byte rows only
    x8 = x4.contiguous()                  # pitch n: 16-byte rows
    g = torch.from_numpy(rs.normal(size=(M, n)).astype(np.float32)).to(cuda)
    for t in (4, 32, 128):
        c4, s4 = ops.quant_act_i8g(x4, t)
        c8, s8 = ops.quant_act_i8g(x8, t)
        assert torch.equal(c4, c8) and torch.equal(s4, s8)
        assert torch.equal(ops.quant_act_i8g_bwd(x4, t, s4, g), ops.quant_act_i8g_bwd(x8, t, s8, g))


@pytest.mark.parametrize("case", [(3, 128, 128, True), (4, 256, 64, True), (2, 96, 32, True), (6, 100, 7, False)],
                         ids=["3x128g128h", "4x256g64h", "2x96g32h", "6x100g7p"])
def test_quant_device_row_through_reference_registry(cuda, case):
    """The plugin's device row for the quant family (host/rows_quant.cpp), reached the way the reference's
    walk reaches it (adjoint_find(op, Side::device)), against the reference's own host row."""
    _need_ref()
    from tests.plugin_util import plugin
    assert plugin().r97host_registered() == 1
    M, n, t, rot = case
    op = "had_quant_act_i8g" if rot else "quant_act_i8g"
    te = t if (rot or 0 < t <= n) else n
    ngrp = -(-n // te)
    rs = np.random.RandomState(n + t)
    x, x64, xd = _x(rs, M, n, cuda)
    tw = ref_twin(op, _params(M, n, t), _ops(M, n, ngrp), {"x": x64})
    fwd = {"x": x64, "codes": tw["codes"], "scale": tw["scale"]}
    cots = {"codes": rs.normal(size=(M, n)), "scale": rs.normal(size=(M, ngrp))}
    host, _ = ref_adjoint(op, _params(M, n, t), _ops(M, n, ngrp), fwd, cots, side="host")
    dev, _ = ref_adjoint(op, _params(M, n, t), _ops(M, n, ngrp), fwd, cots, side="device")
    v64 = _fwht(x64, te) if rot else x64
    s = np.repeat(tw["scale"], te, axis=1)[:, :n]
    m64 = np.abs(v64 * (1.0 / s)) > 127.0
    m32 = _mask32(x.float().numpy(), tw["scale"].astype(np.float32), te, rot)
    same = np.ones((M, n), bool)
    for j in range(ngrp):
        agree = (m64[:, j * te:(j + 1) * te] == m32[:, j * te:(j + 1) * te]).all(axis=1)
        same[:, j * te:(j + 1) * te] = agree[:, None]
    assert same.any()
    err = np.linalg.norm((dev["x"] - host["x"])[same]) / np.linalg.norm(host["x"][same])
    assert err <= 1e-6, err
