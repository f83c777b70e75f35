"""The w8a8 trunk's int8 product on tcgen05 (r97b_gemm_i8g, r97b_gemm_i8g_gated; csrc/gemm_i8.cu) against
the reference's own twins, compiled into oracle/_ref: gemm_nt_q at dtype i8a8h (src/adjoint/host/linear.cpp:
246-282) and the gated narrow fold gemm_nt_q_gated (src/adjoint/host/gemm_nt_q_gated.cpp:256-320), on ragged
shapes (rows past a tile, a short last K group, columns past a tile), and at a trunk-sized shape against the
same grouped formula evaluated exactly in torch (each group's integer product is exact in f32).

Bars: the plain product within 2e-6 of the largest |y| of the f64 twin (its groups' s32 sums are exact; the
f32 fold over at most 32 groups and the scales' products round at about 1e-7). The fold: the quantiser's
scales within 1e-5 relative; codes identical except one apart where v / s lies within 2e-3 of a rounding tie
(the f32 product and its f32 rotation against the twin's f64), at most 1 in 1000; the unrotated product as
bf16 within one bf16 step of the twin's, or 1e-6 of its row's largest value where the groups cancel."""
import numpy as np
import pytest
import torch

import oracle
from oracle import Operand, ref_twin
from r97training_b200 import ops
from r97training_b200._lib import R97bError

pytestmark = pytest.mark.gpu


def _need_ref():
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")


def _inputs(rs, M, N, K):
    G = -(-K // 128)
    a = rs.randint(-127, 128, size=(M, K)).astype(np.int8)
    b = rs.randint(-127, 128, size=(N, K)).astype(np.int8)
    sa = (np.abs(rs.normal(size=(M, G))) * 0.01 + 1e-4).astype(np.float32)
    sb = (np.abs(rs.normal(size=(N, G))) * 0.002 + 1e-5).astype(np.float32)
    return a, b, sa, sb


def _dev(cuda, *xs):
    return [torch.from_numpy(np.ascontiguousarray(x)).to(cuda) for x in xs]


def _padded_i8(cuda, x):
    """x int8 [R, K] in a buffer whose row pitch is K rounded up to 16 (the kernel's operand rule)."""
    R, K = x.shape
    ld = -(-K // 16) * 16
    buf = torch.zeros((R, ld), dtype=torch.int8, device=cuda)
    buf[:, :K] = torch.from_numpy(x).to(cuda)
    return buf[:, :K]


PLAIN = [(3, 12, 256), (130, 260, 208), (1, 4, 128), (257, 516, 384), (64, 1024, 1024)]


@pytest.mark.parametrize("case", PLAIN, ids=[f"{m}x{n}x{k}" for m, n, k in PLAIN])
@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
def test_gemm_i8g_matches_reference_twin(cuda, case, bf16):
    _need_ref()
    M, N, K = case
    G = -(-K // 128)
    rs = np.random.RandomState(M + 7 * N + K)
    a, b, sa, sb = _inputs(rs, M, N, K)
    ops_ = [Operand("a", "i8", (M, K)), Operand("a_scale", "f32", (M, G)), Operand("b", "i8", (N, K)),
            Operand("b_scale", "f32", (N, G)), Operand("y", "f32", (M, N), written=True)]
    want = ref_twin("gemm_nt_q", {"M": M, "K": K, "N": N, "group": 128, "dtype": "i8a8h"}, ops_,
                    {"a": a.astype(np.float64), "a_scale": sa.astype(np.float64), "b": b.astype(np.float64),
                     "b_scale": sb.astype(np.float64)})["y"]
    ad, bd = _padded_i8(cuda, a), _padded_i8(cuda, b)
    sad, sbd = _dev(cuda, sa, sb)
    y = ops.gemm_i8g(ad, sad, bd, sbd, out_dtype=torch.bfloat16 if bf16 else torch.float32)
    got = y.float().cpu().numpy().astype(np.float64)
    if bf16:
        # one bf16 step of the twin's value: the f32 result and the f64 twin may round to neighbours
        ref = torch.from_numpy(want.astype(np.float32)).to(torch.bfloat16).float().numpy()
        assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-30)
    else:
        err = np.abs(got - want).max() / np.abs(want).max()
        assert err <= 2e-6, err


def _fwht(v):
    v = v.copy()
    g = v.reshape(-1, 128)
    h = 1
    while h < 128:
        blk = g.reshape(g.shape[0], 128 // (2 * h), 2, h)
        x0, x1 = blk[:, :, 0, :].copy(), blk[:, :, 1, :].copy()
        blk[:, :, 0, :] = x0 + x1
        blk[:, :, 1, :] = x0 - x1
        h *= 2
    return g.reshape(v.shape)


GATED = [(3, 256, 256, "silu"), (130, 512, 208, "silu"), (64, 256, 384, "sigmoid"), (200, 1024, 512, "silu")]


@pytest.mark.parametrize("case", GATED, ids=[f"{m}x{n}x{k}{act[:3]}" for m, n, k, act in GATED])
def test_gemm_i8g_gated_matches_reference_twin(cuda, case):
    _need_ref()
    M, N, K, act = case
    n, G = N // 2, -(-K // 128)
    rs = np.random.RandomState(3 * M + N + K)
    a, b, sa, sb = _inputs(rs, M, N, K)
    ops_ = [Operand("a", "i8", (M, K)), Operand("a_scale", "f32", (M, G)), Operand("b", "i8", (N, K)),
            Operand("b_scale", "f32", (N, G)), Operand("q", "i8", (M, n), written=True),
            Operand("scale", "f32", (M, n // 128), written=True),
            Operand("out_bf16", "bf16", (M, n), written=True)]
    want = ref_twin("gemm_nt_q_gated", {"M": M, "K": K, "N": N, "group": 128, "act": act, "dtype": "i8a8h"}, ops_,
                    {"a": a.astype(np.float64), "a_scale": sa.astype(np.float64), "b": b.astype(np.float64),
                     "b_scale": sb.astype(np.float64)})
    ad, bd = _padded_i8(cuda, a), _padded_i8(cuda, b)
    sad, sbd = _dev(cuda, sa, sb)
    q, qs, ob = ops.gemm_i8g_gated(ad, sad, bd, sbd, act=act, want_bf16=True)
    q2, qs2, none = ops.gemm_i8g_gated(ad, sad, bd, sbd, act=act, want_bf16=False)
    torch.cuda.synchronize()
    assert none is None
    assert torch.equal(q, q2) and torch.equal(qs, qs2)  # out_bf16 changes nothing else
    got_s = qs.cpu().numpy().astype(np.float64)
    assert np.max(np.abs(got_s / want["scale"] - 1)) < 1e-5
    p = want["out_bf16"]
    ref_b = torch.from_numpy(p.astype(np.float32)).to(torch.bfloat16).float().numpy()
    got_b = ob.float().cpu().numpy()
    # one bf16 step, or the f32 product's own rounding where the groups' sum cancels to near zero
    tol = np.abs(ref_b) * 2.0 ** -7 + 1e-6 * np.abs(p).max(axis=1, keepdims=True)
    assert np.all(np.abs(got_b - ref_b) <= tol)
    wc, gc = want["q"].astype(np.int64), q.cpu().numpy().astype(np.int64)
    bad = gc != wc
    if bad.any():
        u = _fwht(p) / np.repeat(want["scale"], 128, axis=1)
        frac = np.abs(np.abs(u[bad]) - np.floor(np.abs(u[bad])) - 0.5)
        assert np.all(np.abs(gc[bad] - wc[bad]) == 1) and np.all(frac < 2e-3), \
            f"{bad.sum()} codes differ away from a rounding tie"
    assert bad.sum() <= max(2, bad.size // 1000)


def _grouped_torch(a, b, sa, sb):
    """sum_g sa sb (a_g b_g^T) in f64, each group's integer product exact in f32."""
    M, K = a.shape
    y = torch.zeros((M, b.shape[0]), dtype=torch.float64, device=a.device)
    for g in range(-(-K // 128)):
        k0, k1 = 128 * g, min(K, 128 * g + 128)
        s = a[:, k0:k1].float() @ b[:, k0:k1].float().T
        y += s.double() * sa[:, g:g + 1].double() * sb[:, g].double()[None, :]
    return y


def test_gemm_i8g_trunk_size(cuda):
    """A trunk projection's shape (8192 tokens x 4096 -> 4096): against the exact grouped formula."""
    g = torch.Generator(device=cuda).manual_seed(11)
    M, N, K = 8192, 4096, 4096
    a = torch.randint(-127, 128, (M, K), generator=g, device=cuda, dtype=torch.int8)
    b = torch.randint(-127, 128, (N, K), generator=g, device=cuda, dtype=torch.int8)
    sa = torch.rand((M, K // 128), generator=g, device=cuda) * 0.01 + 1e-4
    sb = torch.rand((N, K // 128), generator=g, device=cuda) * 0.002 + 1e-5
    y = ops.gemm_i8g(a, sa, b, sb)
    rows = torch.arange(0, M, 61, device=cuda)
    want = _grouped_torch(a[rows], b, sa[rows], sb)
    err = ((y[rows].double() - want).abs().max() / want.abs().max()).item()
    assert err <= 2e-6, err


def test_gemm_i8g_gated_zero_group_and_clamp(cuda):
    """A row whose product is zero has scale 1 and zero codes; every other group reaches the grid's top."""
    rs = np.random.RandomState(5)
    M, N, K = 4, 256, 128
    a, b, sa, sb = _inputs(rs, M, N, K)
    a[1] = 0
    ad, bd = _padded_i8(cuda, a), _padded_i8(cuda, b)
    sad, sbd = _dev(cuda, sa, sb)
    q, qs, _ = ops.gemm_i8g_gated(ad, sad, bd, sbd)
    assert qs[1, 0].item() == 1.0 and not q[1].any()
    for r in (0, 2, 3):
        assert int(q[r].abs().max().item()) == 127


def test_gemm_i8g_rejects_bad_operands(cuda):
    a = torch.zeros((4, 200), dtype=torch.int8, device=cuda)  # K = 200: not a multiple of 16
    b = torch.zeros((8, 200), dtype=torch.int8, device=cuda)
    s = torch.ones((8, 2), dtype=torch.float32, device=cuda)
    with pytest.raises(R97bError):
        ops.gemm_i8g(a, s[:4], b, s)
    a = torch.zeros((4, 256), dtype=torch.int8, device=cuda)
    b = torch.zeros((192, 256), dtype=torch.int8, device=cuda)  # n = 96: not a multiple of 128
    s = torch.ones((192, 2), dtype=torch.float32, device=cuda)
    with pytest.raises(R97bError):
        ops.gemm_i8g_gated(a, s[:4], b, s)
