"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Integer/byte work (the IQR decode) must match bit for bit; floating-point kernels are held to the
north star's bf16 bar (per-tensor relative L2 <= 1e-2, cosine >= 0.999) or tighter where stated."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import rows as R
from r97training_b200 import iqr as IQ
from r97training_b200 import ops
from r97training_b200._lib import lib
from tests.gpu_util import assert_close_bf16, device_form_desc, rel_l2, to_np
from tests.iqr_forms import FORMS, make_form

pytestmark = pytest.mark.gpu


# ----------------------------------------------------------------------------- IQR decode

@pytest.mark.parametrize("kw", FORMS, ids=[str(i) for i in range(len(FORMS))])
def test_iqr_decode_bit_exact(cuda, kw):
    form = make_form(**kw)
    want_c, want_s = R.iqr_decode(form)
    d, oc, os_, keep = device_form_desc(form, cuda)
    s = torch.cuda.current_stream().cuda_stream
    assert lib().r97_iqr_decode(ctypes.byref(d), ctypes.c_void_p(s)) == 0
    torch.cuda.synchronize()
    assert np.array_equal(oc.cpu().numpy(), want_c)
    assert np.array_equal(os_.cpu().numpy().view(np.uint16), want_s)


def test_iqr_decode_chunk_and_reject(cuda):
    form = make_form(rows=768)
    want_c, want_s = R.iqr_decode(form, row0=256, rows=512)
    d, oc, os_, keep = device_form_desc(form, cuda, row0=256, rows=512)
    assert lib().r97_iqr_decode(ctypes.byref(d), None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(oc.cpu().numpy(), want_c)
    assert np.array_equal(os_.cpu().numpy().view(np.uint16), want_s)
    d2, _, _, keep2 = device_form_desc(form, cuda, row0=100, rows=100)
    assert lib().r97_iqr_decode(ctypes.byref(d2), None) == 1


def test_trunk_decode_and_dequant_large(cuda):
    w = IQ.synth_weight(1024 + 128, 2048, seed=11)   # a short last run of 128 rows
    form = R.trunk_form(w.codes.numpy(), w.scale.numpy(), w.mad_a, w.mad_b, w.cols)
    want_c, want_s = R.iqr_decode(form)
    wd = w.to(cuda)
    c, s = IQ.decode(wd)
    torch.cuda.synchronize()
    assert np.array_equal(c.cpu().numpy(), want_c)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), want_s)
    Wb = IQ.dequant_bf16(wd)
    torch.cuda.synchronize()
    want_w = R.f64_to_bf16(R.dequant_value(want_c, want_s))
    assert np.array_equal(to_np(Wb), want_w)


# ----------------------------------------------------------------------------- GEMM

def _bf(rs, shape, std=1.0):
    return torch.from_numpy((rs.normal(size=shape) * std).astype(np.float32)).to(torch.bfloat16)


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("bn", [64, 128, 256, 512])
def test_gemm_layouts(cuda, a_mn, b_mn, bn):
    """bn 512 is the CTA-pair kernel (256 x 256 tiles over two SMs); the shapes are ragged in M, N and K
    against every tile."""
    rs = np.random.RandomState(100 + 4 * a_mn + 2 * b_mn + bn)
    M, N, K = 384, 320, 448
    A = _bf(rs, (M, K))
    B = _bf(rs, (N, K))
    a_dev = (A.t().contiguous() if a_mn else A).to(cuda)
    b_dev = (B.t().contiguous() if b_mn else B).to(cuda)
    out = torch.zeros((M, N), dtype=torch.float32, device=cuda)
    ops.gemm(a_dev, b_dev, out, a_mn=a_mn, b_mn=b_mn, mode=ops.EPI_STORE_F32, bn=bn)
    torch.cuda.synchronize()
    want = A.double().numpy() @ B.double().numpy().T
    assert rel_l2(to_np(out), want) < 1e-5


@pytest.mark.parametrize("splits", [1, 3])
def test_gemm_pair_kernel_many_tiles(cuda, splits):
    """The CTA-pair kernel over more 256 x 256 tiles than pairs of SMs (every pair runs several tiles, so
    both accumulators and the stage ring wrap), with split-K atomics."""
    rs = np.random.RandomState(7 + splits)
    M, N, K = 2304, 4352, 640
    A, B = _bf(rs, (M, K)), _bf(rs, (N, K))
    out = torch.zeros((M, N), dtype=torch.float32, device=cuda)
    mode = ops.EPI_ATOMIC_F32 if splits > 1 else ops.EPI_STORE_F32
    ops.gemm(A.to(cuda), B.to(cuda), out, mode=mode, splits=splits, bn=512)
    torch.cuda.synchronize()
    want = A.double().numpy() @ B.double().numpy().T
    assert rel_l2(to_np(out), want) < 1e-5


def test_gemm_lora_tail_bf16_epilogue(cuda):
    rs = np.random.RandomState(5)
    M, N, K, r = 256, 512, 1024, 64
    X, W, T, Bl = _bf(rs, (M, K)), _bf(rs, (N, K), 0.02), _bf(rs, (M, r)), _bf(rs, (N, r), 0.1)
    C = _bf(rs, (M, N))
    out = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    ops.gemm(X.to(cuda), W.to(cuda), out, a2=T.to(cuda), b2=Bl.to(cuda), alpha=0.5, addend=C.to(cuda), beta=1.0)
    torch.cuda.synchronize()
    want = 0.5 * (X.double().numpy() @ W.double().numpy().T + T.double().numpy() @ Bl.double().numpy().T) + \
        C.double().numpy()
    assert_close_bf16(to_np(out), want, rel=4e-3, what="lora tail")


def test_gemm_dx_form_mn_major_weight(cuda):
    # dX = [dY | dt] [W ; A]: A-operands K-major, B-operands (W [N,K], A_lora [r,K]) MN-major
    rs = np.random.RandomState(6)
    M, N, K, r = 256, 384, 512, 64
    dY, W, dt, Al = _bf(rs, (M, N)), _bf(rs, (N, K), 0.02), _bf(rs, (M, r)), _bf(rs, (r, K), 0.25)
    out = torch.empty((M, K), dtype=torch.bfloat16, device=cuda)
    ops.gemm(dY.to(cuda), W.to(cuda), out, b_mn=True, a2=dt.to(cuda), b2=Al.to(cuda), M=M, N=K)
    torch.cuda.synchronize()
    want = dY.double().numpy() @ W.double().numpy() + dt.double().numpy() @ Al.double().numpy()
    assert_close_bf16(to_np(out), want, rel=4e-3, what="dx")


@pytest.mark.parametrize("transposed,T,splits,r", [(False, 2048, 4, 64), (True, 2048, 4, 64), (False, 8192, 3, 64),
                                                    (True, 8192, 3, 64), (False, 8192, 8, 64), (True, 8192, 5, 192),
                                                    (False, 1000, 3, 64)])
def test_gemm_split_k_atomic(cuda, transposed, T, splits, r):
    # the adapter-gradient form: reduce over tokens (both operands MN-major), split-K into f32 -- splits that
    # do not divide the token blocks evenly, the vector-atomic row-major epilogue and a ragged token count
    rs = np.random.RandomState(7 + T + splits)
    K = 256
    X, dt = _bf(rs, (T, K)), _bf(rs, (T, r))
    if transposed:   # dA [r, K] += (X^T dt)^T
        out = torch.zeros((r, K), dtype=torch.float32, device=cuda)
        ops.gemm(X.to(cuda), dt.to(cuda), out, a_mn=True, b_mn=True, mode=ops.EPI_ATOMIC_F32T, splits=splits)
        want = dt.double().numpy().T @ X.double().numpy()
    else:            # [K, r]
        out = torch.zeros((K, r), dtype=torch.float32, device=cuda)
        ops.gemm(X.to(cuda), dt.to(cuda), out, a_mn=True, b_mn=True, mode=ops.EPI_ATOMIC_F32, splits=splits)
        want = X.double().numpy().T @ dt.double().numpy()
    torch.cuda.synchronize()
    assert rel_l2(to_np(out), want) < 1e-5


@pytest.mark.parametrize("b_mn,bn,splits", [(False, 64, 2), (True, 64, 3), (False, 128, 2), (True, 256, 4),
                                            (False, 64, 1)])
def test_gemm_split_bf16_deterministic(cuda, b_mn, bn, splits):
    """EPI_SPLIT_BF16: the reduction split across CTAs, partials summed in split order by the tile's last
    split -- the adapter's narrow products (t = s x A^T, dt = s dY B). Ragged M and K, the same bits on a
    repeat, the workspace's counters back at zero afterwards, and a missing workspace rejected."""
    rs = np.random.RandomState(30 + bn + splits)
    M, N, K = 1000, 136 if bn > 64 else 64, 1600
    A, B, C = _bf(rs, (M, K)), _bf(rs, (N, K), 0.05), _bf(rs, (M, N))
    b_dev = (B.t().contiguous() if b_mn else B).to(cuda)
    ws = ops.SplitWorkspace(cuda, 8 << 20)
    outs = []
    for _ in range(2):
        out = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
        ops.gemm(A.to(cuda), b_dev, out, b_mn=b_mn, N=N, mode=ops.EPI_SPLIT_BF16, splits=splits, bn=bn,
                 alpha=2.0, addend=C.to(cuda), beta=1.0, ws=ws.buf)
        outs.append(out)
    torch.cuda.synchronize()
    want = 2.0 * (A.double().numpy() @ B.double().numpy().T) + C.double().numpy()
    assert_close_bf16(to_np(outs[0]), want, rel=4e-3, what="split bf16")
    assert torch.equal(outs[0], outs[1])
    cnt = ws.buf[:(-(-M // 128)) * (-(-N // bn))]
    assert int(cnt.abs().sum()) == 0
    if splits > 1:
        with pytest.raises(Exception):
            ops.gemm(A.to(cuda), b_dev, outs[0], b_mn=b_mn, N=N, mode=ops.EPI_SPLIT_BF16, splits=splits, bn=bn)


def test_gemm_ragged_edges(cuda):
    rs = np.random.RandomState(8)
    M, N, K = 200, 136, 200   # none a multiple of the tile
    A, B = _bf(rs, (M, K)), _bf(rs, (N, K))
    out = torch.full((M, N), 7.0, dtype=torch.float32, device=cuda)
    ops.gemm(A.to(cuda), B.to(cuda), out, mode=ops.EPI_STORE_F32)
    torch.cuda.synchronize()
    assert rel_l2(to_np(out), A.double().numpy() @ B.double().numpy().T) < 1e-5


# ----------------------------------------------------------------------------- norms

@pytest.mark.parametrize("n", [128, 1024, 2048, 4096, 8192, 1280])
def test_rmsnorm(cuda, n):
    rs = np.random.RandomState(n)
    rows = 301
    x, dy, add = _bf(rs, (rows, n)), _bf(rs, (rows, n)), _bf(rs, (rows, n))
    w = torch.from_numpy(rs.normal(size=n).astype(np.float32))
    y = ops.rmsnorm_fwd(x.to(cuda), w.to(cuda), eps=1e-6)
    dx = ops.rmsnorm_bwd(x.to(cuda), w.to(cuda), dy.to(cuda), addend=add.to(cuda), eps=1e-6)
    torch.cuda.synchronize()
    xn, wn, dyn = x.double().numpy(), w.double().numpy(), dy.double().numpy()
    assert_close_bf16(to_np(y), R.rmsnorm_fwd(xn, wn), rel=5e-3, what="rmsnorm fwd")
    assert_close_bf16(to_np(dx), R.rmsnorm_bwd(xn, wn, dyn) + add.double().numpy(), rel=5e-3, what="rmsnorm bwd")


@pytest.mark.parametrize("sig", [False, True])
def test_gated_rmsnorm(cuda, sig):
    rs = np.random.RandomState(9)
    rows, n = 4097, 128
    x, z, do = _bf(rs, (rows, n)), _bf(rs, (rows, n)), _bf(rs, (rows, n), 1e-2)
    w = torch.from_numpy(rs.normal(size=n).astype(np.float32))
    o = ops.gated_rmsnorm_fwd(x.to(cuda), z.to(cuda), w.to(cuda), sigmoid=sig)
    dx, dz = ops.gated_rmsnorm_bwd(x.to(cuda), z.to(cuda), w.to(cuda), do.to(cuda), sigmoid=sig)
    torch.cuda.synchronize()
    xn, zn, wn, don = (t.double().numpy() for t in (x, z, w, do))
    assert_close_bf16(to_np(o), R.gated_rmsnorm_fwd(xn, zn, wn, sigmoid=sig), rel=5e-3, what="grms fwd")
    rdx, rdz = R.gated_rmsnorm_bwd(xn, zn, wn, don, sigmoid=sig)
    assert_close_bf16(to_np(dx), rdx, rel=5e-3, what="grms dx")
    assert_close_bf16(to_np(dz), rdz, rel=5e-3, what="grms dz")


# ----------------------------------------------------------------------------- CE / KLD

@pytest.mark.parametrize("vocab,rows", [(1000, 17), (151936, 17), (1003, 700)])
def test_ce_kld(cuda, vocab, rows):
    # 700 rows with a ragged vocabulary (no 16-byte rows: one value a load)
    rs = np.random.RandomState(vocab % 1000 + rows)
    s = _bf(rs, (rows, vocab), 2.0)
    t = _bf(rs, (rows, vocab), 2.0)
    tg = rs.randint(0, vocab, size=rows).astype(np.int32)
    tg[3] = -1
    tg[rows - 2] = -1
    # a row with a large maximum: bf16 keeps ~3 digits there, so the row is offset by a constant the loss
    # must not absorb (log(s) - (x_t - m), the reference's order)
    s[5] = (s[5].float() + 2.0 ** 14).bfloat16()
    sd = s.to(cuda)
    grad = torch.empty_like(sd)
    lce, lkl = ops.ce_kld(sd, torch.from_numpy(tg).to(cuda), t.to(cuda), grad=grad, grad_scale=0.5, w_ce=1.0,
                          w_kl=0.3)
    torch.cuda.synchronize()
    sn, tn = s.double().numpy(), t.double().numpy()
    l1, g1 = R.ce_rows(sn, tg, 0.5)
    l2, g2 = R.kld_rows(sn, tn, 0.5, targets=tg)
    np.testing.assert_allclose(lce.cpu().numpy(), l1, rtol=1e-4, atol=1e-4)
    # the KL sum carries t - s, which row 5's offset makes ~1.6e4: f32 keeps ~2e-3 of it absolute there
    kl = lkl.cpu().numpy()
    keep = np.arange(rows) != 5
    np.testing.assert_allclose(kl[keep], l2[keep], rtol=1e-3, atol=1e-4)
    assert abs(kl[5] - l2[5]) <= 4e-3, (kl[5], l2[5])
    assert_close_bf16(to_np(grad), g1 + 0.3 * g2, rel=5e-3, what="ce+kl grad")
    # in place
    lce2, _ = ops.ce_kld(sd, torch.from_numpy(tg).to(cuda), grad=sd, grad_scale=0.5)
    torch.cuda.synchronize()
    assert_close_bf16(to_np(sd), g1, rel=5e-3, what="ce in place")


# ----------------------------------------------------------------------------- AdamW

def _powf(x, y):
    libm = ctypes.CDLL("libm.so.6")
    libm.powf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    return libm.powf(x, y)


def test_adamw_bit_exact(cuda):
    rs = np.random.RandomState(12)
    n, steps = 100003, 3
    w0 = rs.normal(size=n).astype(np.float32)
    gs = (rs.normal(size=(steps, n)) * 1e-2).astype(np.float32)
    w, m, v = w0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    wd_, md, vd = (torch.from_numpy(a.copy()).to(cuda) for a in (w0, m, v))
    b1, b2, eps, wdec = 0.9, 0.999, 1e-8, 0.01
    for t in range(1, steps + 1):
        lr = R.scheduled_lr(1e-4, 0, 0, 0.1, t)
        R.adamw_update(w, m, v, gs[t - 1], lr, b1, b2, eps, wdec, t)
        bc1 = np.float32(1.0) - np.float32(_powf(b1, float(t)))
        bc2 = np.float32(1.0) - np.float32(_powf(b2, float(t)))
        g = torch.from_numpy(gs[t - 1].copy()).to(cuda)
        ops.adamw_step(wd_, md, vd, g, lr=float(lr), beta1=b1, beta2=b2, eps=eps, weight_decay=wdec, bc1=float(bc1),
                       bc2=float(bc2))
    torch.cuda.synchronize()
    assert np.array_equal(wd_.cpu().numpy().view(np.uint32), w.view(np.uint32))


def test_global_norm_and_clip(cuda):
    rs = np.random.RandomState(13)
    n = 300001
    g = (rs.normal(size=n) * 1e-2).astype(np.float32)
    gd = torch.from_numpy(g).to(cuda)
    norm, scale = ops.global_norm(gd, max_norm=0.5)
    torch.cuda.synchronize()
    parts = [np.sum(g[i:i + 4096].astype(np.float64) ** 2) for i in range(0, n, 4096)]
    want = np.float32(np.sqrt(np.sum(parts)))
    assert abs(float(norm) - float(want)) <= 1e-6 * float(want)
    assert abs(float(scale) - min(1.0, 0.5 / float(want))) < 1e-6


def test_gated_rmsnorm_strided_z(cuda):
    """z read from (and dz written into) the z columns of a wider fused projection row."""
    rs = np.random.RandomState(10)
    T, H, n, pad = 257, 4, 128, 96
    x, do = _bf(rs, (T * H, n)), _bf(rs, (T * H, n), 1e-2)
    wide = _bf(rs, (T, pad + H * n + 64))
    w = torch.from_numpy(rs.normal(size=n).astype(np.float32))
    wd = wide.to(cuda)
    zs = wd[:, pad:pad + H * n]
    o = ops.gated_rmsnorm_fwd(x.to(cuda), zs, w.to(cuda))
    dwide = torch.zeros_like(wd)
    dx, _ = ops.gated_rmsnorm_bwd(x.to(cuda), zs, w.to(cuda), do.to(cuda), dz=dwide[:, pad:pad + H * n])
    torch.cuda.synchronize()
    zn = wide.double().numpy()[:, pad:pad + H * n].reshape(T * H, n)
    xn, wn, don = x.double().numpy(), w.double().numpy(), do.double().numpy()
    assert_close_bf16(to_np(o), R.gated_rmsnorm_fwd(xn, zn, wn), rel=5e-3, what="o")
    rdx, rdz = R.gated_rmsnorm_bwd(xn, zn, wn, don)
    assert_close_bf16(to_np(dx), rdx, rel=5e-3, what="dx")
    got = to_np(dwide)
    assert_close_bf16(got[:, pad:pad + H * n].reshape(T * H, n), rdz, rel=5e-3, what="dz")
    assert not got[:, :pad].any() and not got[:, pad + H * n:].any()


def test_cast_segments_table(cuda):
    """r97b_cast_segments: many f32 -> bf16 casts of 2-D views (strided rows, column blocks of a wider
    destination) in one launch, equal to torch's round-to-nearest-even cast."""
    rs = np.random.RandomState(3)
    flat = torch.from_numpy(rs.normal(size=100000).astype(np.float32)).to(cuda)
    wide = torch.zeros((96, 64), dtype=torch.bfloat16, device=cuda)
    a_dst = torch.empty((16, 256), dtype=torch.bfloat16, device=cuda)
    pairs = [(flat[:4096].view(16, 256), a_dst),
             (flat[4096:4096 + 48 * 32].view(48, 32), wide[:48, :32]),
             (flat[8192:8192 + 48 * 32].view(48, 32), wide[48:, 32:])]
    table = ops.CastTable(pairs, cuda)
    table.run()
    torch.cuda.synchronize()
    for src, dst in pairs:
        assert torch.equal(dst, src.to(torch.bfloat16))
    assert int(wide[:48, 32:].float().abs().sum()) == 0 and int(wide[48:, :32].float().abs().sum()) == 0


@pytest.mark.parametrize("M,F,K", [(384, 256, 320), (1000, 512, 448)])
def test_gemm_swiglu_epilogues_match_unfused(cuda, M, F, K):
    """EPI_SWIGLU (the gate/up GEMM writing [g | u] and silu(g) u) and EPI_SWIGLU_BWD (the down GEMM's input
    adjoint writing [dg | du]) give the same bits as the plain GEMM followed by the standalone SwiGLU
    kernels, with the LoRA tail in the forward."""
    rs = np.random.RandomState(M + F)
    r = 64
    X, W, T, Bl = _bf(rs, (M, K)), _bf(rs, (2 * F, K), 0.05), _bf(rs, (M, 2 * r)), _bf(rs, (2 * F, 2 * r), 0.1)
    X, W, T, Bl = X.to(cuda), W.to(cuda), T.to(cuda), Bl.to(cuda)
    gu_ref = torch.empty((M, 2 * F), dtype=torch.bfloat16, device=cuda)
    ops.gemm(X, W, gu_ref, a2=T, b2=Bl, bn=512)
    a_ref = torch.empty((M, F), dtype=torch.bfloat16, device=cuda)
    ops.swiglu_fwd(gu_ref, a_ref)
    gu = torch.empty_like(gu_ref)
    a = torch.empty_like(a_ref)
    ops.gemm(X, W, gu, a2=T, b2=Bl, mode=ops.EPI_SWIGLU, out2=a)
    # the backward: da = dY Wd (Wd [Kd, F] read MN-major), then SwiGLU's adjoint
    Kd = 256
    dY, Wd = _bf(rs, (M, Kd)).to(cuda), _bf(rs, (Kd, F), 0.05).to(cuda)
    da = torch.empty((M, F), dtype=torch.bfloat16, device=cuda)
    ops.gemm(dY, Wd, da, b_mn=True, N=F)
    dgu_ref = torch.empty_like(gu_ref)
    ops.swiglu_bwd(gu_ref, da, dgu_ref)
    dgu = torch.empty_like(gu_ref)
    ops.gemm(dY, Wd, dgu, b_mn=True, N=F, mode=ops.EPI_SWIGLU_BWD, addend=gu_ref)
    torch.cuda.synchronize()
    assert torch.equal(gu, gu_ref)
    assert torch.equal(a, a_ref)
    assert torch.equal(dgu, dgu_ref)
