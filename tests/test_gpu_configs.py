"""The BASELINE configurations 1-3 at their full sizes, through the product's calls, against the f64 oracle
(oracle/rows.py, oracle/gdn.py -- restatements of the reference's host rows, pinned to them in
tests/test_oracle_pin*.py) on the same bf16-rounded inputs, with the inputs' stated distributions.
Where the f64 oracle cannot run the whole case in seconds (the vocab head), it runs on sampled rows and
size-independent properties cover the rest. Tolerance: the north star's bf16 bar (per-tensor relative
L2 <= 1e-2, cosine >= 0.999)."""
import math

import numpy as np
import pytest
import torch

from oracle import gdn as G
from oracle import rows as R
from r97training_b200 import iqr as IQ
from r97training_b200 import ops
from r97training_b200.gdn import GdnPlan
from tests.gpu_util import assert_close_bf16, to_np

pytestmark = pytest.mark.gpu


def _bf(x):
    return torch.from_numpy(np.asarray(x, np.float32)).bfloat16()


def test_config1_lora_linear_full_size(cuda):
    """Config 1: X [256 x 2048] ~ N(0,1); W [2048 x 2048] IQR (uniform codes, scales |N(0, 0.02)|); LoRA r 16,
    alpha 32 (s = 2), A ~ N(0, 1/16), B ~ N(0, 0.01); dY ~ N(0, 1e-2). Y, dX, dA, dB through the model's
    GEMM calls (the narrow shrink / expand products on their split tilings, the fused tail, the split-K
    adapter gradients)."""
    rs = np.random.RandomState(1)
    M, K, N, r, s = 256, 2048, 2048, 16, 2.0
    X = _bf(rs.normal(size=(M, K)))
    A = _bf(rs.normal(size=(r, K)) / 4.0)
    B = _bf(rs.normal(size=(N, r)) * 0.01)
    dY = _bf(rs.normal(size=(M, N)) * 1e-2)
    w = IQ.synth_weight(N, K, seed=5, device=cuda, scale_std=0.02)
    Wd = IQ.dequant_bf16(w)
    x, a, b, dy = (t.to(cuda) for t in (X, A, B, dY))
    ws = ops.SplitWorkspace(cuda, 8 << 20)
    t = torch.empty((M, r), dtype=torch.bfloat16, device=cuda)
    bn, sp = ops.skinny_tiling(M, r, K)
    ops.gemm(x, a, t, alpha=s, bn=bn, splits=sp, mode=ops.EPI_SPLIT_BF16 if sp > 1 else ops.EPI_STORE_BF16,
             ws=ws.buf)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    ops.gemm(x, Wd, y, a2=t, b2=b)
    dt = torch.empty((M, r), dtype=torch.bfloat16, device=cuda)
    bn, sp = ops.skinny_tiling(M, r, N)
    ops.gemm(dy, b, dt, b_mn=True, alpha=s, N=r, bn=bn, splits=sp,
             mode=ops.EPI_SPLIT_BF16 if sp > 1 else ops.EPI_STORE_BF16, ws=ws.buf)
    dx = torch.empty((M, K), dtype=torch.bfloat16, device=cuda)
    ops.gemm(dy, Wd, dx, b_mn=True, a2=dt, b2=a, N=K)
    dA = torch.zeros((r, K), dtype=torch.float32, device=cuda)
    bn, sp = ops.grad_tiling(K, r, M)
    ops.gemm(x, dt, dA, a_mn=True, b_mn=True, mode=ops.EPI_ATOMIC_F32T, splits=sp, bn=bn, M=K, N=r)
    dB = torch.zeros((N, r), dtype=torch.float32, device=cuda)
    bn, sp = ops.grad_tiling(N, r, M)
    ops.gemm(dy, t, dB, a_mn=True, b_mn=True, mode=ops.EPI_ATOMIC_F32, splits=sp, bn=bn, M=N, N=r)
    torch.cuda.synchronize()
    Wn = to_np(Wd)
    xn, an, bnp, dyn = (u.double().numpy() for u in (X, A, B, dY))
    y_ref, t_ref = R.lora_fwd(xn, Wn, an, bnp, s)
    dx_ref, dA_ref, dB_ref, _ = R.lora_bwd(xn, Wn, an, bnp, s, t_ref, dyn)
    assert_close_bf16(to_np(y), y_ref, what="Y")
    assert_close_bf16(to_np(dx), dx_ref, what="dX")
    assert_close_bf16(to_np(dA), dA_ref, what="dA")
    assert_close_bf16(to_np(dB), dB_ref, what="dB")


def test_config2_gdn_layer_with_gated_norm_full_size(cuda):
    """Config 2: one GatedDeltaNet layer and its gated RMSNorm, T 4096, batch 1, 16 value heads and 16 QK
    heads of 128, chunk 64; q, k L2-normalised N(0,1), v ~ N(0,1), beta = sigmoid(N(0,1)), the log decay
    -softplus(N(0,1)) accumulated within chunks, z ~ N(0,1), the norm's gain ~ N(0,1), upstream ~ N(0,1e-2).
    The chain o = gdn(q,k,v), y = gated_rmsnorm(o, z) and its adjoint against the f64 oracle's chain."""
    H = Hg = 16
    d = G.synth_inputs([4096], H, Hg, seed=42)
    rs = np.random.RandomState(43)
    T = 4096
    q, k, v = (_bf(d[n]) for n in ("q", "k", "v"))
    z = _bf(rs.normal(size=(T * H, 128)))
    wn = rs.normal(size=128).astype(np.float32)
    dy = _bf(rs.normal(size=(T * H, 128)) * 1e-2)
    g, beta = d["g"].astype(np.float32), d["beta"].astype(np.float32)
    plan = GdnPlan(d["cu"], H, Hg, cuda)
    o, _, sv = plan.forward(q.to(cuda), k.to(cuda), v.to(cuda), torch.from_numpy(g).to(cuda),
                            torch.from_numpy(beta).to(cuda))
    zd, wd, dyd = z.to(cuda), torch.from_numpy(wn).to(cuda), dy.to(cuda)
    y = ops.gated_rmsnorm_fwd(o.view(T * H, 128), zd, wd)
    do, dz = ops.gated_rmsnorm_bwd(o.view(T * H, 128), zd, wd, dyd)
    grads = plan.backward(sv, do.view(T, H, 128))
    torch.cuda.synchronize()
    qn, kn, vn = (t.double().numpy() for t in (q, k, v))
    A = G.kkt_fwd(kn, beta.astype(np.float64), g.astype(np.float64), d["cu"])
    o_ref, _ = G.scan_fwd(qn, kn, vn, A, g.astype(np.float64), beta.astype(np.float64), d["cu"])
    zn, dyn = z.double().numpy(), dy.double().numpy()
    y_ref = R.gated_rmsnorm_fwd(o_ref.reshape(T * H, 128), zn, wn.astype(np.float64))
    do_ref, dz_ref = R.gated_rmsnorm_bwd(o_ref.reshape(T * H, 128), zn, wn.astype(np.float64), dyn)
    ref = G.layer_fwd_bwd(qn, kn, vn, g.astype(np.float64), beta.astype(np.float64), d["cu"],
                          do_ref.reshape(T, H, 128))
    assert_close_bf16(to_np(o), o_ref, what="o")
    assert_close_bf16(to_np(y), y_ref, what="y")
    assert_close_bf16(to_np(dz), dz_ref, what="dz")
    for name in ("dq", "dk", "dv", "dbeta", "dg"):
        assert_close_bf16(to_np(grads[name]), ref[name], what=name)


def test_config3_vocab_head_ce_kld_full_size(cuda):
    """Config 3: hidden [8192 x 2048] ~ N(0,1); the tied head [151936 x 2048] in IQR form; targets uniform
    over the vocabulary; teacher logits ~ N(0,2). Logits in chunks of 2048 rows (never the whole matrix),
    the CE + KL gradient in place, d(hidden) = grad W. Every row: finite losses, KL >= 0, and gradient rows
    that sum to zero (softmax - onehot, softmax - softmax); 48 sampled rows against the f64 oracle."""
    rs = np.random.RandomState(3)
    T, Dm, V, chunk = 8192, 2048, 151936, 2048
    h = torch.randn(T, Dm, generator=torch.Generator().manual_seed(3)).bfloat16().to(cuda)
    w = IQ.synth_weight(V, Dm, seed=9, device=cuda, scale_std=0.02 / 37.0)
    Wd = IQ.dequant_bf16(w)
    tg = torch.from_numpy(rs.randint(0, V, size=T).astype(np.int32)).to(cuda)
    gen = torch.Generator(device=cuda).manual_seed(4)
    teacher = (torch.randn(T, V, device=cuda, generator=gen) * 2.0).bfloat16()
    logits = torch.empty((chunk, V), dtype=torch.bfloat16, device=cuda)
    dh = torch.empty_like(h)
    loss_ce = torch.empty(T, device=cuda)
    loss_kl = torch.empty(T, device=cuda)
    row_sum = torch.empty(T, device=cuda)
    row_abs = torch.empty(T, device=cuda)
    sample = np.array(sorted(rs.choice(T, size=48, replace=False)))
    kept = {}
    scale = 1.0 / T
    for r0 in range(0, T, chunk):
        ops.gemm(h[r0:r0 + chunk], Wd, logits)
        for i in sample[(sample >= r0) & (sample < r0 + chunk)]:
            kept[int(i)] = logits[i - r0].float().cpu().numpy()
        ops.ce_kld(logits, tg[r0:r0 + chunk], teacher[r0:r0 + chunk], grad=logits, grad_scale=scale,
                   loss_ce=loss_ce[r0:r0 + chunk], loss_kl=loss_kl[r0:r0 + chunk])
        gf = logits.float()
        row_sum[r0:r0 + chunk] = gf.sum(1)
        row_abs[r0:r0 + chunk] = gf.abs().sum(1)
        for i in sample[(sample >= r0) & (sample < r0 + chunk)]:
            kept[("g", int(i))] = logits[i - r0].float().cpu().numpy()
        ops.gemm(logits, Wd, dh[r0:r0 + chunk], b_mn=True, N=Dm)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(loss_ce).all()) and bool(torch.isfinite(loss_kl).all())
    assert float(loss_kl.min()) >= -1e-3
    assert bool((row_sum.abs() <= 1e-2 * row_abs + 1e-7).all()), float((row_sum.abs() / row_abs).max())
    # the sampled rows against the oracle (the logits' bf16 values as both sides see them)
    lg = np.stack([kept[int(i)] for i in sample]).astype(np.float64)
    tn = teacher[torch.from_numpy(sample).to(cuda)].double().cpu().numpy()
    tgn = tg.cpu().numpy()[sample]
    lce, gce = R.ce_rows(lg, tgn, scale)
    lkl, gkl = R.kld_rows(lg, tn, scale)
    got_g = np.stack([kept[("g", int(i))] for i in sample])
    assert_close_bf16(got_g, gce + gkl, what="CE + KL gradient rows")
    np.testing.assert_allclose(loss_ce.cpu().numpy()[sample], lce, rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(loss_kl.cpu().numpy()[sample], lkl, rtol=2e-3, atol=2e-3)
    # d(hidden) of the sampled rows: the stored bf16 gradient times the head, in f64
    Wn = Wd.double().cpu().numpy()
    dh_ref = got_g.astype(np.float64) @ Wn
    assert_close_bf16(to_np(dh[torch.from_numpy(sample).to(cuda)]), dh_ref, what="d(hidden) rows")
    assert math.isfinite(float(dh.float().abs().max()))


@pytest.mark.parametrize("M,N,K,r,addend", [(256, 2048, 2048, 16, False), (1000, 1536, 512, 64, True)])
def test_qlinear_lora_entry_points_vs_oracle(cuda, M, N, K, r, addend):
    """r97b_qlinear_lora_fwd / _bwd (the decode, the adapter's narrow products and the base product in one
    call each) against the f64 rows on config 1's distributions; the backward reuses the forward's decode
    and accumulates into the gradients it is given."""
    rs = np.random.RandomState(M + r)
    s = 32.0 / 16.0
    X = _bf(rs.normal(size=(M, K)))
    A = _bf(rs.normal(size=(r, K)) / 4.0)
    B = _bf(rs.normal(size=(N, r)) * 0.01)
    dY = _bf(rs.normal(size=(M, N)) * 1e-2)
    C = _bf(rs.normal(size=(M, N))) if addend else None
    w = IQ.synth_weight(N, K, seed=M + N, device=cuda, scale_std=0.02)
    wb = torch.empty((N, K), dtype=torch.bfloat16, device=cuda)
    x, a, b, dy = (u.to(cuda) for u in (X, A, B, dY))
    y, t = ops.qlinear_lora_fwd(w, wb, x, a, b, s, addend=None if C is None else C.to(cuda))
    dA0 = torch.from_numpy(rs.normal(size=(r, K)).astype(np.float32)).to(cuda)
    dB0 = torch.from_numpy(rs.normal(size=(N, r)).astype(np.float32)).to(cuda)
    dA, dB = dA0.clone(), dB0.clone()
    dx = ops.qlinear_lora_bwd(wb, x, a, b, t, dy, s, dA, dB)
    torch.cuda.synchronize()
    Wn = to_np(IQ.dequant_bf16(w))
    assert torch.equal(wb, IQ.dequant_bf16(w))
    xn, an, bnp, dyn = (u.double().numpy() for u in (X, A, B, dY))
    y_ref, t_ref = R.lora_fwd(xn, Wn, an, bnp, s)
    if C is not None:
        y_ref = y_ref + C.double().numpy()
    dx_ref, dA_ref, dB_ref, _ = R.lora_bwd(xn, Wn, an, bnp, s, t_ref, dyn)
    assert_close_bf16(to_np(y), y_ref, what="y")
    assert_close_bf16(to_np(t), s * t_ref, what="t")
    assert_close_bf16(to_np(dx), dx_ref, what="dx")
    assert_close_bf16(to_np(dA) - to_np(dA0), dA_ref, what="dA")
    assert_close_bf16(to_np(dB) - to_np(dB0), dB_ref, what="dB")
