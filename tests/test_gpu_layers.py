"""GPU parity of the block kernels around the recurrence: the GDN conv prep (causal conv + silu + q/k L2
norm) and gates, forward and backward, on ragged sequences, against the oracle pinned to the reference's
gdn_conv_prep row; and SwiGLU against silu_mul."""
import numpy as np
import pytest
import torch

from oracle import rows as R
from r97training_b200 import ops
from r97training_b200.gdn import GdnPlan
from tests.gpu_util import assert_close_bf16, to_np

pytestmark = pytest.mark.gpu


def _bf(a):
    return torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16)


@pytest.mark.parametrize("lens,Hg,H", [((200, 37, 100), 2, 4), ((4096,), 4, 8),
                                       ((1, 2, 3, 5, 1, 29, 30, 4), 2, 2),  # sequences shorter than the taps and the tiles
                                       ((7,), 1, 4),                        # one tile, partly past T; four value heads a key head
                                       ((58, 29, 87), 3, 6)])               # tile-aligned sequence ends
def test_conv_prep_fwd_bwd(cuda, lens, Hg, H):
    rs = np.random.RandomState(sum(lens))
    K = 128
    T = sum(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    C = (2 * Hg + H) * K
    extra = 64  # the projection row is wider than the conv channels (z and the gates follow)
    x = _bf(rs.normal(size=(T, C + extra)))
    w = (rs.normal(size=(C, 4)) * 0.5).astype(np.float32)
    xn = x.double().numpy()
    q, k, v = R.conv_prep_fwd(xn, w.astype(np.float64), cu, Hg, H, K)
    xd = x.to(cuda)
    cud = torch.from_numpy(cu).to(cuda)
    wd = torch.from_numpy(w).to(cuda)
    qd = torch.empty((T, Hg, K), dtype=torch.bfloat16, device=cuda)
    kd, vd = torch.empty_like(qd), torch.empty((T, H, K), dtype=torch.bfloat16, device=cuda)
    ops.conv_prep_fwd(xd, wd, cud, len(lens), Hg, H, qd, kd, vd)
    # dq, dk per value head (as the GDN backward leaves them); the adjoint sums each key head's value heads
    grp = H // Hg
    dqh, dkh = (rs.normal(size=(T, H, K)).astype(np.float32) for _ in range(2))
    dv = rs.normal(size=(T, H, K)).astype(np.float32)
    dq = dqh.reshape(T, Hg, grp, K).sum(2)
    dk = dkh.reshape(T, Hg, grp, K).sum(2)
    torch.cuda.synchronize()
    assert_close_bf16(to_np(qd), q, rel=5e-3, what="q")
    assert_close_bf16(to_np(kd), k, rel=5e-3, what="k")
    assert_close_bf16(to_np(vd), v, rel=5e-3, what="v")
    want = R.conv_prep_bwd(xn, w.astype(np.float64), cu, Hg, H, dq, dk, dv, K)
    for per_value_head in (False, True):
        dx = torch.zeros((T, C + extra), dtype=torch.bfloat16, device=cuda)
        a, b = (dqh, dkh) if per_value_head else (dq, dk)
        ops.conv_prep_bwd(xd, wd, cud, len(lens), Hg, H, torch.from_numpy(np.ascontiguousarray(a)).to(cuda),
                          torch.from_numpy(np.ascontiguousarray(b)).to(cuda), torch.from_numpy(dv).to(cuda), dx)
        torch.cuda.synchronize()
        assert_close_bf16(to_np(dx)[:, :C], want, rel=5e-3, what=f"dx (per value head: {per_value_head})")
        assert not to_np(dx)[:, C:].any()  # columns past the conv channels are not written


@pytest.mark.parametrize("H", [8, 40])
def test_gates_fwd_bwd(cuda, H):
    """ragged chunks (a 9-token sequence, chunk tails of 22 and 9 tokens) and head counts below and past a
    block's 32 heads"""
    rs = np.random.RandomState(3 + H)
    lens = (150, 64, 9)
    T = sum(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    ba = _bf(rs.normal(size=(T, 2 * H)) * 2)
    a_log = np.log(rs.uniform(1, 16, size=H)).astype(np.float32)
    dt_bias = (rs.normal(size=H) * 0.1).astype(np.float32)
    plan = GdnPlan(cu, H, H, cuda)
    g = torch.empty((T, H), dtype=torch.float32, device=cuda)
    beta = torch.empty_like(g)
    bad, al, dtb = ba.to(cuda), torch.from_numpy(a_log).to(cuda), torch.from_numpy(dt_bias).to(cuda)
    ops.gates_fwd(bad, al, dtb, plan, g, beta)
    dg, db = rs.normal(size=(T, H)).astype(np.float32), rs.normal(size=(T, H)).astype(np.float32)
    dba = torch.empty_like(bad)
    ops.gates_bwd(bad, al, dtb, plan, torch.from_numpy(dg).to(cuda), torch.from_numpy(db).to(cuda), dba)
    torch.cuda.synchronize()
    ban = ba.double().numpy()
    wg, wb = R.gates_fwd(ban[:, H:], ban[:, :H], a_log.astype(np.float64), dt_bias.astype(np.float64), cu)
    np.testing.assert_allclose(to_np(g), wg, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(to_np(beta), wb, rtol=1e-5, atol=1e-6)
    da, dbg = R.gates_bwd(ban[:, H:], ban[:, :H], a_log.astype(np.float64), dt_bias.astype(np.float64), cu, dg, db)
    assert_close_bf16(to_np(dba)[:, H:], da, rel=5e-3, what="da")
    assert_close_bf16(to_np(dba)[:, :H], dbg, rel=5e-3, what="db")


def test_swiglu(cuda):
    rs = np.random.RandomState(4)
    rows, n = 333, 1024
    gu = _bf(rs.normal(size=(rows, 2 * n)))
    dy = _bf(rs.normal(size=(rows, n)))
    y = torch.empty((rows, n), dtype=torch.bfloat16, device=cuda)
    ops.swiglu_fwd(gu.to(cuda), y)
    dgu = torch.empty((rows, 2 * n), dtype=torch.bfloat16, device=cuda)
    ops.swiglu_bwd(gu.to(cuda), dy.to(cuda), dgu)
    torch.cuda.synchronize()
    g, u, d = gu.double().numpy()[:, :n], gu.double().numpy()[:, n:], dy.double().numpy()
    sg = 1 / (1 + np.exp(-g))
    assert_close_bf16(to_np(y), g * sg * u, rel=5e-3, what="swiglu")
    assert_close_bf16(to_np(dgu)[:, :n], d * u * sg * (1 + g * (1 - sg)), rel=5e-3, what="dgate")
    assert_close_bf16(to_np(dgu)[:, n:], d * g * sg, rel=5e-3, what="dup")
