"""GPU parity of the attention core on this package's tcgen05 kernels, through the C ABI: the forward
(r97b_attn_fwd, csrc/attn_fwd.cu) against the oracle's attention restatement (oracle/rows.py attention_fwd,
pinned to the reference's own attn_paged twin) and a plain PyTorch fp32 reference, and the backward
(r97b_attn_bwd, csrc/attn.cu) from that forward's output and log-sum-exp, against fp32 autograd and the
oracle's attention_bwd (pinned to the reference's host adjoint). Tolerance: the north star's bf16 bar (per-tensor
relative L2 <= 1e-2, cosine >= 0.999); the log-sum-exp, an f32 output, to 1e-4 absolute."""
import math

import numpy as np
import pytest
import torch

from oracle import rows as R
from r97training_b200 import ops
from tests.gpu_util import assert_close_bf16, to_np

pytestmark = pytest.mark.gpu


def _ref_grads(q, k, v, do, scale):
    """fp32 autograd of softmax(scale q k^T, causal) v with k/v shared by groups of query heads."""
    grp = q.shape[1] // k.shape[1]
    qf, kf, vf = (t.float().detach().requires_grad_(True) for t in (q, k, v))
    ke, ve = kf.repeat_interleave(grp, dim=1), vf.repeat_interleave(grp, dim=1)
    s = torch.matmul(qf, ke.transpose(-1, -2)) * scale
    S = q.shape[2]
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
    p = torch.softmax(s.masked_fill(mask, float("-inf")), dim=-1)
    o = torch.matmul(p, ve)
    o.backward(do.float())
    return o.detach(), qf.grad, kf.grad, vf.grad


@pytest.mark.parametrize("B,Hq,Hkv,S,D", [(1, 4, 2, 256, 256), (2, 4, 1, 384, 128), (1, 2, 2, 128, 256),
                                          (1, 8, 2, 640, 256)])
def test_attn_bwd_vs_fp32(cuda, B, Hq, Hkv, S, D):
    g = torch.Generator(device=cuda).manual_seed(B * 1000 + Hq * 100 + S + D)
    q = torch.randn(B, Hq, S, D, device=cuda, generator=g).bfloat16()
    k = torch.randn(B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    v = torch.randn(B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    do = (torch.randn(B, Hq, S, D, device=cuda, generator=g) * 0.1).bfloat16()
    scale = 1.0 / math.sqrt(D)
    o, lse = ops.attn_fwd(q, k, v, scale)
    assert o.is_contiguous() and tuple(lse.shape) == (B, Hq, S)
    ws = ops.attn_bwd_workspace(B, Hq, S, cuda)
    dq, dk, dv = ops.attn_bwd(q, k, v, o, do, lse.contiguous(), scale, ws)
    o_ref, dq_ref, dk_ref, dv_ref = _ref_grads(q, k, v, do, scale)
    torch.cuda.synchronize()
    assert_close_bf16(to_np(o), to_np(o_ref), what="o (forward)")
    assert_close_bf16(to_np(dv), to_np(dv_ref), what="dv")
    assert_close_bf16(to_np(dk), to_np(dk_ref), what="dk")
    assert_close_bf16(to_np(dq), to_np(dq_ref), what="dq")
    # a second call into the same workspace gives the same bits
    dq2, dk2, dv2 = ops.attn_bwd(q, k, v, o, do, lse.contiguous(), scale, ws)
    torch.cuda.synchronize()
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2) and torch.equal(dv, dv2)


@pytest.mark.parametrize("B,Hq,Hkv,S,D", [(1, 2, 1, 128, 256), (2, 4, 2, 384, 128), (1, 3, 3, 256, 256),
                                          (1, 4, 1, 640, 128)])
def test_attn_fwd_vs_oracle(cuda, B, Hq, Hkv, S, D):
    """The forward's output and log-sum-exp against the oracle's f64 attention (the reference's attn_paged
    twin's arithmetic) on the same bf16 inputs, plus a second call into fresh outputs giving the same bits."""
    rs = np.random.RandomState(B * 7 + Hq * 5 + S + D)
    qn = rs.normal(size=(B, Hq, S, D))
    kn = rs.normal(size=(B, Hkv, S, D))
    vn = rs.normal(size=(B, Hkv, S, D))
    q, k, v = (torch.from_numpy(a).float().bfloat16().to(cuda) for a in (qn, kn, vn))
    scale = 1.0 / math.sqrt(D)
    o, lse = ops.attn_fwd(q, k, v, scale)
    o2, lse2 = ops.attn_fwd(q, k, v, scale)
    torch.cuda.synchronize()
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
    qf, kf, vf = (t.double().cpu().numpy() for t in (q, k, v))
    for b in range(B):
        # the oracle's layout: [tokens, heads, D]
        want = R.attention_fwd(qf[b].transpose(1, 0, 2), kf[b].transpose(1, 0, 2), vf[b].transpose(1, 0, 2),
                               scale).transpose(1, 0, 2)
        assert_close_bf16(to_np(o[b]), want, what=f"o[{b}]")
        s_ = np.einsum("hsd,htd->hst", qf[b], np.repeat(kf[b], Hq // Hkv, axis=0)) * scale
        s_ = np.where(np.triu(np.ones((S, S), bool), 1)[None], -np.inf, s_)
        mx = s_.max(-1)
        want_lse = mx + np.log(np.exp(s_ - mx[..., None]).sum(-1))
        np.testing.assert_allclose(lse[b].cpu().numpy(), want_lse, rtol=0, atol=1e-4)


def test_attn_fwd_rejects_bad_shapes(cuda):
    q = torch.zeros(1, 2, 100, 256, device=cuda, dtype=torch.bfloat16)  # S not a multiple of 128
    with pytest.raises(Exception):
        ops.attn_fwd(q, q[:, :1], q[:, :1], 0.0625)
    q = torch.zeros(1, 2, 128, 192, device=cuda, dtype=torch.bfloat16)  # D neither 128 nor 256
    with pytest.raises(Exception):
        ops.attn_fwd(q, q[:, :1].contiguous(), q[:, :1].contiguous(), 0.0625)


def test_attn_bwd_rejects_bad_shapes(cuda):
    q = torch.zeros(1, 2, 100, 256, device=cuda, dtype=torch.bfloat16)  # S not a multiple of 128
    k = torch.zeros(1, 1, 100, 256, device=cuda, dtype=torch.bfloat16)
    lse = torch.zeros(1, 2, 100, device=cuda)
    ws = torch.empty(1 << 20, dtype=torch.uint8, device=cuda)
    with pytest.raises(Exception):
        ops.attn_bwd(q, k, k, q, q, lse, 0.0625, ws)


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope(x, cos, sin, rot):
    """partial NeoX rotation of the first `rot` dims: pairs (j, j + rot/2), positions along dim -2."""
    half = rot // 2
    x1, x2, rest = x[..., :half], x[..., half:rot], x[..., rot:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin, rest], dim=-1)


@pytest.mark.parametrize("Dh,rot", [(256, 64), (128, 64), (128, 32)])
def test_attention_block_vs_fp32(cuda, Dh, rot):
    """The whole gated-attention sublayer of the model step -- RMSNorm, the fused q(+gate)/k/v projection with
    its LoRA tail, q/k RMSNorm, partial NeoX RoPE, causal GQA attention (this package's forward and
    backward), the sigmoid output gate, the o projection with its LoRA tail and the residual -- forward and
    backward through TrainStep, against an fp32 autograd restatement on the same decoded weights and adapter
    (the reference's attention twin/adjoint arithmetic, src/adjoint/host/attention.cpp:261-414)."""
    from r97training_b200 import iqr as IQ
    from r97training_b200.model import Adapter, HybridConfig, HybridModel, TrainStep
    cfg = HybridConfig(hidden=512, layers=4, gdn_heads=4, gdn_qk_heads=2, attn_heads=4, attn_kv_heads=2, ffn=512,
                       vocab=512, rank=8, alpha=16, seq=256, micro_batch=2, attn_head_dim=Dh, rotary_dim=rot)
    model = HybridModel(cfg, cuda)
    ad = Adapter(model, cuda, b_std=0.05)
    step = TrainStep(model, ad, head_chunk=128)
    li = 3
    blk = model.blocks[li]
    assert blk["kind"] == "attn"
    T, d, Dh, Hq, Hkv, S, B = cfg.tokens, cfg.hidden, cfg.attn_head_dim, cfg.attn_heads, cfg.attn_kv_heads, cfg.seq, \
        cfg.micro_batch
    g = torch.Generator(device=cuda).manual_seed(11)
    x = torch.randn(T, d, device=cuda, generator=g).bfloat16()
    dh1 = (torch.randn(T, d, device=cuda, generator=g) * 0.1).bfloat16()
    sv = {}
    h1 = step._attn_fwd(li, blk, x, sv)
    ad.g.zero_()
    dx = step._attn_bwd(li, blk, x, sv, dh1)
    torch.cuda.synchronize()

    s = cfg.lora_scale
    g_qkv, g_o = blk["groups"][0], blk["groups"][1]

    def weights(grp):
        W = torch.cat([IQ.dequant_bf16(w).float() for w in grp.iqr], 0)
        A = ad.a_view(ad.w, grp).detach().clone().requires_grad_(True)
        Bs = [ad.b_view(ad.w, grp, i).detach().clone().requires_grad_(True) for i in range(len(grp.projs))]
        return W, A, Bs

    def lin(xin, grp, W, A, Bs):
        r = cfg.rank
        t = xin @ A.t()
        lora = torch.cat([(t[:, i * r:(i + 1) * r] @ Bs[i].t()) for i in range(len(Bs))], 1)
        return xin @ W.t() + s * lora

    Wq, Aq, Bq = weights(g_qkv)
    Wo, Ao, Bo = weights(g_o)
    xf = x.float().requires_grad_(True)
    n1 = _rms(xf, blk["w_in"], cfg.eps)
    y = lin(n1, g_qkv, Wq, Aq, Bq)
    qn = 2 * Hq * Dh
    yq = y[:, :qn].view(B, S, Hq, 2 * Dh)
    q, gate = yq[..., :Dh], yq[..., Dh:]
    k = y[:, qn:qn + Hkv * Dh].view(B, S, Hkv, Dh)
    v = y[:, qn + Hkv * Dh:].view(B, S, Hkv, Dh)
    cos, sin = model.rope_cos[:S][None, :, None, :], model.rope_sin[:S][None, :, None, :]
    q = _rope(_rms(q, blk["q_norm"], cfg.eps), cos, sin, cfg.rotary_dim).transpose(1, 2)
    k = _rope(_rms(k, blk["k_norm"], cfg.eps), cos, sin, cfg.rotary_dim).transpose(1, 2)
    v = v.transpose(1, 2)
    grp = Hq // Hkv
    sc = (q @ k.repeat_interleave(grp, 1).transpose(-1, -2)) / math.sqrt(Dh)
    mask = torch.ones(S, S, dtype=torch.bool, device=cuda).triu(1)
    attn = torch.softmax(sc.masked_fill(mask, float("-inf")), -1) @ v.repeat_interleave(grp, 1)
    ga = (attn.transpose(1, 2) * torch.sigmoid(gate)).reshape(T, Hq * Dh)
    ref_h1 = xf + lin(ga, g_o, Wo, Ao, Bo)
    ref_h1.backward(dh1.float())
    assert_close_bf16(to_np(h1), to_np(ref_h1), what="h1")
    assert_close_bf16(to_np(dx), to_np(xf.grad), what="dx")
    for grp_, A, Bs, name in ((g_qkv, Aq, Bq, "qkv"), (g_o, Ao, Bo, "o")):
        assert_close_bf16(to_np(ad.a_view(ad.g, grp_)), to_np(A.grad), what=f"dA {name}")
        for i in range(len(Bs)):
            assert_close_bf16(to_np(ad.b_view(ad.g, grp_, i)), to_np(Bs[i].grad), what=f"dB {name}.{i}")
