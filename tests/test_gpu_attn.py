"""GPU parity of the attention backward (r97b_attn_bwd, the tcgen05 passes of csrc/attn.cu) against a plain
PyTorch fp32 reference of causal grouped-query attention, through the C ABI. The forward's output and
log-sum-exp come from torch's flash kernel, as in the model step. Tolerance: the north star's bf16 bar
(per-tensor relative L2 <= 1e-2, cosine >= 0.999)."""
import math

import pytest
import torch

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
    fa = torch.ops.aten._scaled_dot_product_flash_attention(q, k, v, 0.0, True, False)
    o, lse = fa[0], fa[1]
    assert o.is_contiguous() and tuple(lse.shape) == (B, Hq, S)
    ws = ops.attn_bwd_workspace(B, Hq, S, cuda)
    dq, dk, dv = ops.attn_bwd(q, k, v, o, do, lse.contiguous(), scale, ws)
    o_ref, dq_ref, dk_ref, dv_ref = _ref_grads(q, k, v, do, scale)
    torch.cuda.synchronize()
    assert_close_bf16(to_np(o), to_np(o_ref), what="o (flash forward)")
    assert_close_bf16(to_np(dv), to_np(dv_ref), what="dv")
    assert_close_bf16(to_np(dk), to_np(dk_ref), what="dk")
    assert_close_bf16(to_np(dq), to_np(dq_ref), what="dq")
    # a second call into the same workspace gives the same bits
    dq2, dk2, dv2 = ops.attn_bwd(q, k, v, o, do, lse.contiguous(), scale, ws)
    torch.cuda.synchronize()
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2) and torch.equal(dv, dv2)


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
    its LoRA tail, q/k RMSNorm, partial NeoX RoPE, causal GQA attention (flash forward, this package's
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
