"""Small, self-contained cases of the hot kernels, for profiling one launch under ncu:

    python -m r97training_b200.profile_cases gemm      # the config-5 gate_up forward GEMM (8192 x 24576 x 4096)
    python -m r97training_b200.profile_cases gemm_dx   # its input adjoint (B operand MN-major)
    python -m r97training_b200.profile_cases gemm_swiglu  # the gate_up forward as the step runs it: LoRA tail,
                                                          # SwiGLU in the epilogue (8192 x 24576 x 4096 + 128)
    python -m r97training_b200.profile_cases gdn       # one config-5 GDN layer, forward + backward
    python -m r97training_b200.profile_cases decode    # the IQR decode of a 24576 x 4096 weight
    python -m r97training_b200.profile_cases norms     # rmsnorm fwd/bwd at 8192 x 4096
    python -m r97training_b200.profile_cases gnorm     # gated rmsnorm fwd/bwd at 8192 tokens x 32 heads x 128
    python -m r97training_b200.profile_cases swiglu    # SwiGLU fwd/bwd at 8192 x 12288
    python -m r97training_b200.profile_cases loss      # CE over 2048 x 151936 bf16 logits (one head chunk)
    python -m r97training_b200.profile_cases adamw     # AdamW over the config-5 adapter (160.4 M f32 params)
    python -m r97training_b200.profile_cases conv      # GDN conv prep fwd + bwd at 8192 tokens, 8192 channels
    python -m r97training_b200.profile_cases step      # one config-5 training step after one warm-up step,
                                                       # inside an NVTX range "step" (ncu --nvtx-include step/)

Each case allocates a few hundred MB to a few GB (operands larger than the 126 MB L2), runs two warm-up
launches and then the launches to capture, and exits.
"""
from __future__ import annotations

import sys

import torch


def main(case: str) -> None:
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    if case == "gemm_swiglu":
        from . import ops
        M, F, K, r = 8192, 12288, 4096, 128
        X = torch.randn(M, K, device=dev).bfloat16()
        W = (torch.randn(2 * F, K, device=dev) * 0.02).bfloat16()
        t = torch.randn(M, r, device=dev).bfloat16()
        Bb = (torch.randn(2 * F, r, device=dev) * 0.02).bfloat16()
        gu = torch.empty(M, 2 * F, device=dev, dtype=torch.bfloat16)
        a = torch.empty(M, F, device=dev, dtype=torch.bfloat16)
        for _ in range(3):
            ops.gemm(X, W, gu, a2=t, b2=Bb, mode=ops.EPI_SWIGLU, out2=a)
    elif case in ("gemm", "gemm_dx"):
        from . import ops
        M, N, K = 8192, 24576, 4096
        X = torch.randn(M, K, device=dev).bfloat16()
        W = (torch.randn(N, K, device=dev) * 0.02).bfloat16()
        if case == "gemm":
            Y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            for _ in range(3):
                ops.gemm(X, W, Y)
        else:
            dY = torch.randn(M, N, device=dev).bfloat16()
            dX = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
            for _ in range(3):
                ops.gemm(dY, W, dX, b_mn=True, N=K)
    elif case == "gdn":
        from .gdn import GdnPlan
        T, H, Hg = 8192, 32, 16
        q = torch.nn.functional.normalize(torch.randn(T, Hg, 128, device=dev), dim=-1).bfloat16()
        k = torch.nn.functional.normalize(torch.randn(T, Hg, 128, device=dev), dim=-1).bfloat16()
        v = torch.randn(T, H, 128, device=dev).bfloat16()
        g = (-torch.nn.functional.softplus(torch.randn(T, H, device=dev))).view(-1, 64, H).cumsum(1).view(T, H)
        beta = torch.sigmoid(torch.randn(T, H, device=dev))
        do = (torch.randn(T, H, 128, device=dev) * 1e-2).bfloat16()
        plan = GdnPlan([0, 4096, 8192], H, Hg, dev)
        for _ in range(2):
            o, _, sv = plan.forward(q, k, v, g.contiguous(), beta)
            plan.backward(sv, do)
    elif case == "decode":
        from . import iqr as IQ
        w = IQ.synth_weight(24576, 4096, seed=1, device=dev)
        out = torch.empty(24576, 4096, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            IQ.dequant_bf16(w, out=out)
    elif case == "norms":
        from . import ops
        x = torch.randn(8192, 4096, device=dev).bfloat16()
        dy = torch.randn(8192, 4096, device=dev).bfloat16()
        w = torch.ones(4096, device=dev)
        for _ in range(3):
            ops.rmsnorm_fwd(x, w)
            ops.rmsnorm_bwd(x, w, dy, addend=dy)
    elif case == "gnorm":
        from . import ops
        T, H = 8192, 32
        x = torch.randn(T * H, 128, device=dev).bfloat16()
        z = torch.randn(T, H * 128, device=dev).bfloat16()
        do = torch.randn(T * H, 128, device=dev).bfloat16()
        w = torch.ones(128, device=dev)
        dx, dz = torch.empty_like(x), torch.empty_like(z)
        for _ in range(3):
            ops.gated_rmsnorm_fwd(x, z, w)
            ops.gated_rmsnorm_bwd(x, z, w, do, dx=dx, dz=dz)
    elif case == "swiglu":
        from . import ops
        T, F = 8192, 12288
        gu = torch.randn(T, 2 * F, device=dev).bfloat16()
        y = torch.empty(T, F, device=dev, dtype=torch.bfloat16)
        dy = torch.randn(T, F, device=dev).bfloat16()
        dgu = torch.empty_like(gu)
        for _ in range(3):
            ops.swiglu_fwd(gu, y)
            ops.swiglu_bwd(gu, dy, dgu)
    elif case == "loss":
        from . import ops
        rows, vocab = 2048, 151936
        logits = (torch.randn(rows, vocab, device=dev) * 2).bfloat16()
        tgt = torch.randint(0, vocab, (rows,), device=dev, dtype=torch.int32)
        loss = torch.empty(rows, device=dev)
        grad = torch.empty_like(logits)
        for _ in range(3):
            ops.ce_kld(logits, tgt, loss_ce=loss, grad=grad, grad_scale=1.0 / rows)
    elif case == "adamw":
        from . import ops
        n = 160_432_128
        w = torch.randn(n, device=dev) * 0.01
        m, v, g = torch.zeros_like(w), torch.zeros_like(w), torch.randn(n, device=dev) * 1e-3
        for i in range(3):
            ops.adamw_step(w, m, v, g, lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0,
                           bc1=1.0 - 0.9 ** (i + 1), bc2=1.0 - 0.999 ** (i + 1))
    elif case == "conv":
        from . import ops
        T, Hg, H = 8192, 16, 32
        C = (2 * Hg + H) * 128
        x = torch.randn(T, C + 8256, device=dev).bfloat16()
        cw = torch.randn(C, 4, device=dev) * 0.5
        cu = torch.tensor([0, 4096, 8192], dtype=torch.int32, device=dev)
        q = torch.empty(T, Hg, 128, device=dev, dtype=torch.bfloat16)
        k, v = torch.empty_like(q), torch.empty(T, H, 128, device=dev, dtype=torch.bfloat16)
        dq, dk, dv = (torch.randn(T, H, 128, device=dev) for _ in range(3))
        dx = torch.zeros_like(x)
        for _ in range(3):
            ops.conv_prep_fwd(x, cw, cu, 2, Hg, H, q, k, v)
            ops.conv_prep_bwd(x, cw, cu, 2, Hg, H, dq, dk, dv, dx)
    elif case == "step":
        from .model import CONFIG5, Adapter, HybridModel, TrainStep
        model = HybridModel(CONFIG5, dev)
        adapter = Adapter(model, dev)
        step = TrainStep(model, adapter)
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)
        ids = torch.randint(0, CONFIG5.vocab, (CONFIG5.micro_batch, CONFIG5.seq), device=dev, generator=gen,
                            dtype=torch.int32)
        step.run(ids)
        adapter.adamw()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("step")
        step.run(ids)
        adapter.adamw()
        torch.cuda.nvtx.range_pop()
    else:
        raise SystemExit(f"unknown case {case}")
    torch.cuda.synchronize()


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "gemm")
