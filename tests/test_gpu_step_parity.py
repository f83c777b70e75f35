"""Whole-step parity: one LoRA training step of a small hybrid model on the B200 kernels (TrainStep: decode,
fused LoRA GEMMs, conv prep, GDN, gated attention, MLP, chunked head + CE, the fixed reverse walk) against
the same step composed from the reference's OWN rows in f64 (oracle/step.py: every twin and host adjoint
through the reference's registry, the reference_step.cpp pattern), on the same seeded base weights, adapter
and token ids. The bar is the north star's: the loss, and every adapter leaf's gradient at per-tensor
relative L2 <= 1e-2 and cosine >= 0.999."""
import numpy as np
import pytest
import torch

import oracle
from tests.plugin_util import cosine, rel_l2

pytestmark = pytest.mark.gpu


def _run(cuda, cfg, seed, b_std):
    from oracle import step as S
    from r97training_b200.model import Adapter, HybridModel, TrainStep
    model = HybridModel(cfg, cuda)
    ad = Adapter(model, cuda, b_std=b_std)
    step = TrainStep(model, ad, head_chunk=128)
    rs = np.random.RandomState(seed)
    ids = rs.randint(0, cfg.vocab, size=(cfg.micro_batch, cfg.seq)).astype(np.int32)
    loss = float(step.run(torch.from_numpy(ids).to(cuda)))
    torch.cuda.synchronize()
    g = ad.g.cpu().numpy()
    w = ad.w.cpu().numpy()
    lora, mine = {}, {}
    for name, shape, off in zip(ad.names, ad.shapes, ad.offsets):
        n = shape[0] * shape[1]
        lora[name] = w[off:off + n].reshape(shape)
        mine[name] = g[off:off + n].reshape(shape)
    tg = np.concatenate([ids[:, 1:], -np.ones((cfg.micro_batch, 1), np.int32)], axis=1)
    ref_loss, ref = S.reference_step(S.model_from_torch(model, lora), ids, tg)
    return loss, ref_loss, mine, ref


@pytest.mark.parametrize("b_std", [1e-3, 2e-2])
def test_step_loss_and_every_adapter_gradient_vs_reference_rows(cuda, b_std):
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")
    from r97training_b200.model import HybridConfig
    cfg = HybridConfig(hidden=256, layers=4, gdn_heads=4, gdn_qk_heads=2, attn_heads=2, attn_kv_heads=1, ffn=512,
                       vocab=1024, rank=8, alpha=16.0, seq=128, micro_batch=2)
    loss, ref_loss, mine, ref = _run(cuda, cfg, seed=11, b_std=b_std)
    assert abs(loss - ref_loss) <= 2e-3 * abs(ref_loss), (loss, ref_loss)
    assert sorted(mine) == sorted(ref)
    worst = []
    for name in sorted(ref):
        r, c = rel_l2(mine[name], ref[name]), cosine(mine[name], ref[name])
        worst.append((r, c, name))
        assert r <= 1e-2 and c >= 0.999, f"{name}: rel_l2 {r:.3e} cosine {c:.6f}"
    worst.sort(reverse=True)
    print(f"\nstep parity (B std {b_std}): loss {loss:.6f} vs {ref_loss:.6f}; worst leaves "
          + "; ".join(f"{n} rel {r:.2e} cos {c:.6f}" for r, c, n in worst[:3]))
