"""The whole LoRA step of a small hybrid model on the GPU: several steps of forward, CE, backward and
AdamW stay finite, reduce the loss on a fixed batch, and give every adapter leaf a gradient."""
import pytest
import torch

from r97training_b200.model import Adapter, HybridConfig, HybridModel, TrainStep

pytestmark = pytest.mark.gpu


def test_small_hybrid_steps_are_finite_and_learn(cuda):
    cfg = HybridConfig(hidden=512, layers=4, gdn_heads=4, gdn_qk_heads=2, attn_heads=2, attn_kv_heads=1, ffn=1024,
                       vocab=4096, rank=16, alpha=32, seq=256, micro_batch=2, lr=1e-3)
    model = HybridModel(cfg, cuda)
    ad = Adapter(model, cuda)
    step = TrainStep(model, ad, head_chunk=256)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(5)
    ids = torch.randint(0, cfg.vocab, (cfg.micro_batch, cfg.seq), device=cuda, generator=gen, dtype=torch.int32)
    losses = []
    for i in range(6):
        loss = step.run(ids)
        assert bool(torch.isfinite(ad.g).all()), f"non-finite gradient at step {i}"
        if i == 0:
            for name, shape, off in zip(ad.names, ad.shapes, ad.offsets):
                n = shape[0] * shape[1]
                assert float(ad.g[off:off + n].abs().max()) > 0, f"{name} got no gradient"
        ad.adamw()
        losses.append(float(loss))
    assert all(torch.isfinite(torch.tensor(losses))), losses
    assert losses[-1] < losses[0], losses
