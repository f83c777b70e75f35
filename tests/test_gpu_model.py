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


def test_graph_replay_matches_eager_steps(cuda):
    """The step captured as one CUDA graph and replayed gives the eager step's results from the same start:
    one step's adapter gradient (captured without the update) and the losses of four steps with AdamW
    inside the graph. The runs are not bit-identical: the GDN adjoint adds some per-row terms with
    shared-memory float atomics and the adapter-gradient GEMMs reduce their split-K partials with float
    atomics, so sums land in a different order from run to run. That changes the last bits of f32 sums
    (now and then flipping a bf16 rounding downstream), so the gradient is held to relative L2 <= 5e-4 and
    cosine >= 0.9999, well inside the north star's bar (1e-2 and 0.999), and two eager runs are held to the
    same."""
    from r97training_b200.model import GraphStep
    cfg = HybridConfig(hidden=512, layers=4, gdn_heads=4, gdn_qk_heads=2, attn_heads=2, attn_kv_heads=1, ffn=1024,
                       vocab=4096, rank=16, alpha=32, seq=256, micro_batch=2, lr=1e-3)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(7)
    batches = [torch.randint(0, cfg.vocab, (cfg.micro_batch, cfg.seq), device=cuda, generator=gen,
                             dtype=torch.int32) for _ in range(4)]

    def fresh():
        model = HybridModel(cfg, cuda)
        ad = Adapter(model, cuda)
        return ad, TrainStep(model, ad, head_chunk=256)

    grads = []
    for graph in (False, False, True):
        ad, step = fresh()
        step.run(batches[0])  # eager first: attributes, encoders and buffers are set up outside a capture
        if graph:
            ad.g.zero_()
            gs = GraphStep(step, batches[0], update=False)
            gs.replay(batches[0])
        torch.cuda.synchronize()
        grads.append(ad.g.double().clone())
    for other, what in ((grads[1], "eager vs eager"), (grads[2], "graph vs eager")):
        rel = float((other - grads[0]).norm() / grads[0].norm())
        cos = float((other * grads[0]).sum() / (other.norm() * grads[0].norm()))
        assert rel <= 5e-4 and cos >= 0.9999, (what, rel, cos)

    losses = []
    for graph in (False, True):
        ad, step = fresh()
        ls = [float(step.run(batches[0]))]
        ad.adamw()
        if graph:
            gs = GraphStep(step, batches[1])
            for b in batches[1:]:
                ls.append(float(gs.replay(b)))
        else:
            for b in batches[1:]:
                ls.append(float(step.run(b)))
                ad.adamw()
        torch.cuda.synchronize()
        assert ad.step == 4
        losses.append(ls)
    for a, b in zip(*losses):
        assert abs(a - b) <= 1e-3 * abs(a), losses


def test_trained_adapter_saves_and_loads_as_peft(cuda, tmp_path):
    """The device adapter after a training step written as a PEFT directory straight from device memory
    (r97host_adapter_write) and loaded into a fresh adapter of the same model: the same f32 master weights,
    and module paths the reference's container names (`model.layers.<i>.{self_attn,linear_attn,mlp}.<proj>`)."""
    from r97training_b200 import peft
    cfg = HybridConfig(hidden=256, layers=4, gdn_heads=4, gdn_qk_heads=2, attn_heads=2, attn_kv_heads=1, ffn=512,
                       vocab=1024, rank=8, alpha=16, seq=128, micro_batch=2)
    model = HybridModel(cfg, cuda)
    ad = Adapter(model, cuda)
    step = TrainStep(model, ad, head_chunk=128)
    ids = torch.randint(0, cfg.vocab, (cfg.micro_batch, cfg.seq), device=cuda, dtype=torch.int32)
    step.run(ids)
    ad.adamw()
    torch.cuda.synchronize()
    assert "model.layers.3.self_attn.q_proj.lora_A" in ad.names
    assert "model.layers.0.linear_attn.in_proj_qkvz.lora_B" in ad.names
    assert "model.layers.0.mlp.down_proj.lora_A" in ad.names
    out = str(tmp_path / "adapter")
    peft.save_adapter(ad, out, base_model="synthetic-hybrid")
    fresh = Adapter(model, cuda)
    rank, alpha, dt = peft.load_adapter(fresh, out)
    torch.cuda.synchronize()
    assert (rank, alpha, dt) == (8, 16.0, "f32")
    assert torch.equal(fresh.w, ad.w)
    for key in ad.a_bf:
        assert torch.equal(fresh.a_bf[key], ad.a_bf[key]) and torch.equal(fresh.b_blk[key], ad.b_blk[key])
