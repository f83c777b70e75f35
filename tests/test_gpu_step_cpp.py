"""The C++ training step (host/step.cpp, the reference's StepFn over libr97b200.so) against the Python step
(model.TrainStep) on the same model, adapter and batch: the same kernels in the same order, so the same loss
and gradients up to the float atomics whose summation order varies from run to run (the adapter-gradient
GEMMs' split-K and the GDN adjoint's per-row sums). The loss is held to 1e-5 relative and every leaf to three
times the spread of two runs of the Python step itself, at least 1e-3. Measured: most runs bit-identical; now
and then one shared-memory atomic sum in the GDN adjoint lands one ulp apart, a bf16 rounding downstream flips,
and the first layer's GDN in-projection leaves (whose gradient passes every layer's near-cancelling GDN sums)
move by 3.6e-4 -- the same outcome whichever of the two steps it happens in. Checked twice: through r97host_step_run on device buffers, and through the StepFn the reference's trainer
calls (r97host_step_call: a Batch with score masks, a ParamSet by name, the gradient ParamSet back)."""
import numpy as np
import pytest
import torch

from tests.plugin_util import rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", ["cfg5", "cfg4"])
def test_cpp_step_matches_python_step(cuda, shape):
    from r97training_b200.cstep import CStep
    from r97training_b200.model import Adapter, HybridConfig, HybridModel, TrainStep
    base = dict(hidden=256, layers=4, gdn_heads=4, gdn_qk_heads=2, attn_heads=2, attn_kv_heads=1, ffn=512,
                vocab=1024, rank=8, alpha=16.0, seq=128, micro_batch=2)
    cfg = HybridConfig(**(base if shape == "cfg5" else dict(base, attn_head_dim=128, lora_mlp=False)))
    model = HybridModel(cfg, cuda)
    ad = Adapter(model, cuda, b_std=2e-2)
    step = TrainStep(model, ad, head_chunk=128)
    cs = CStep(model, head_chunk=128)
    assert cs.numel == ad.numel
    assert [(n, o, s) for n, o, s in cs.params] == list(zip(ad.names, ad.offsets, [tuple(s) for s in ad.shapes]))
    rs = np.random.RandomState(3)
    ids = rs.randint(0, cfg.vocab, size=(cfg.micro_batch, cfg.seq)).astype(np.int32)
    score = (rs.uniform(size=ids.shape) < 0.8).astype(np.uint8)
    score[:, 0] = 0
    tg = np.full(ids.shape, -1, np.int32)
    tg[:, :-1] = np.where(score[:, 1:] == 1, ids[:, 1:], -1)
    n_scored = int((tg >= 0).sum())
    ids_d = torch.from_numpy(ids).to(cuda)
    tg_d = torch.from_numpy(tg.reshape(-1)).to(cuda)
    loss_py = float(step.run(ids_d, tg_d, n_scored=n_scored)) * n_scored
    g_py = ad.g.clone()
    ad.g.zero_()
    step.run(ids_d, tg_d, n_scored=n_scored)
    g_py2 = ad.g.clone()
    g_c = torch.zeros_like(ad.g)
    loss_c = cs.run(ids_d.reshape(-1), tg_d, n_scored, ad.w, g_c)
    torch.cuda.synchronize()
    assert abs(loss_c - loss_py) <= 1e-5 * abs(loss_py), (loss_c, loss_py)
    gp, gc, gp2 = g_py.cpu().numpy(), g_c.cpu().numpy(), g_py2.cpu().numpy()
    spread = max(rel_l2(gp2[o:o + r * c], gp[o:o + r * c]) for _, o, (r, c) in cs.params)
    bound = max(3 * spread, 1e-3)
    for name, off, (r, c) in cs.params:
        a, b = gc[off:off + r * c], gp[off:off + r * c]
        assert rel_l2(a, b) <= bound, (name, rel_l2(a, b), spread)
    # through the StepFn
    w = ad.w.cpu().numpy()
    values = {n: w[o:o + r * c] for n, o, (r, c) in cs.params}
    loss_f, scored, grads = cs.call([ids[0], ids[1]], [score[0], score[1]], values)
    assert scored == n_scored
    assert abs(loss_f - loss_py) <= 1e-5 * abs(loss_py), (loss_f, loss_py)
    for name, off, (r, c) in cs.params:
        assert rel_l2(grads[name].ravel(), gp[off:off + r * c]) <= bound, name
    cs.close()


def test_cpp_step_pads_short_sequences(cuda):
    """A Batch whose sequences are shorter than the step's length: padded, the padding unscored; the loss and
    scored count are those of the real tokens."""
    from r97training_b200.cstep import CStep
    from r97training_b200.model import Adapter, HybridConfig, HybridModel
    cfg = HybridConfig(hidden=256, layers=4, gdn_heads=4, gdn_qk_heads=2, attn_heads=2, attn_kv_heads=1, ffn=512,
                       vocab=1024, rank=8, alpha=16.0, seq=128, micro_batch=2)
    model = HybridModel(cfg, cuda)
    ad = Adapter(model, cuda)
    cs = CStep(model, head_chunk=128)
    rs = np.random.RandomState(4)
    seqs = [rs.randint(0, cfg.vocab, size=100), rs.randint(0, cfg.vocab, size=37)]
    scores = [np.r_[0, np.ones(99, np.uint8)], np.r_[0, np.ones(36, np.uint8)]]
    w = ad.w.cpu().numpy()
    loss, scored, grads = cs.call(seqs, scores, {n: w[o:o + r * c] for n, o, (r, c) in cs.params})
    assert scored == 99 + 36
    assert np.isfinite(loss) and loss > 0
    assert all(np.isfinite(g).all() for g in grads.values())
    with pytest.raises(RuntimeError):
        cs.call([rs.randint(0, cfg.vocab, size=200), seqs[1]], [np.ones(200, np.uint8), scores[1]],
                {n: w[o:o + r * c] for n, o, (r, c) in cs.params})
    cs.close()
