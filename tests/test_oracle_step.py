"""The composed reference step (oracle/step.py: the hybrid model's forward through the reference's own
twins, its reverse walk through the reference's own host adjoints) checked on the CPU against central finite
differences of its own forward: every LoRA factor gradient it returns is the derivative of the loss it
returns, so the walk wires the rows in the right order. A small 2-block hybrid (one GDN block, one gated
attention block) over two 80-token sequences, f64 throughout."""
import numpy as np
import pytest
import torch

import oracle


def _tiny():
    from oracle import step as S
    from r97training_b200.model import HybridConfig, HybridModel, groups_of, module_path
    cfg = HybridConfig(hidden=128, layers=2, gdn_per_attn=1, gdn_heads=4, gdn_qk_heads=2, head_k=32, attn_heads=4,
                       attn_kv_heads=2, attn_head_dim=32, rotary_dim=16, ffn=128, vocab=256, rank=4, alpha=8.0,
                       seq=80, micro_batch=2)
    model = HybridModel(cfg, torch.device("cpu"))
    rs = np.random.RandomState(0)
    lora = {}
    for li, kind in enumerate(cfg.kinds):
        for _, k, projs in groups_of(cfg, kind):
            for pname, n in projs:
                p = module_path(li, kind, pname)
                lora[p + ".lora_A"] = rs.uniform(-1, 1, size=(cfg.rank, k)) / np.sqrt(k)
                lora[p + ".lora_B"] = rs.normal(size=(n, cfg.rank)) * 0.05
    m = S.model_from_torch(model, lora)
    ids = rs.randint(0, cfg.vocab, size=(cfg.micro_batch, cfg.seq))
    tg = np.concatenate([ids[:, 1:], -np.ones((cfg.micro_batch, 1), int)], axis=1)
    return m, ids, tg


def test_composed_reference_step_matches_finite_differences():
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")
    from oracle import step as S
    m, ids, tg = _tiny()
    loss, grads = S.reference_step(m, ids, tg, f64_loss=True)
    assert np.isfinite(loss) and loss > 0
    assert sorted(grads) == sorted(m["lora"]), "every LoRA factor gets a gradient"
    rs = np.random.RandomState(1)
    names = ["model.layers.0.linear_attn.in_proj_qkvz.lora_A", "model.layers.0.linear_attn.in_proj_ba.lora_B",
             "model.layers.0.linear_attn.out_proj.lora_A", "model.layers.0.mlp.gate_proj.lora_B",
             "model.layers.1.self_attn.q_proj.lora_A", "model.layers.1.self_attn.k_proj.lora_B",
             "model.layers.1.self_attn.v_proj.lora_A", "model.layers.1.self_attn.o_proj.lora_B",
             "model.layers.1.mlp.down_proj.lora_A"]
    eps = 1e-4
    for name in names:
        w = m["lora"][name]
        idx = tuple(rs.randint(0, s) for s in w.shape)
        g = float(grads[name].reshape(w.shape)[idx])
        old = w[idx]
        w[idx] = old + eps
        lp, _ = S.reference_step(m, ids, tg, backward=False, f64_loss=True)
        w[idx] = old - eps
        lm, _ = S.reference_step(m, ids, tg, backward=False, f64_loss=True)
        w[idx] = old
        fd = (lp - lm) / (2 * eps)
        # the gradient is stored as f32 (the reference's ParamSet): compare at f32 resolution
        assert abs(fd - g) <= 2e-5 * max(abs(fd), abs(g)) + 1e-9, (name, idx, fd, g)


def test_bf16_storage_replay_is_deterministic_and_scoped():
    """The rows replayed at the B200 step's storage precision: the same loss and gradients on a second call
    (the reference's rows are deterministic), a loss within bf16 rounding of the exact step's, and the mode
    ends with the call."""
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")
    from oracle import step as S
    m, ids, tg = _tiny()
    l0, _ = S.reference_step(m, ids, tg, backward=False)
    l1, g1 = S.reference_step(m, ids, tg, bf16_store=True)
    l2, g2 = S.reference_step(m, ids, tg, bf16_store=True)
    assert l1 == l2 and all(np.array_equal(g1[n], g2[n]) for n in g1)
    assert abs(l1 - l0) <= 1e-2 * abs(l0), (l0, l1)
    assert S._store is S._exact
