"""The reference's own training loop over the B200 step: its Trainer (src/trainer.cpp, compiled into the test
oracle from the reference tree) with its Optimiser, token-budget Batcher, checkpoint and resume, driving the
C++ StepFn of host/step.cpp (r97host_step_fn_new) -- what `Trainer::run` calls in the reference's trainer.

Checked: four steps in one run against two steps, a checkpoint, and a resumed run of two more from a fresh
start: the resumed run restores the weights, optimiser state, step and batcher position from trainer.state and
continues with the same losses and the same weights (up to the float atomics of the step's gradient sums)."""
import ctypes
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _run(cs, values, seqs, out, resume, count, total):
    lib = oracle.ref_lib()
    lib.ref_trainer_run.restype = ctypes.c_int64
    lib.ref_trainer_run.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_double,
                                    ctypes.c_int64, ctypes.c_int64, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p,
                                    ctypes.c_char_p, ctypes.c_int64]
    names = [n for n, _, _ in cs.params]
    shapes = np.array([s for _, _, s in cs.params], np.int64).reshape(-1)
    cnames = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
    vals = np.ascontiguousarray(np.concatenate([values[n].ravel() for n in names]).astype(np.float32))
    lengths = np.array([len(s) for s in seqs], np.int64)
    ids = np.ascontiguousarray(np.concatenate(seqs).astype(np.int32))
    losses = np.zeros(count, np.float64)
    ckpt = ctypes.create_string_buffer(4096)
    from r97training_b200.cstep import lib as hlib
    fn = hlib().r97host_step_fn_new(cs.handle)
    assert fn
    try:
        taken = lib.ref_trainer_run(fn, len(names), ctypes.cast(cnames, ctypes.c_void_p), shapes.ctypes.data,
                                    vals.ctypes.data, len(seqs), lengths.ctypes.data, ids.ctypes.data, 256, 1e-3,
                                    total, count, out.encode(), (resume or "").encode(), losses.ctypes.data, ckpt,
                                    4096)
    finally:
        hlib().r97host_step_fn_free(fn)
    assert taken == count, lib.ref_last_error().decode()
    res, off = {}, 0
    for n, _, (r, c) in cs.params:
        res[n] = vals[off:off + r * c].reshape(r, c).copy()
        off += r * c
    return res, losses, ckpt.value.decode()


def test_reference_trainer_drives_the_b200_step_and_resumes(cuda, tmp_path):
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")
    from r97training_b200.cstep import CStep
    from r97training_b200.model import Adapter, HybridConfig, HybridModel
    cfg = HybridConfig(hidden=256, layers=4, gdn_heads=4, gdn_qk_heads=2, attn_heads=2, attn_kv_heads=1, ffn=512,
                       vocab=1024, rank=8, alpha=16.0, seq=128, micro_batch=2)
    model = HybridModel(cfg, cuda)
    ad = Adapter(model, cuda, b_std=2e-2)
    cs = CStep(model, head_chunk=128)
    w = ad.w.cpu().numpy()
    init = {n: w[o:o + r * c].reshape(r, c).copy() for n, o, (r, c) in cs.params}
    rs = np.random.RandomState(12)
    # lengths above a third of the 256-token budget: at most two sequences a step, each within the step's 128
    seqs = [rs.randint(0, cfg.vocab, size=rs.randint(96, 129)) for _ in range(24)]
    full, losses_full, _ = _run(cs, init, seqs, str(tmp_path / "a"), None, 4, 4)
    half, losses_half, ckpt = _run(cs, init, seqs, str(tmp_path / "b"), None, 2, 4)
    assert os.path.exists(os.path.join(ckpt, "trainer.state")) and os.path.exists(os.path.join(ckpt, "adapter",
                                                                                                  "adapter.marker"))
    fresh = {n: np.zeros_like(v) for n, v in init.items()}  # the resume replaces these with the checkpoint's
    rest, losses_rest, _ = _run(cs, fresh, seqs, str(tmp_path / "b"), ckpt, 2, 4)
    cs.close()
    assert np.all(np.isfinite(losses_full)) and np.all(losses_full > 0)
    np.testing.assert_allclose(losses_half, losses_full[:2], rtol=1e-4)
    np.testing.assert_allclose(losses_rest, losses_full[2:], rtol=1e-3)
    a = np.concatenate([full[n].ravel() - init[n].ravel() for n in init])
    b = np.concatenate([rest[n].ravel() - init[n].ravel() for n in init])
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    assert cos >= 0.99, cos  # AdamW's first steps move each weight by ~lr whatever the gradient's size
    assert any(np.abs(full[n] - init[n]).max() > 0 for n in init)
