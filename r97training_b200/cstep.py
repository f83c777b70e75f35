"""The training step as C++ (libr97host.so, host/step.cpp) driven from Python: the same model and adapter as
``model.TrainStep``, run by the C++ step that the reference's trainer would call as its StepFn
(r97host_step_create / _run / _call, include/r97host.h). The frozen weights stay the HybridModel's device
buffers; the C++ step owns its activations."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from . import build as B

c_i32, c_i64, c_f32, c_vp, c_u32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_uint32


class R97hostIqrWeight(ctypes.Structure):
    _fields_ = [("codes", c_vp), ("scale", c_vp), ("rows", c_i64), ("cols", c_i64), ("mad_a", c_u32),
                ("mad_b", c_u32), ("bits", c_i32), ("state_bits", c_i32), ("run_rows", c_i32), ("_pad", c_i32)]


class R97hostStepConfig(ctypes.Structure):
    _fields_ = [(n, c_i32) for n in ("hidden", "layers", "gdn_per_attn", "gdn_heads", "gdn_qk_heads", "head_k",
                                     "attn_heads", "attn_kv_heads", "attn_head_dim", "rotary_dim", "ffn", "vocab",
                                     "rank", "seq", "micro_batch", "lora_mlp", "head_chunk", "_pad")] + \
               [("alpha", c_f32), ("eps", c_f32)]


class R97hostStepWeights(ctypes.Structure):
    _fields_ = [("proj", c_vp), ("norms", c_vp), ("w_final", c_vp), ("head", R97hostIqrWeight),
                ("rope_cos", c_vp), ("rope_sin", c_vp)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(B.HOSTLIB):
            B.build_all()
        L = ctypes.CDLL(B.HOSTLIB)
        L.r97host_step_create.restype = c_vp
        L.r97host_step_create.argtypes = [c_vp, c_vp]
        L.r97host_step_destroy.argtypes = [c_vp]
        L.r97host_step_error.restype = ctypes.c_char_p
        L.r97host_step_adapter_numel.restype = c_i64
        L.r97host_step_adapter_numel.argtypes = [c_vp]
        L.r97host_step_param_count.restype = c_i32
        L.r97host_step_param_count.argtypes = [c_vp]
        L.r97host_step_param.restype = ctypes.c_char_p
        L.r97host_step_param.argtypes = [c_vp, c_i32, c_vp, c_vp, c_vp]
        L.r97host_step_arena_bytes.restype = c_i64
        L.r97host_step_arena_bytes.argtypes = [c_vp]
        L.r97host_step_run.restype = c_i32
        L.r97host_step_run.argtypes = [c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp]
        L.r97host_step_fn_new.restype = c_vp
        L.r97host_step_fn_new.argtypes = [c_vp]
        L.r97host_step_fn_free.argtypes = [c_vp]
        L.r97host_step_call.restype = c_i32
        L.r97host_step_call.argtypes = [c_vp, c_i32, c_vp, c_vp, c_vp, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]
        _lib = L
    return _lib


def _iqr(w) -> R97hostIqrWeight:
    return R97hostIqrWeight(w.codes.data_ptr(), w.scale.data_ptr(), w.rows, w.cols, w.mad_a, w.mad_b, w.bits,
                            w.state_bits, w.run_rows, 0)


class CStep:
    """The C++ step over a HybridModel's weights (device buffers kept alive by the model)."""

    def __init__(self, model, head_chunk: int = 2048):
        c = model.cfg
        self.model = model
        cfg = R97hostStepConfig(c.hidden, c.layers, c.gdn_per_attn, c.gdn_heads, c.gdn_qk_heads, c.head_k,
                                c.attn_heads, c.attn_kv_heads, c.attn_head_dim, c.rotary_dim, c.ffn, c.vocab, c.rank,
                                c.seq, c.micro_batch, int(c.lora_mlp), head_chunk, 0, c.alpha, c.eps)
        projs = [_iqr(w) for blk in model.blocks for g in blk["groups"] for w in g.iqr]
        self._proj = (R97hostIqrWeight * len(projs))(*projs)
        norms = []
        for blk in model.blocks:
            if blk["kind"] == "gdn":
                keys = ("w_in", "w_post", "conv_w", "a_log", "dt_bias", "gnorm_w")
            else:
                keys = ("w_in", "w_post", "q_norm", "k_norm", None, None)
            norms += [blk[k].data_ptr() if k else None for k in keys]
        self._norms = (c_vp * len(norms))(*norms)
        w = R97hostStepWeights(ctypes.cast(self._proj, c_vp), ctypes.cast(self._norms, c_vp), model.w_final.data_ptr(),
                               _iqr(model.head), model.rope_cos.data_ptr(), model.rope_sin.data_ptr())
        self.handle = lib().r97host_step_create(ctypes.byref(cfg), ctypes.byref(w))
        if not self.handle:
            raise RuntimeError(lib().r97host_step_error().decode())
        self.numel = int(lib().r97host_step_adapter_numel(self.handle))
        self.params = []
        for i in range(int(lib().r97host_step_param_count(self.handle))):
            off, r, cc = c_i64(), c_i64(), c_i64()
            name = lib().r97host_step_param(self.handle, i, ctypes.byref(off), ctypes.byref(r), ctypes.byref(cc))
            self.params.append((name.decode(), int(off.value), (int(r.value), int(cc.value))))

    def run(self, ids, targets, n_scored, adapter_w, adapter_g, stream=None):
        """One step on device tensors; returns the CE summed over the scored rows. The gradient is added into
        adapter_g."""
        loss = ctypes.c_double()
        s = (stream or torch.cuda.current_stream()).cuda_stream
        rc = lib().r97host_step_run(self.handle, ids.data_ptr(), targets.data_ptr(), int(n_scored),
                                    adapter_w.data_ptr(), adapter_g.data_ptr(), ctypes.byref(loss), s)
        if rc != 0:
            raise RuntimeError(lib().r97host_step_error().decode())
        return loss.value

    def call(self, seqs, scores, values):
        """Through the reference's StepFn: `seqs` / `scores` lists of int arrays (one per sequence), `values`
        {leaf name: f32 array}. Returns (loss sum, scored, {leaf name: gradient})."""
        lengths = np.array([len(s) for s in seqs], np.int64)
        ids = np.ascontiguousarray(np.concatenate(seqs).astype(np.int32))
        sc = np.ascontiguousarray(np.concatenate(scores).astype(np.uint8))
        names = [n for n, _, _ in self.params]
        shapes = np.array([s for _, _, s in self.params], np.int64).reshape(-1)
        vals = np.ascontiguousarray(np.concatenate([np.asarray(values[n], np.float32).ravel() for n in names]))
        grads = np.zeros_like(vals)
        cnames = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
        loss, scored = ctypes.c_double(), c_i64()
        rc = lib().r97host_step_call(self.handle, len(seqs), lengths.ctypes.data, ids.ctypes.data, sc.ctypes.data,
                                     len(names), ctypes.cast(cnames, c_vp), shapes.ctypes.data, vals.ctypes.data,
                                     grads.ctypes.data, ctypes.byref(loss), ctypes.byref(scored))
        if rc != 0:
            raise RuntimeError(lib().r97host_step_error().decode())
        out, off = {}, 0
        for n, _, (r, cc) in self.params:
            out[n] = grads[off:off + r * cc].reshape(r, cc)
            off += r * cc
        return loss.value, int(scored.value), out

    def close(self):
        if self.handle:
            lib().r97host_step_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
