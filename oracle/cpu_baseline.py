"""TEST INFRASTRUCTURE / CPU BASELINE -- times the reference's OWN host rows (oracle/_ref/libr97ref.so,
compiled from the reference tree) on a bounded sample of the bench workload and extrapolates a
tokens/s figure. Used only by bench.py's cpu_baseline leg and its `--impl reference` arm.

What one sampled "step" runs, all through the reference's registry (twin + host adjoint per op):
  * one GDN block and one attention block's rows on 8 and on M sampled tokens: rmsnorm x2, every
    projection's gemm_nt on its stored IQR weight (twin + dX adjoint), its lora_shrink / lora_expand (twins +
    adjoints, dA/dB), gdn_gated_rmsnorm, silu_mul; the per-token slope between the two plus the calls' fixed
    cost once per step, scaled by the 24 / 8 block counts;
  * gdn_kkt_solve + gdn_chunk_scan (twins + adjoints) on one 64-token chunk of every value head, scaled
    per token;
  * the tied head: logits_gemm twin + adjoint on 8 and M tokens, ce_position per row, fitted the same way;
  * the IQR decode (r97_iqr_decode_host) of one 4096 x 4096 weight, scaled to every base weight once per
    step of 8192 tokens, and one AdamW Optimiser update of 16M parameters scaled to the adapter size.
Not timed: the causal attention core (about 3% of the step's FLOPs), the conv prep and the gates
(elementwise). The reference's full host-only step (R97_WITH_HIP=OFF r97train) needs radiance, which
is absent, so this per-op composition of the same host rows stands in for it.
"""
from __future__ import annotations

import os
import time

import numpy as np

from . import Operand, ref_adjoint, ref_lib, ref_twin
from . import rows as R


def _stored(n, k, rs):
    codes = rs.randint(-126, 127, size=(n, k), dtype=np.int8)
    sc = np.abs(rs.normal(0, 0.02, size=(n, k // 128))).astype(np.float32)
    u = sc.view(np.uint32)
    return codes, ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _linear(M, n, k, r, rs, scale=2.0):
    """gemm_nt (stored weight) + lora_shrink + lora_expand twins and adjoints for one projection; returns
    the timed part as a callable (inputs are generated before it)."""
    x = rs.normal(size=(M, k))
    dy = rs.normal(size=(M, n)) * 1e-2
    codes, sb = _stored(n, k, rs)
    A = rs.normal(size=(1, r, k)) * 0.02
    B = rs.normal(size=(1, n, r)) * 0.01
    return lambda: _linear_run(M, n, k, r, x, dy, codes, sb, A, B, scale)


def _linear_run(M, n, k, r, x, dy, codes, sb, A, B, scale):
    ops = [Operand("a", "bf16", (M, k)), Operand("b", "iqr", (n, k), stored=(codes, sb)),
           Operand("y", "bf16", (M, n), written=True)]
    p = {"M": M, "N": n, "K": k}
    y = ref_twin("gemm_nt", p, ops, {"a": x, "b": None})["y"]
    ref_adjoint("gemm_nt", p, ops, {"a": x, "b": None, "y": y}, {"y": dy})
    slot = np.zeros(M)
    sh = [Operand("a", "bf16", (M, k)), Operand("none:1", "invalid", (0,)), Operand("slot", "i32", (M,)),
          Operand("lora_a", "f32", (1, r, k)), Operand("t", "f32", (M, r), written=True)]
    t = ref_twin("lora_shrink", {}, sh, {"a": x, "none:1": None, "slot": slot, "lora_a": A})["t"]
    ex = [Operand("t", "f32", (M, r)), Operand("slot", "i32", (M,)), Operand("lora_b", "f32", (1, n, r)),
          Operand("scale", "f32", (1, n)), Operand("y", "bf16", (M, n), written=True)]
    sc = np.full((1, n), scale)
    y2 = ref_twin("lora_expand", {}, ex, {"t": t, "slot": slot, "lora_b": B, "scale": sc})["y"]
    dc, _ = ref_adjoint("lora_expand", {}, ex, {"t": t, "slot": slot, "lora_b": B, "scale": sc, "y": y2}, {"y": dy})
    ref_adjoint("lora_shrink", {}, sh, {"a": x, "none:1": None, "slot": slot, "lora_a": A, "t": t}, {"t": dc["t"]})


def _rmsnorm(M, n, rs):
    x, w, dy = rs.normal(size=(M, n)), rs.normal(size=n), rs.normal(size=(M, n))
    ops = [Operand("x", "bf16", (M, n)), Operand("w", "f32", (n,)), Operand("y", "bf16", (M, n), written=True)]
    y = ref_twin("rmsnorm", {"eps": "1e-06"}, ops, {"x": x, "w": w})["y"]
    ref_adjoint("rmsnorm", {"eps": "1e-06"}, ops, {"x": x, "w": w, "y": y}, {"y": dy})


def _silu_mul(M, n, rs):
    x, dy = rs.normal(size=(M, 2 * n)), rs.normal(size=(M, n))
    ops = [Operand("gate_up", "bf16", (M, 2 * n)), Operand("y", "bf16", (M, n), written=True)]
    y = ref_twin("silu_mul", {"n": n}, ops, {"gate_up": x})["y"]
    ref_adjoint("silu_mul", {"n": n}, ops, {"gate_up": x, "y": y}, {"y": dy})


def _gated_norm(rows, rs):
    x, z, w, do = rs.normal(size=(rows, 128)), rs.normal(size=(rows, 128)), rs.normal(size=128), rs.normal(size=(rows, 128))
    ops = [Operand("x", "bf16", (rows, 128)), Operand("z", "bf16", (rows, 128)), Operand("w", "f32", (128,)),
           Operand("o", "bf16", (rows, 128), written=True)]
    o = ref_twin("gdn_gated_rmsnorm", {"channels": 128}, ops, {"x": x, "z": z, "w": w})["o"]
    ref_adjoint("gdn_gated_rmsnorm", {"channels": 128}, ops, {"x": x, "z": z, "w": w, "o": o}, {"o": do})


def _gdn_core(T, H, Hg, rs):
    from .gdn import synth_inputs
    d = synth_inputs([T], H, Hg, seed=int(rs.randint(1 << 30)))
    S = 1
    kk = [Operand("k", "bf16", (T, Hg, 128)), Operand("beta", "f32", (T, H)), Operand("g", "f32", (T, H)),
          Operand("cu_seqlens", "i32", (S + 1,)), Operand("A", "bf16", (T, H, 64), written=True)]
    p = {"chunk": 64, "head_k": 128}
    A = ref_twin("gdn_kkt_solve", p, kk, {"k": d["k"], "beta": d["beta"], "g": d["g"], "cu_seqlens": d["cu"]})["A"]
    sc = [Operand("q", "bf16", (T, Hg, 128)), Operand("k", "bf16", (T, Hg, 128)), Operand("v", "bf16", (T, H, 128)),
          Operand("A", "bf16", (T, H, 64)), Operand("g", "f32", (T, H)), Operand("beta", "f32", (T, H)),
          Operand("h0", "f32", (S, H, 128, 128)), Operand("cu_seqlens", "i32", (S + 1,)),
          Operand("o", "bf16", (T, H, 128), written=True), Operand("ht", "f32", (S, H, 128, 128), written=True),
          Operand("state_idx", "i32", (S,))]
    ps = {"head_k": 128, "head_v": 128, "chunk": 64}
    reads = dict(q=d["q"], k=d["k"], v=d["v"], A=A, g=d["g"], beta=d["beta"], h0=np.zeros((S, H, 128, 128)),
                 cu_seqlens=d["cu"], state_idx=np.zeros(S))
    out = ref_twin("gdn_chunk_scan", ps, sc, reads)
    dc, _ = ref_adjoint("gdn_chunk_scan", ps, sc, dict(reads, **out), {"o": d["do"], "ht": np.zeros((S, H, 128, 128))})
    ref_adjoint("gdn_kkt_solve", p, kk, {"k": d["k"], "beta": d["beta"], "g": d["g"], "cu_seqlens": d["cu"], "A": A},
                {"A": dc["A"]})


def _head(M, vocab, d, rs):
    x = rs.normal(size=(M, d))
    codes, sb = _stored(vocab, d, rs)
    tg = rs.randint(vocab, size=M)
    return lambda: _head_run(M, vocab, d, x, codes, sb, tg)


def _head_run(M, vocab, d, x, codes, sb, tg):
    ops = [Operand("x", "bf16", (M, d)), Operand("lm_head", "iqr", (vocab, d), stored=(codes, sb)),
           Operand("logits", "f32", (M, vocab), written=True)]
    p = {"n_embd": d, "n_vocab": vocab}
    lg = ref_twin("logits_gemm", p, ops, {"x": x, "lm_head": None})["logits"]
    lib = ref_lib()
    grad = np.zeros((M, vocab), np.float64)
    for i in range(M):
        row = np.ascontiguousarray(lg[i].astype(np.float32))
        g = np.zeros(vocab, np.float32)
        lib.ref_ce_position(row.ctypes.data, vocab, int(tg[i]), g.ctypes.data, 1.0 / 8192)
        grad[i] = g
    ref_adjoint("logits_gemm", p, ops, {"x": x, "lm_head": None, "logits": lg}, {"logits": grad})


# The row slices are sized for this many tokens whatever M is, so every M times the same slices (the same
# fixed cost per call) and a larger M only costs proportionally more.
_M_SLICE = 64


def _best(run, reps: int = 2) -> float:
    """The shortest of `reps` timings of run() (the host's other load only ever adds time)."""
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        run()
        best = min(best, time.perf_counter() - t0)
    return best


# The few tokens every part is also timed on: the difference to M tokens is the marginal cost.
_M_FEW = 8


def _fit(t1: float, t2: float, m1: int, m2: int):
    """(seconds per token, fixed seconds per call) from a part timed on m1 and on m2 > m1 tokens: the
    difference is the marginal cost of m2 - m1 tokens; what is left of the first time is the call's fixed
    cost (staging the operands, the stored weight's table), which a real step pays once per layer for all of
    its tokens."""
    slope = max(0.0, (t2 - t1) / (m2 - m1))
    return slope, max(0.0, t1 - slope * m1)


def sample_step(cfg, M: int, seed: int = 0, macs_budget: float = 0.6e9) -> dict:
    """Runs one bounded sample and returns {part: seconds} plus the extrapolated seconds per token.
    `cfg` is a plain dict: hidden, ffn, rank, alpha, vocab, gdn_heads, gdn_qk_heads, seq, micro_batch,
    kinds (the block kinds), groups ({kind: [(group, in width, [(projection, out width)])]}),
    base_weights (elements of every base weight incl. the head) and adapter_params.

    The sample is bounded by slicing output rows: a projection's rows cost the same each, so a
    projection of n rows is run on n / f of them and its time scaled by f, with f chosen so one block
    kind's products on 2 x 64 tokens stay near `macs_budget` multiply-adds (and likewise the head's vocabulary
    rows); each timing is the best of two.
    Each block kind and the head run on 8 and on M (> 8) tokens: the per-token cost is the slope between
    the two, and the rest -- the rows' fixed cost per call -- is charged once per step of seq x micro_batch
    tokens, the way the reference's step calls each row once per layer for all of its tokens. The estimate
    therefore does not depend on M beyond the timing noise."""
    rs = np.random.RandomState(seed)
    parts = {}
    r = cfg["rank"]
    step_tokens = cfg["seq"] * cfg["micro_batch"]

    def block(kind, m, f):
        projs = [(n, k) for _, k, pr in cfg["groups"][kind] for _, n in pr]
        sliced = []
        for n, k in projs:
            ns = max(64, int(round(n / f / 64)) * 64) if n > 64 else n
            sliced.append((n / ns, _linear(m, ns, k, r, rs, cfg["alpha"] / r)))
        t = 0.0
        t0 = time.perf_counter()
        _rmsnorm(m, cfg["hidden"], rs)
        _rmsnorm(m, cfg["hidden"], rs)
        _silu_mul(m, cfg["ffn"], rs)
        if kind == "gdn":
            _gated_norm(m * cfg["gdn_heads"], rs)
        t += time.perf_counter() - t0
        for scale, run in sliced:
            t += _best(run) * scale
        return t

    per_kind = {}
    for kind in ("gdn", "attn"):
        projs = [(n, k) for _, k, pr in cfg["groups"][kind] for _, n in pr]
        f = max(1.0, 2 * _M_SLICE * sum(n * k for n, k in projs) / macs_budget)
        t1, t2 = block(kind, _M_FEW, f), block(kind, M, f)
        slope, fixed = _fit(t1, t2, _M_FEW, M)
        parts[f"{kind}_block_per_token"] = slope
        parts[f"{kind}_block_fixed"] = fixed
        parts[f"{kind}_slice_factor"] = f
        per_kind[kind] = slope + fixed / step_tokens
    t0 = time.perf_counter()
    _gdn_core(64, cfg["gdn_heads"], cfg["gdn_qk_heads"], rs)
    parts["gdn_core_64tok"] = time.perf_counter() - t0
    fh = max(1.0, 2 * _M_SLICE * cfg["vocab"] * cfg["hidden"] / macs_budget)
    vs = max(64, int(round(cfg["vocab"] / fh / 64)) * 64)
    th = []
    for m in (_M_FEW, M):
        head_run = _head(m, vs, cfg["hidden"], rs)
        th.append(_best(head_run) * (cfg["vocab"] / vs))
        del head_run
    slope, fixed = _fit(th[0], th[1], _M_FEW, M)
    parts["head_per_token"], parts["head_fixed"] = slope, fixed
    parts["head_slice_factor"] = cfg["vocab"] / vs
    # the IQR decode of one 4096 x 4096 weight (r97_iqr_decode_host)
    rows = cols = 4096
    codes = rs.randint(0, 256, size=(rows, cols // 2)).astype(np.uint8)
    scale = np.abs(rs.normal(0, 0.02, size=(rows, cols // 128))).astype(np.float32)
    form = R.trunk_form(codes, scale, int(rs.randint(1 << 24)) | 1, int(rs.randint(1 << 31)), cols)
    t0 = time.perf_counter()
    R.iqr_decode(form, lib=ref_lib())
    parts["decode_4096x4096"] = time.perf_counter() - t0
    n_adam = 1 << 24
    w = rs.normal(size=n_adam).astype(np.float32)
    g = (rs.normal(size=n_adam) * 1e-3).astype(np.float32)
    t0 = time.perf_counter()
    ref_lib().ref_adamw(w.ctypes.data, n_adam, g.ctypes.data, 1, 1e-4, 0.9, 0.999, 1e-8, 0.0, 0.0, 0, 0, 0)
    parts["adamw_16M"] = time.perf_counter() - t0
    kinds = cfg["kinds"]
    n_gdn, n_attn = kinds.count("gdn"), kinds.count("attn")
    per_token = (n_gdn * per_kind["gdn"] + n_attn * per_kind["attn"]
                 + parts["head_per_token"] + parts["head_fixed"] / step_tokens
                 + n_gdn * parts["gdn_core_64tok"] / 64
                 + parts["decode_4096x4096"] * (cfg["base_weights"] / (4096.0 * 4096.0)) / step_tokens
                 + parts["adamw_16M"] * (cfg["adapter_params"] / float(n_adam)) / step_tokens)
    parts["seconds_per_token"] = per_token
    return parts


def threads() -> int:
    return int(os.environ.get("R97_THREADS", os.cpu_count() or 1))
