"""The LoRA training step of the synthetic hybrid model (configs 4 and 5), on the B200 kernels.

Architecture (BASELINE configs 4/5; the reference's target is the same family, Qwen3.5/3.8 hybrid):
a stack of blocks in a repeating 3 x GatedDeltaNet : 1 x gated-attention pattern, each block
``x + mixer(rmsnorm(x))`` then ``+ swiglu_mlp(rmsnorm(.))``; a tied, IQR-stored head; CE loss.
Every base projection is stored as an IQR weight (``iqr.IqrWeight``) and decoded to bf16 right before
its GEMM; every projection carries a LoRA adapter (rank r, scale alpha / r).

Projections that read the same input are one fused GEMM: base rows stacked, and the adapters' tails
stacked into one (A_all, block-diagonal B) pair, so a group's forward is two launches
(t = s x A_all^T, then Y = x W^T + t B_blk^T) and its input adjoint is two (dt = s dY B_blk, then
dX = dY W + dt A_all) plus the adapter-gradient GEMMs (dA_all = dt^T x, dB_i = dY_i^T t_i) -- the
reference's gemm_nt + lora_shrink + lora_expand rows (src/adjoint/host/linear.cpp, lora.cpp) per group.

The backward is explicit: every layer's forward saves what its adjoint reads (HBM holds a step's
activations: about 60 GB at config 5), and the reverse walk calls the kernels' adjoints in the
reverse op order -- the fixed per-layer schedule the reference's backward_block walks over its tape.
The attention core (softmax(q k^T) v, causal, GQA) runs on this package's tcgen05 kernels: the forward
(csrc/attn_fwd.cu) saves its output and per-row log-sum-exp for the backward (csrc/attn.cu).
"""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import iqr as IQ
from . import ops
from .gdn import GdnPlan


@dataclass
class HybridConfig:
    hidden: int = 4096
    layers: int = 32
    gdn_per_attn: int = 3
    gdn_heads: int = 32        # value heads
    gdn_qk_heads: int = 16
    head_k: int = 128
    attn_heads: int = 16
    attn_kv_heads: int = 4
    attn_head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 1e7
    ffn: int = 12288
    vocab: int = 151936
    eps: float = 1e-6
    rank: int = 64
    alpha: float = 128.0
    seq: int = 4096
    micro_batch: int = 2
    lr: float = 1e-4
    seed: int = 1234
    lora_mlp: bool = True      # adapters on the MLP projections too (config 4 names only the mixers')

    @property
    def kinds(self):
        p = self.gdn_per_attn + 1
        return ["attn" if (i % p) == p - 1 else "gdn" for i in range(self.layers)]

    @property
    def lora_scale(self):
        return self.alpha / self.rank

    @property
    def tokens(self):
        return self.seq * self.micro_batch


CONFIG5 = HybridConfig()
# config 4 as BASELINE.json states it: attention head dim 128 (rotary on the first 64 dims); GDN head counts are
# not stated there: 8 value heads and 4 key heads of 128
# and LoRA on q/k/v/o and the GDN in / out projections only
CONFIG4 = HybridConfig(hidden=1024, layers=24, gdn_heads=8, gdn_qk_heads=4, attn_heads=8, attn_kv_heads=2,
                       attn_head_dim=128, ffn=3584, rank=32, alpha=64.0, micro_batch=4, lora_mlp=False)


def groups_of(cfg: HybridConfig, kind: str):
    """The fused projection groups of one block: (group name, input width, [(projection, out width)])."""
    d, H, Hg, K = cfg.hidden, cfg.gdn_heads, cfg.gdn_qk_heads, cfg.head_k
    if kind == "gdn":
        mixer = [("in", d, [("in_proj_qkvz", 2 * Hg * K + 2 * H * K), ("in_proj_ba", 2 * H)]),
                 ("out", H * K, [("out_proj", d)])]
    else:
        Dh = cfg.attn_head_dim
        mixer = [("qkv", d, [("q_proj", 2 * cfg.attn_heads * Dh), ("k_proj", cfg.attn_kv_heads * Dh),
                             ("v_proj", cfg.attn_kv_heads * Dh)]),
                 ("o", cfg.attn_heads * Dh, [("o_proj", d)])]
    mlp = [("gu", d, [("gate_proj", cfg.ffn), ("up_proj", cfg.ffn)]), ("down", cfg.ffn, [("down_proj", d)])]
    return mixer + mlp


def has_lora(cfg: HybridConfig, group: str) -> bool:
    """Whether the projection group carries adapters: every group, or the mixers' only (cfg.lora_mlp)."""
    return cfg.lora_mlp or group not in ("gu", "down")


def module_path(layer: int, kind: str, proj: str) -> str:
    """The module's path as the reference's container names it (`model.layers.3.self_attn.q_proj`; the
    GatedDeltaNet mixer's projections under `linear_attn`, the MLP's under `mlp`), the prefix of its
    adapter parameters `<module>.lora_A` / `<module>.lora_B` (src/delta_lora.cpp:6-13, 130-136)."""
    if proj in ("gate_proj", "up_proj", "down_proj"):
        family = "mlp"
    else:
        family = "linear_attn" if kind == "gdn" else "self_attn"
    return f"model.layers.{layer}.{family}.{proj}"


# ============================================================================================ weights

@dataclass
class Group:
    name: str
    k: int                     # input width
    projs: list                # [(name, out width)]
    iqr: list = field(default_factory=list)  # IqrWeight per projection
    lora: bool = True          # carries adapters
    # adapter views into the flat buffers (set by Adapter)
    a_off: int = 0
    b_offs: list = field(default_factory=list)

    @property
    def n(self):
        return sum(o for _, o in self.projs)

    @property
    def r_all(self):
        return len(self.projs)


class HybridModel:
    """The frozen base on one device: IQR projections, norms, GDN parameters, tied IQR head."""

    def __init__(self, cfg: HybridConfig, device):
        self.cfg, self.device = cfg, device
        gen = torch.Generator(device=device)
        gen.manual_seed(cfg.seed)
        seed = cfg.seed * 7919
        self.blocks = []
        for li, kind in enumerate(cfg.kinds):
            blk = dict(kind=kind, groups=[])
            for gname, k, projs in groups_of(cfg, kind):
                g = Group(gname, k, projs, lora=has_lora(cfg, gname))
                for pname, n in projs:
                    seed += 1
                    # scales ~ |N(0, s)| with s chosen so the dequantised weight has std ~ 1/sqrt(fan_in)
                    # (codes of the mad codebook have std ~ 37)
                    g.iqr.append(IQ.synth_weight(n, k, seed, device=device, scale_std=1.0 / (37.0 * math.sqrt(k))))
                blk["groups"].append(g)
            d = cfg.hidden
            blk["w_in"] = (1.0 + 0.1 * torch.randn(d, generator=gen, device=device)).float()
            blk["w_post"] = (1.0 + 0.1 * torch.randn(d, generator=gen, device=device)).float()
            if kind == "gdn":
                H, Hg, K = cfg.gdn_heads, cfg.gdn_qk_heads, cfg.head_k
                conv_dim = (2 * Hg + H) * K
                blk["conv_w"] = (0.5 * torch.randn(conv_dim, 4, generator=gen, device=device)).float().contiguous()
                blk["a_log"] = torch.log(torch.empty(H, device=device).uniform_(1.0, 16.0, generator=gen)).float()
                blk["dt_bias"] = (0.1 * torch.randn(H, generator=gen, device=device)).float()
                blk["gnorm_w"] = (1.0 + 0.1 * torch.randn(K, generator=gen, device=device)).float()
            else:
                Dh = cfg.attn_head_dim
                blk["q_norm"] = (1.0 + 0.1 * torch.randn(Dh, generator=gen, device=device)).float()
                blk["k_norm"] = (1.0 + 0.1 * torch.randn(Dh, generator=gen, device=device)).float()
            self.blocks.append(blk)
        self.w_final = (1.0 + 0.1 * torch.randn(cfg.hidden, generator=gen, device=device)).float()
        self.head = IQ.synth_weight(cfg.vocab, cfg.hidden, seed + 1, device=device,
                                    scale_std=1.0 / (37.0 * math.sqrt(cfg.hidden)))
        half = cfg.rotary_dim // 2
        inv = 1.0 / (cfg.rope_theta ** (np.arange(half, dtype=np.float64) * 2.0 / cfg.rotary_dim))
        ang = np.arange(cfg.seq, dtype=np.float64)[:, None] * inv[None, :]
        self.rope_cos = torch.from_numpy(np.cos(ang).astype(np.float32)).to(device)
        self.rope_sin = torch.from_numpy(np.sin(ang).astype(np.float32)).to(device)

    def base_bytes(self) -> int:
        n = self.head.nbytes
        for blk in self.blocks:
            for g in blk["groups"]:
                n += sum(w.nbytes for w in g.iqr)
        return n


class Adapter:
    """The LoRA adapter of every projection in one flat f32 buffer (master weights), with its gradient,
    the AdamW moments, and the bf16 mirrors the GEMMs read: A_all [r_all * rank, k] per group (compact)
    and B as a block-diagonal [n, r_all * rank] per group. Leaf names follow the reference's
    `<module>.lora_A` / `<module>.lora_B` convention (src/delta_lora.cpp)."""

    def __init__(self, model: HybridModel, device, b_std: float = 1e-3):
        cfg, r = model.cfg, model.cfg.rank
        self.cfg, self.device = cfg, device
        self.names, self.shapes, self.offsets = [], [], []
        off = 0
        self.layer_ranges = []
        for li, blk in enumerate(model.blocks):
            start = off
            for g in blk["groups"]:
                if not g.lora:
                    continue
                g.a_off = off
                for pname, _ in g.projs:
                    self.names.append(f"{module_path(li, blk['kind'], pname)}.lora_A")
                    self.shapes.append((r, g.k))
                    self.offsets.append(off)
                    off += r * g.k
                g.b_offs = []
                for pname, n in g.projs:
                    self.names.append(f"{module_path(li, blk['kind'], pname)}.lora_B")
                    self.shapes.append((n, r))
                    self.offsets.append(off)
                    g.b_offs.append(off)
                    off += n * r
            self.layer_ranges.append((start, off))
        self.numel = off
        gen = torch.Generator(device=device)
        gen.manual_seed(cfg.seed + 99)
        self.w = torch.empty(off, dtype=torch.float32, device=device)
        for (name, shape, o) in zip(self.names, self.shapes, self.offsets):
            n = shape[0] * shape[1]
            if name.endswith("lora_A"):  # PEFT init: U(-1/sqrt(fan_in), 1/sqrt(fan_in)) (src/delta_lora.cpp:115-136)
                b = 1.0 / math.sqrt(shape[1])
                self.w[o:o + n].uniform_(-b, b, generator=gen)
            else:
                self.w[o:o + n].normal_(0.0, b_std, generator=gen)
        self.g = torch.zeros_like(self.w)
        self.m = torch.zeros_like(self.w)
        self.v = torch.zeros_like(self.w)
        self.step = 0
        self.sched = torch.zeros(3, dtype=torch.float32, device=device)  # lr, bc1, bc2 of the current step
        # bf16 mirrors
        self.a_bf, self.b_blk = {}, {}
        for li, blk in enumerate(model.blocks):
            for g in blk["groups"]:
                if not g.lora:
                    continue
                self.a_bf[(li, g.name)] = torch.empty((g.r_all * r, g.k), dtype=torch.bfloat16, device=device)
                self.b_blk[(li, g.name)] = torch.zeros((g.n, g.r_all * r), dtype=torch.bfloat16, device=device)
        self.model = model
        self._casts = None
        self.refresh_mirrors()

    def a_view(self, buf, g):
        r = self.cfg.rank
        return buf[g.a_off:g.a_off + g.r_all * r * g.k].view(g.r_all * r, g.k)

    def b_view(self, buf, g, i):
        r, n = self.cfg.rank, g.projs[i][1]
        return buf[g.b_offs[i]:g.b_offs[i] + n * r].view(n, r)

    def _mirror_pairs(self):
        r = self.cfg.rank
        pairs = []
        for li, blk in enumerate(self.model.blocks):
            for g in blk["groups"]:
                if not g.lora:
                    continue
                pairs.append((self.a_view(self.w, g), self.a_bf[(li, g.name)]))
                row = 0
                for i, (_, n) in enumerate(g.projs):
                    pairs.append((self.b_view(self.w, g, i), self.b_blk[(li, g.name)][row:row + n, i * r:(i + 1) * r]))
                    row += n
        return pairs

    def refresh_mirrors(self, stream=None):
        """The bf16 mirrors from the f32 master weights: every A_all and B_i block in one launch."""
        if self._casts is None:
            pairs = self._mirror_pairs()
            try:
                self._casts = ops.CastTable(pairs, self.device)
            except ops.R97bError:  # a rank that is not a multiple of 8: one cast per block
                self._casts = pairs
        if isinstance(self._casts, ops.CastTable):
            self._casts.run(stream)
        else:
            for src, dst in self._casts:
                ops.cast_f32_bf16(src, dst, stream=stream)

    def advance_schedule(self, lr=None, beta1=0.9, beta2=0.999, stream=None):
        """Counts one more step and writes its lr and bias corrections bc1 = 1 - beta1^t, bc2 = 1 - beta2^t
        (f32 powf, as the reference's optimiser forms them) into the device schedule `sched` the update
        reads; stream-ordered before whatever is queued after it."""
        import ctypes
        self.step += 1
        t = self.step
        libm = ctypes.CDLL("libm.so.6")
        libm.powf.restype = ctypes.c_float
        libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
        bc1 = float(np.float32(1.0) - np.float32(libm.powf(beta1, float(t))))
        bc2 = float(np.float32(1.0) - np.float32(libm.powf(beta2, float(t))))
        vals = torch.tensor([self.cfg.lr if lr is None else lr, bc1, bc2], dtype=torch.float32)
        with torch.cuda.stream(stream or torch.cuda.current_stream()):
            self.sched.copy_(vals)  # pageable source: staged before the call returns

    def update(self, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, stream=None):
        """The AdamW update at the schedule's current step, then the gradient is cleared and the bf16
        mirrors refreshed; reads its step-dependent scalars from `sched`, so it can live in a CUDA graph."""
        ops.adamw_step_dev(self.w, self.m, self.v, self.g, self.sched, beta1=beta1, beta2=beta2, eps=eps,
                           weight_decay=weight_decay, zero_grad=True, stream=stream)
        self.refresh_mirrors(stream=stream)

    def adamw(self, lr=None, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, stream=None):
        """One AdamW update of the whole adapter (bit-identical to the reference Optimiser's f32 update),
        then the gradient is cleared and the bf16 mirrors refreshed."""
        self.advance_schedule(lr, beta1, beta2, stream=stream)
        self.update(beta1, beta2, eps, weight_decay, stream=stream)


# ============================================================================================ the step

class Workspace:
    """Decoded-weight scratch (one block's projections at a time) and the head's logits chunk."""

    def __init__(self, model: HybridModel, head_chunk: int):
        cfg = model.cfg
        most = 0
        for blk in model.blocks:
            for g in blk["groups"]:
                most = max(most, g.n * g.k)
        self.w_scratch = torch.empty(most, dtype=torch.bfloat16, device=model.device)
        self.head_w = torch.empty((cfg.vocab, cfg.hidden), dtype=torch.bfloat16, device=model.device)
        self.logits = torch.empty((head_chunk, cfg.vocab), dtype=torch.bfloat16, device=model.device)
        self.head_chunk = head_chunk


def decode_group(g: Group, out: torch.Tensor, stream=None) -> torch.Tensor:
    """The group's base rows, stacked, decoded to bf16 into `out` ([n, k])."""
    W = out[:g.n * g.k].view(g.n, g.k)
    row = 0
    for w in g.iqr:
        IQ.dequant_bf16(w, out=W[row:row + w.rows], stream=stream)
        row += w.rows
    return W


class TrainStep:
    """Forward, loss and backward of one micro-batch through the whole model, then (optionally) AdamW.

    ``run(ids)`` takes int32 token ids [micro_batch, seq] on the device, returns the mean CE loss (a device
    scalar) and leaves the adapter gradient in ``adapter.g``. ``grad_hook(layer)`` is called as each
    layer's adapter gradient becomes final in the reverse walk (the data-parallel all-reduce hook)."""

    def __init__(self, model: HybridModel, adapter: Adapter, head_chunk: int = 2048, keep_decoded: bool = True):
        self.model, self.adapter, self.cfg = model, adapter, model.cfg
        self.ws = Workspace(model, head_chunk)
        # keep_decoded: each projection group is decoded once a step, in the forward, into a buffer of its
        # own that the same layer's backward reads again (13.8 GB bf16 at config 5, against a second
        # decode of every weight); False decodes into one shared scratch in both passes.
        self.keep_decoded = keep_decoded
        self.w_keep = {}
        self.w_pending = {}  # (layer, group) -> the side-stream event its prefetched decode completes
        cfg = self.cfg
        self.T = cfg.tokens
        cu = np.arange(0, self.T + 1, cfg.seq, dtype=np.int32)
        self.cu_dev = torch.from_numpy(cu).to(model.device)
        self.plan = GdnPlan(cu, cfg.gdn_heads, cfg.gdn_qk_heads, model.device)
        self.grad_hook = None
        self.launches = 0
        self.split_ws = ops.SplitWorkspace(model.device)
        # the side stream the GDN layers' out-projection adapter gradients run on (None: all on one stream)
        self.side = torch.cuda.Stream(device=model.device) if model.device.type == "cuda" else None
        self.attn_ws = None  # the attention backward's P / dS tiles, allocated at the first attention layer

    # ------------------------------------------------------------------ decoded base weights
    def _w_fwd(self, li, g: Group) -> torch.Tensor:
        """The group's base weight for the forward: decoded now, or by `_prefetch` on the side stream."""
        if not self.keep_decoded:
            return decode_group(g, self.ws.w_scratch)
        ev = self.w_pending.pop((li, g.name), None)
        if ev is not None:
            torch.cuda.current_stream().wait_event(ev)
            return self.w_keep[(li, g.name)][:g.n * g.k].view(g.n, g.k)
        buf = self.w_keep.get((li, g.name))
        if buf is None:
            buf = torch.empty(g.n * g.k, dtype=torch.bfloat16, device=self.model.device)
            self.w_keep[(li, g.name)] = buf
        return decode_group(g, buf)

    def _prefetch(self, li, groups):
        """Decodes `groups` of layer li on the side stream (ordered after the work queued so far), for a
        `_w_fwd` of the same layer to wait on instead of decoding: during a GDN state pass, which holds 128 of
        the SMs, the decode runs on the rest."""
        if not self.keep_decoded or self.side is None:
            return
        ev0 = torch.cuda.Event()
        ev0.record()
        self.side.wait_event(ev0)
        for g in groups:
            buf = self.w_keep.get((li, g.name))
            if buf is None:
                buf = torch.empty(g.n * g.k, dtype=torch.bfloat16, device=self.model.device)
                self.w_keep[(li, g.name)] = buf
            with torch.cuda.stream(self.side):
                decode_group(g, buf)
                ev = torch.cuda.Event()
                ev.record()
            self.w_pending[(li, g.name)] = ev

    def _w_bwd(self, li, g: Group) -> torch.Tensor:
        """The group's base weight for the backward: this step's forward decode, or decoded again."""
        if not self.keep_decoded:
            return decode_group(g, self.ws.w_scratch)
        return self.w_keep[(li, g.name)][:g.n * g.k].view(g.n, g.k)

    # ------------------------------------------------------------------ fused LoRA linear
    def _lin_fwd(self, li, g: Group, x: torch.Tensor, W: torch.Tensor, out: torch.Tensor, addend=None,
                 swiglu_out=None):
        """t = s x A_all^T ; out = x W^T + t B_blk^T (+ addend). Returns t (saved for dB). With `swiglu_out`
        (the gate/up group) the GEMM's epilogue also writes silu(g) u there."""
        cfg, ad = self.cfg, self.adapter
        if not g.lora:
            if swiglu_out is not None:
                ops.gemm(x, W, out, mode=ops.EPI_SWIGLU, out2=swiglu_out)
            else:
                ops.gemm(x, W, out, addend=addend, beta=1.0)
            return None
        t = torch.empty((x.shape[0], g.r_all * cfg.rank), dtype=torch.bfloat16, device=x.device)
        self._skinny(x, ad.a_bf[(li, g.name)], t, g.k, False)
        # the tail's B is block-diagonal: each output column has `rank` non-zero tail entries
        work = 2.0 * x.shape[0] * g.n * (g.k + cfg.rank)
        if swiglu_out is not None:
            ops.gemm(x, W, out, a2=t, b2=ad.b_blk[(li, g.name)], mode=ops.EPI_SWIGLU, out2=swiglu_out, flops=work)
        else:
            ops.gemm(x, W, out, a2=t, b2=ad.b_blk[(li, g.name)], addend=addend, beta=1.0, flops=work)
        return t

    def _skinny(self, a, b, out, K, b_mn):
        """out = s a b^T for the adapter's narrow products (t = s x A_all^T, dt = s dY B_blk): tiled and
        split so that ~all SMs share the read of `a` (ops.skinny_tiling)."""
        M, N = out.shape
        bn, splits = ops.skinny_tiling(M, N, K)
        ops.gemm(a, b, out, b_mn=b_mn, alpha=self.cfg.lora_scale, N=N, bn=bn, splits=splits,
                 mode=ops.EPI_SPLIT_BF16 if splits > 1 else ops.EPI_STORE_BF16, ws=self.split_ws.buf)

    def _lin_bwd(self, li, g: Group, x: torch.Tensor, t: torch.Tensor, W: torch.Tensor, dy: torch.Tensor,
                 dx_out: torch.Tensor, swiglu_gu=None, side=None):
        """dt = s dY B_blk ; dX = dY W + dt A_all ; dA_all += dt^T x ; dB_i += dY_i^T t_i. With `swiglu_gu`
        (the down group, whose input is silu(g) u) dx_out receives SwiGLU's adjoint [dg | du] instead. With
        `side` (a stream), the two adapter-gradient products are issued there, ordered after dt, and the
        caller joins it before the layer's gradient is read."""
        cfg, ad = self.cfg, self.adapter
        r = cfg.rank
        if not g.lora:
            if swiglu_gu is not None:
                ops.gemm(dy, W, dx_out, b_mn=True, N=g.k, mode=ops.EPI_SWIGLU_BWD, addend=swiglu_gu)
            else:
                ops.gemm(dy, W, dx_out, b_mn=True, N=g.k)
            return
        dt = torch.empty((dy.shape[0], g.r_all * r), dtype=torch.bfloat16, device=dy.device)
        self._skinny(dy, ad.b_blk[(li, g.name)], dt, g.n, True)
        if swiglu_gu is not None:
            ops.gemm(dy, W, dx_out, b_mn=True, a2=dt, b2=ad.a_bf[(li, g.name)], N=g.k, mode=ops.EPI_SWIGLU_BWD,
                     addend=swiglu_gu)
        else:
            ops.gemm(dy, W, dx_out, b_mn=True, a2=dt, b2=ad.a_bf[(li, g.name)], N=g.k)
        if side is not None:
            ev = torch.cuda.Event()
            ev.record()
            side.wait_event(ev)
            for u in (x, t, dy, dt):
                u.record_stream(side)
        with torch.cuda.stream(side) if side is not None else contextlib.nullcontext():
            bn, splits = ops.grad_tiling(g.k, g.r_all * r, dy.shape[0])
            ops.gemm(x, dt, ad.a_view(ad.g, g), a_mn=True, b_mn=True, mode=ops.EPI_ATOMIC_F32T, splits=splits,
                     bn=bn, M=g.k, N=g.r_all * r)
            col = 0
            for i, (_, n) in enumerate(g.projs):
                bn, splits = ops.grad_tiling(n, r, dy.shape[0])
                ops.gemm(dy[:, col:col + n], t[:, i * r:(i + 1) * r], ad.b_view(ad.g, g, i), a_mn=True,
                         b_mn=True, mode=ops.EPI_ATOMIC_F32, splits=splits, bn=bn, M=n, N=r)
                col += n

    # ------------------------------------------------------------------ blocks
    def _gdn_fwd(self, li, blk, x, sv):
        cfg, T = self.cfg, self.T
        H, Hg, K = cfg.gdn_heads, cfg.gdn_qk_heads, cfg.head_k
        g_in, g_out = blk["groups"][0], blk["groups"][1]
        n1 = ops.rmsnorm_fwd(x, blk["w_in"], eps=cfg.eps)
        W = self._w_fwd(li, g_in)
        y_in = torch.empty((T, g_in.n), dtype=torch.bfloat16, device=x.device)
        t_in = self._lin_fwd(li, g_in, n1, W, y_in)
        qk = Hg * K
        q = torch.empty((T, Hg, K), dtype=torch.bfloat16, device=x.device)
        k = torch.empty_like(q)
        v = torch.empty((T, H, K), dtype=torch.bfloat16, device=x.device)
        ops.conv_prep_fwd(y_in, blk["conv_w"], self.cu_dev, self.plan.n_seq, Hg, H, q, k, v)
        gg = torch.empty((T, H), dtype=torch.float32, device=x.device)
        beta = torch.empty_like(gg)
        ba = y_in[:, 2 * qk + 2 * H * K:]
        ops.gates_fwd(ba, blk["a_log"], blk["dt_bias"], self.plan, gg, beta)
        # the block's remaining weights, and the next block's input projection, decode on the side stream
        # while the GDN state pass holds 128 SMs
        self._prefetch(li, [g_out, blk["groups"][2], blk["groups"][3]])
        if li + 1 < len(self.model.blocks):
            self._prefetch(li + 1, [self.model.blocks[li + 1]["groups"][0]])
        o, _, gsv = self.plan.forward(q, k, v, gg, beta)
        z = y_in[:, 2 * qk + H * K:2 * qk + 2 * H * K]  # read in place (strided), no copy
        on = ops.gated_rmsnorm_fwd(o.view(T * H, K), z, blk["gnorm_w"], eps=cfg.eps).view(T, H * K)
        W = self._w_fwd(li, g_out)
        h1 = torch.empty_like(x)
        t_out = self._lin_fwd(li, g_out, on, W, h1, addend=x)
        sv.update(n1=n1, y_in=y_in, t_in=t_in, gsv=gsv, o=o, on=on, t_out=t_out)
        return h1

    def _gdn_bwd(self, li, blk, x, sv, dh1):
        cfg, T = self.cfg, self.T
        H, Hg, K = cfg.gdn_heads, cfg.gdn_qk_heads, cfg.head_k
        g_in, g_out = blk["groups"][0], blk["groups"][1]
        qk = Hg * K
        W = self._w_bwd(li, g_out)
        don = torch.empty((T, H * K), dtype=torch.bfloat16, device=x.device)
        # the out-projection's adapter gradients need nothing the GDN adjoint computes: on the side stream they
        # run beside it (its state passes hold 128 of the SMs), joined before the layer's gradient is read
        self._lin_bwd(li, g_out, sv["on"], sv["t_out"], W, dh1, don, side=self.side)
        y_in = sv["y_in"]
        zsl = slice(2 * qk + H * K, 2 * qk + 2 * H * K)
        d_yin = torch.empty_like(y_in)
        do = torch.empty((T, H, K), dtype=torch.bfloat16, device=x.device)
        # dz lands straight in its columns of the projection's cotangent
        ops.gated_rmsnorm_bwd(sv["o"].view(T * H, K), y_in[:, zsl], blk["gnorm_w"], don.view(T * H, K),
                              eps=cfg.eps, dx=do.view(T * H, K), dz=d_yin[:, zsl])
        # dq, dk stay per value head: the conv adjoint sums each key head's value heads as it reads them
        gr = self.plan.backward(sv["gsv"], do, sum_heads=False)
        ops.conv_prep_bwd(y_in, blk["conv_w"], self.cu_dev, self.plan.n_seq, Hg, H, gr["dq"], gr["dk"], gr["dv"],
                          d_yin)
        ba = y_in[:, 2 * qk + 2 * H * K:]
        ops.gates_bwd(ba, blk["a_log"], blk["dt_bias"], self.plan, gr["dg"], gr["dbeta"],
                      d_yin[:, 2 * qk + 2 * H * K:])
        W = self._w_bwd(li, g_in)
        dn1 = torch.empty_like(x)
        self._lin_bwd(li, g_in, sv["n1"], sv["t_in"], W, d_yin, dn1)
        if self.side is not None:
            torch.cuda.current_stream().wait_stream(self.side)
        return ops.rmsnorm_bwd(x, blk["w_in"], dn1, addend=dh1, eps=cfg.eps)

    def _attn_fwd(self, li, blk, x, sv):
        cfg, T, S = self.cfg, self.T, self.cfg.seq
        Hq, Hkv, Dh, B = cfg.attn_heads, cfg.attn_kv_heads, cfg.attn_head_dim, cfg.micro_batch
        g_qkv, g_o = blk["groups"][0], blk["groups"][1]
        n1 = ops.rmsnorm_fwd(x, blk["w_in"], eps=cfg.eps)
        W = self._w_fwd(li, g_qkv)
        y = torch.empty((T, g_qkv.n), dtype=torch.bfloat16, device=x.device)
        t_qkv = self._lin_fwd(li, g_qkv, n1, W, y)
        qn = 2 * Hq * Dh
        qr = torch.empty((B, Hq, S, Dh), dtype=torch.bfloat16, device=x.device)
        kr = torch.empty((B, Hkv, S, Dh), dtype=torch.bfloat16, device=x.device)
        vt = torch.empty((B, Hkv, S, Dh), dtype=torch.bfloat16, device=x.device)
        ops.qk_norm_rope_fwd(y, 2 * Dh, Hq, Dh, blk["q_norm"], self.model.rope_cos, self.model.rope_sin,
                             cfg.rotary_dim, S, cfg.eps, qr)
        ops.qk_norm_rope_fwd(y[:, qn:], Dh, Hkv, Dh, blk["k_norm"], self.model.rope_cos, self.model.rope_sin,
                             cfg.rotary_dim, S, cfg.eps, kr)
        ops.to_bhsd(y[:, qn + Hkv * Dh:], Dh, Hkv, Dh, S, vt)
        # the attention core on this package's tcgen05 kernel (csrc/attn_fwd.cu); its output and per-row
        # log-sum-exp feed the matching backward below
        attn, lse = ops.attn_fwd(qr, kr, vt, 1.0 / math.sqrt(Dh))
        fa = (attn, lse)
        ga = torch.empty((T, Hq * Dh), dtype=torch.bfloat16, device=x.device)
        ops.gate_mul_fwd(attn, y[:, Dh:], 2 * Dh, Hq, Dh, S, ga)
        W = self._w_fwd(li, g_o)
        h1 = torch.empty_like(x)
        t_o = self._lin_fwd(li, g_o, ga, W, h1, addend=x)
        sv.update(n1=n1, y=y, t_qkv=t_qkv, qkv=(qr, kr, vt), fa=fa, attn=attn, ga=ga, t_o=t_o)
        return h1

    def _attn_bwd(self, li, blk, x, sv, dh1):
        cfg, T, S = self.cfg, self.T, self.cfg.seq
        Hq, Hkv, Dh, B = cfg.attn_heads, cfg.attn_kv_heads, cfg.attn_head_dim, cfg.micro_batch
        g_qkv, g_o = blk["groups"][0], blk["groups"][1]
        qn = 2 * Hq * Dh
        W = self._w_bwd(li, g_o)
        dga = torch.empty((T, Hq * Dh), dtype=torch.bfloat16, device=x.device)
        self._lin_bwd(li, g_o, sv["ga"], sv["t_o"], W, dh1, dga)
        y = sv["y"]
        dy = torch.empty_like(y)
        dattn = torch.empty((B, Hq, S, Dh), dtype=torch.bfloat16, device=x.device)
        ops.gate_mul_bwd(sv["attn"], y[:, Dh:], 2 * Dh, Hq, Dh, S, dga, dattn, dy[:, Dh:])
        qg, kg, vg = sv["qkv"]
        fa = sv["fa"]
        # the attention core's adjoint on this package's tensor-core passes (csrc/attn.cu), from the
        # forward's output and log-sum-exp
        if self.attn_ws is None:
            self.attn_ws = ops.attn_bwd_workspace(B, Hq, S, x.device)
        dq, dk, dv = ops.attn_bwd(qg, kg, vg, fa[0], dattn, fa[1], 1.0 / math.sqrt(Dh), self.attn_ws)
        ops.qk_norm_rope_bwd(y, 2 * Dh, Hq, Dh, blk["q_norm"], self.model.rope_cos, self.model.rope_sin,
                             cfg.rotary_dim, S, cfg.eps, dq, dy)
        ops.qk_norm_rope_bwd(y[:, qn:], Dh, Hkv, Dh, blk["k_norm"], self.model.rope_cos, self.model.rope_sin,
                             cfg.rotary_dim, S, cfg.eps, dk, dy[:, qn:])
        ops.to_bhsd(dy[:, qn + Hkv * Dh:], Dh, Hkv, Dh, S, dv, reverse=True)
        W = self._w_bwd(li, g_qkv)
        dn1 = torch.empty_like(x)
        self._lin_bwd(li, g_qkv, sv["n1"], sv["t_qkv"], W, dy, dn1)
        return ops.rmsnorm_bwd(x, blk["w_in"], dn1, addend=dh1, eps=cfg.eps)

    def _mlp_fwd(self, li, blk, h1, sv):
        cfg, T = self.cfg, self.T
        g_gu, g_d = blk["groups"][2], blk["groups"][3]
        n2 = ops.rmsnorm_fwd(h1, blk["w_post"], eps=cfg.eps)
        W = self._w_fwd(li, g_gu)
        y_gu = torch.empty((T, 2 * cfg.ffn), dtype=torch.bfloat16, device=h1.device)
        a = torch.empty((T, cfg.ffn), dtype=torch.bfloat16, device=h1.device)
        t_gu = self._lin_fwd(li, g_gu, n2, W, y_gu, swiglu_out=a)  # SwiGLU in the GEMM's epilogue
        W = self._w_fwd(li, g_d)
        xn = torch.empty_like(h1)
        t_d = self._lin_fwd(li, g_d, a, W, xn, addend=h1)
        sv.update(n2=n2, y_gu=y_gu, t_gu=t_gu, a=a, t_d=t_d)
        return xn

    def _mlp_bwd(self, li, blk, h1, sv, dxn):
        cfg, T = self.cfg, self.T
        g_gu, g_d = blk["groups"][2], blk["groups"][3]
        W = self._w_bwd(li, g_d)
        dgu = torch.empty_like(sv["y_gu"])
        self._lin_bwd(li, g_d, sv["a"], sv["t_d"], W, dxn, dgu, swiglu_gu=sv["y_gu"])  # SwiGLU's adjoint fused
        W = self._w_bwd(li, g_gu)
        dn2 = torch.empty_like(h1)
        self._lin_bwd(li, g_gu, sv["n2"], sv["t_gu"], W, dgu, dn2)
        return ops.rmsnorm_bwd(h1, blk["w_post"], dn2, addend=dxn, eps=cfg.eps)

    # ------------------------------------------------------------------ the whole step
    def run(self, ids: torch.Tensor, targets: torch.Tensor | None = None, n_scored: int | None = None):
        """ids: int32 [micro_batch, seq] (device). targets: int32 [micro_batch * seq] with -1 where a row
        is not scored; default: next-token targets, the last position of each sequence unscored.
        n_scored: how many rows targets scores, when the caller knows it (default targets: from the shape;
        explicit targets without it: counted on the device, which synchronises the host once).
        Returns the mean CE over scored rows (device f32 scalar)."""
        cfg, model, T = self.cfg, self.model, self.T
        ids = ids.reshape(-1).to(torch.int32).contiguous()
        if targets is None:
            n_scored = int(cfg.micro_batch * (cfg.seq - 1))
            targets = torch.empty_like(ids)
            tv = targets.view(cfg.micro_batch, cfg.seq)
            tv[:, :-1] = ids.view(cfg.micro_batch, cfg.seq)[:, 1:]
            tv[:, -1] = -1
        # the tied head, decoded once for the embedding and both head products
        IQ.dequant_bf16(model.head, out=self.ws.head_w)
        x = torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device=model.device)
        ops.embed(self.ws.head_w, ids, x)
        saved = []
        for li, blk in enumerate(model.blocks):
            sv = dict(x=x)
            h1 = self._gdn_fwd(li, blk, x, sv) if blk["kind"] == "gdn" else self._attn_fwd(li, blk, x, sv)
            sv["h1"] = h1
            x = self._mlp_fwd(li, blk, h1, sv)
            saved.append(sv)
        # head: final norm, logits in chunks, CE in place, d(normed) = grad @ W_head
        nf = ops.rmsnorm_fwd(x, model.w_final, eps=cfg.eps)
        if n_scored is None:
            n_scored = int((targets >= 0).sum().item())
        scale = 1.0 / max(n_scored, 1)
        dnf = torch.empty_like(nf)
        loss_rows = torch.empty(T, dtype=torch.float32, device=model.device)
        hc = self.ws.head_chunk
        for r0 in range(0, T, hc):
            r1 = min(T, r0 + hc)
            lg = self.ws.logits[:r1 - r0]
            ops.gemm(nf[r0:r1], self.ws.head_w, lg)
            ops.ce_kld(lg, targets[r0:r1], grad=lg, grad_scale=scale, loss_ce=loss_rows[r0:r1])
            ops.gemm(lg, self.ws.head_w, dnf[r0:r1], b_mn=True, N=cfg.hidden)
        dx = ops.rmsnorm_bwd(x, model.w_final, dnf, eps=cfg.eps)
        for li in range(len(model.blocks) - 1, -1, -1):
            blk, sv = model.blocks[li], saved[li]
            dh1 = self._mlp_bwd(li, blk, sv["h1"], sv, dx)
            if blk["kind"] == "gdn":
                dx = self._gdn_bwd(li, blk, sv["x"], sv, dh1)
            else:
                dx = self._attn_bwd(li, blk, sv["x"], sv, dh1)
            saved[li] = None
            if self.grad_hook is not None:
                self.grad_hook(li)
        return loss_rows.sum() * scale


class GraphStep:
    """One whole training step captured as a CUDA graph and replayed: forward, loss, backward and (with
    `update`) the AdamW update, over static input and output buffers. The host's share of a step becomes
    a copy of the token ids, the schedule write and one graph launch, instead of ~2000 kernel launches.

    The step must have run eagerly at least once first (kernel attributes, tensor-map encoders and the
    decoded-weight buffers are set up on first use, outside any capture). With `buckets` (a data-parallel
    dp.GradBuckets over the adapter gradient, whose collectives have run eagerly once) the per-layer
    all-reduces are captured too, on their side stream as the reverse walk finishes each layer, and joined
    before the update; a graph that holds collectives must be released (``release``) before the process
    group is destroyed."""

    def __init__(self, step: "TrainStep", ids: torch.Tensor, update: bool = True, buckets=None):
        self.step, self.update = step, update
        dev = step.model.device
        self.ids = ids.reshape(-1).to(torch.int32).clone()
        hook, step.grad_hook = step.grad_hook, (buckets.ready if buckets is not None else None)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(self.graph):
                self.loss = step.run(self.ids)
                if buckets is not None:
                    buckets.join()
                if update:
                    step.adapter.update()
        finally:
            step.grad_hook = hook

    def release(self) -> None:
        """Frees the graph (and any collectives captured in it)."""
        if self.graph is not None:
            self.graph.reset()
            self.graph = None

    def replay(self, ids: torch.Tensor | None = None, lr=None) -> torch.Tensor:
        """Runs one step on `ids` (copied into the captured input; None reuses the last ids) and returns the
        captured loss tensor (valid until the next replay)."""
        if ids is not None:
            self.ids.copy_(ids.reshape(-1), non_blocking=True)
        if self.update:
            self.step.adapter.advance_schedule(lr)
        self.graph.replay()
        return self.loss


def flops_per_token(cfg: HybridConfig) -> float:
    """Algorithmic FLOPs of one trained token (forward + backward), counted from the shapes: the base
    products 2 x (fwd) + 2 x (dX) per weight element, the adapter's shrink/expand forward, their input
    adjoints and the two gradient products, the head forward and its dX, attention (causal, averaged over
    the sequence) and the GDN chunk products."""
    d, r = cfg.hidden, cfg.rank
    lin = lora = 0
    for kind in cfg.kinds:
        for gname, k, projs in groups_of(cfg, kind):
            for _, n in projs:
                lin += n * k
                if has_lora(cfg, gname):
                    lora += r * (n + k)
    head = cfg.vocab * d
    f = 4.0 * lin + 4.0 * head + 6.0 * lora * 2 / 2 * 1.0
    # attention core: fwd 4 S/2 Dh per head per token (QK^T and PV, causal half), bwd 2.5x fwd
    n_attn = cfg.kinds.count("attn")
    f += n_attn * cfg.attn_heads * 4.0 * (cfg.seq / 2) * cfg.attn_head_dim * 3.5
    # GDN: per chunk of 64 and value head, fwd ~ 6 L K V + 2 L^2 K + 2 L^2 V + L^3/3, bwd ~ 2 x fwd
    L, K = 64, cfg.head_k
    per_chunk = 6 * L * K * K + 2 * L * L * K + 2 * L * L * K + L ** 3 / 3
    f += cfg.kinds.count("gdn") * cfg.gdn_heads * per_chunk / L * 3.0
    return f
