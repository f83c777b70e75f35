"""Torch-facing wrappers over the C ABI of libr97b200.so.

Torch tensors supply device memory and the current CUDA stream; the arithmetic is the library's
sm_100a kernels. Every wrapper checks shapes, dtypes and contiguity, then calls the C entry point and
raises R97bError on a non-zero status. Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import (R97bAttnBwd, R97bAttnFwd, R97bCastSeg, R97bError, R97bGemm, R97bMat, R97bQLinearLora,
                   R97bQLinearLoraBwd, check, lib)

EPI_STORE_BF16, EPI_STORE_F32, EPI_ATOMIC_F32, EPI_ATOMIC_F32T, EPI_SPLIT_BF16 = 0, 1, 2, 3, 4
EPI_SWIGLU, EPI_SWIGLU_BWD = 5, 6


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _need(t: torch.Tensor, dtype, name: str):
    if not t.is_cuda:
        raise R97bError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise R97bError(f"{name} must be {dtype}, got {t.dtype}")


# ------------------------------------------------------------------------------------------ GEMM

def _mat(t: torch.Tensor, mn_major: bool, rows: int, k: int, name: str) -> R97bMat:
    """Operand of logical shape [rows, k]: K-major = stored [rows, k]; MN-major = stored [k, rows]."""
    _need(t, torch.bfloat16, name)
    if t.dim() != 2 or t.stride(1) != 1:
        raise R97bError(f"{name} must be a 2-D row-major view")
    want = (k, rows) if mn_major else (rows, k)
    if tuple(t.shape) != want:
        raise R97bError(f"{name} has shape {tuple(t.shape)}, expected {want}")
    return R97bMat(t.data_ptr(), t.stride(0), int(mn_major), 0)


def gemm(a1, b1, out, *, a_mn=False, b_mn=False, a2=None, b2=None, mode=EPI_STORE_BF16, alpha=1.0,
         addend=None, beta=1.0, splits=1, bn=0, M=None, N=None, ws=None, out2=None, stream=None, flops=None):
    """out (+)= alpha * (A1 B1^T + A2 B2^T) (+ beta * addend); see include/r97b.h (r97b_gemm).

    A1 is [M, K1] (K-major) or stored [K1, M] (a_mn); B1 is [N, K1] or stored [K1, N] (b_mn); the optional
    tail (a2, b2) has the same majorness with its own K2. EPI_SPLIT_BF16 with splits > 1 needs `ws`, a
    zero-initialised device buffer of at least r97b_gemm_workspace_bytes bytes (see SplitWorkspace).
    EPI_SWIGLU writes [g | u] to `out` and silu(g) u to `out2`; EPI_SWIGLU_BWD reads [g | u] as `addend`
    and writes [dg | du] to `out` (N = the SwiGLU width). `flops` is the algorithmic work the profile
    (GEMM_PROFILE) counts for this call when it is less than 2 M N (K1 + K2) (a block-diagonal tail)."""
    if M is None:
        M = a1.shape[1] if a_mn else a1.shape[0]
    if N is None:
        N = b1.shape[1] if b_mn else b1.shape[0]
    K1 = a1.shape[0] if a_mn else a1.shape[1]
    g = R97bGemm()
    g.M, g.N, g.K1 = M, N, K1
    g.a1 = _mat(a1, a_mn, M, K1, "a1")
    g.b1 = _mat(b1, b_mn, N, K1, "b1")
    if a2 is not None:
        K2 = a2.shape[0] if a_mn else a2.shape[1]
        g.K2 = K2
        g.a2 = _mat(a2, a_mn, M, K2, "a2")
        g.b2 = _mat(b2, b_mn, N, K2, "b2")
    g.mode, g.splits, g.alpha, g.beta, g.bn = mode, splits, alpha, beta, bn
    if mode == EPI_SPLIT_BF16:
        need = int(lib().r97b_gemm_workspace_bytes(ctypes.byref(g)))
        if need < 0:
            raise R97bError("r97b_gemm: bad split GEMM description")
        if need > 0:
            if ws is None or ws.numel() * ws.element_size() < need or ws.device != out.device:
                raise R97bError(f"r97b_gemm: the split GEMM needs a {need}-byte workspace on {out.device}")
            g.ws, g.ws_bytes = ws.data_ptr(), ws.numel() * ws.element_size()
    if mode == EPI_SWIGLU:
        _need(out2, torch.bfloat16, "out2")
        if out2.dim() != 2 or out2.stride(1) != 1 or tuple(out2.shape) != (M, N // 2):
            raise R97bError("out2 must be a row-major [M, N / 2] view")
        g.out2, g.ldo2 = out2.data_ptr(), out2.stride(0)
    if mode in (EPI_STORE_BF16, EPI_SPLIT_BF16, EPI_SWIGLU, EPI_SWIGLU_BWD):
        _need(out, torch.bfloat16, "out")
    else:
        _need(out, torch.float32, "out")
    if out.dim() != 2 or out.stride(1) != 1:
        raise R97bError("out must be a 2-D row-major view")
    g.out, g.ldo = out.data_ptr(), out.stride(0)
    if addend is not None:
        _need(addend, torch.bfloat16, "addend")
        g.addend, g.ld_add = addend.data_ptr(), addend.stride(0)
    prof = GEMM_PROFILE
    if prof is not None:
        s = stream if stream is not None else torch.cuda.current_stream()
        # inside a graph capture the events become record nodes of the graph, re-recorded at every replay
        ext = torch.cuda.is_current_stream_capturing()
        e0 = torch.cuda.Event(enable_timing=True, external=ext)
        e1 = torch.cuda.Event(enable_timing=True, external=ext)
        e0.record(s)
    check(lib().r97b_gemm(ctypes.byref(g), _stream(stream)), "r97b_gemm")
    if prof is not None:
        e1.record(s)
        full = 2.0 * M * N * (K1 + (g.K2 if a2 is not None else 0))
        shape = f"{M}x{N}x{K1}+{g.K2 if a2 is not None else 0} mode {mode} mn {int(a_mn)}{int(b_mn)}"
        prof.append((e0, e1, full if flops is None else float(flops), shape))
    return out


def skinny_tiling(M: int, N: int, K: int, sms: int = 148):
    """(bn, splits) for a GEMM with few output columns (the adapter's shrink and expand products, N = a
    few x 64, bf16 out): bn 64 up to 64 columns, else 128; the reduction is split in two (EPI_SPLIT_BF16)
    when the tiles would fill under 100 of the SMs and a split pays for its partial tiles -- always at 64
    columns, and for wider outputs only with a long reduction (K >= 8192). Measured on B200 at the
    config-5 shapes (M = 8192)."""
    bn = 64 if N <= 64 else 128
    units = -(-M // 128) * -(-N // bn)
    splits = 2 if units < 100 and (N <= 64 or K >= 8192) else 1
    return bn, splits


def grad_tiling(M: int, N: int, K: int = 8192, sms: int = 148) -> tuple:
    """(bn, splits) for the adapter-gradient GEMMs (f32 atomic accumulation, reduction over the K tokens): the
    split count s (at most 8, K / s >= 1024) minimising ceil(tiles s / sms) / s -- the waves of work each
    tile's share takes -- ties to the fewer splits. Measured on B200 at the config-5 shapes (M = 64 .. 12288
    output rows, N = 64 .. 192): within 5 % of the best of s = 1 .. 8 everywhere."""
    bn = 128 if N >= 128 else 64
    tiles = -(-M // 128) * -(-N // bn)
    best = 1
    for s in range(2, max(1, min(8, K // 1024)) + 1):
        if -(-tiles * s // sms) * best < -(-tiles * best // sms) * s:
            best = s
    return bn, best


class SplitWorkspace:
    """A zero-initialised device buffer for EPI_SPLIT_BF16 GEMMs on one stream: its tile counters return
    to zero after every call, so consecutive calls share it; calls on different streams need their own."""

    def __init__(self, device, nbytes: int = 64 << 20):
        self.buf = torch.zeros(nbytes // 4, dtype=torch.int32, device=device)


# When a list, every gemm() appends (start event, end event, algorithmic FLOPs, shape) recorded on its stream (in a
# captured graph: recorded again by every replay, so a summary after replays reads the last one):
# bench.py's live measurement of the tensor-core GEMM's launch durations.
GEMM_PROFILE = None


def gemm_profile_summary(prof):
    """(launches, total device ms, total FLOPs) of a recorded profile (synchronises)."""
    torch.cuda.synchronize()
    ms = sum(e[0].elapsed_time(e[1]) for e in prof)
    return len(prof), ms, sum(e[2] for e in prof)


def gemm_profile_by_shape(prof):
    """{shape: (launches, device ms, FLOPs)} of a recorded profile (synchronises)."""
    torch.cuda.synchronize()
    out = {}
    for e0, e1, f, shape in prof:
        n, ms, fl = out.get(shape, (0, 0.0, 0.0))
        out[shape] = (n + 1, ms + e0.elapsed_time(e1), fl + f)
    return out


# ------------------------------------------------------------------------------------------ norms

def rmsnorm_fwd(x, w, *, eps=1e-6, wadd=0.0, mult=1.0, out=None, rstd=None, stream=None):
    _need(x, torch.bfloat16, "x")
    n = x.shape[-1]
    rows = x.numel() // n
    out = torch.empty_like(x) if out is None else out
    check(lib().r97b_rmsnorm_fwd(_ptr(x), _ptr(w), _ptr(out), _ptr(rstd), rows, n, eps, wadd, mult, _stream(stream)),
          "r97b_rmsnorm_fwd")
    return out


def rmsnorm_bwd(x, w, dy, *, addend=None, eps=1e-6, wadd=0.0, mult=1.0, out=None, stream=None):
    _need(x, torch.bfloat16, "x")
    _need(dy, torch.bfloat16, "dy")
    n = x.shape[-1]
    rows = x.numel() // n
    out = torch.empty_like(x) if out is None else out
    check(lib().r97b_rmsnorm_bwd(_ptr(x), _ptr(w), _ptr(dy), _ptr(addend), _ptr(out), rows, n, eps, wadd, mult,
                                 _stream(stream)), "r97b_rmsnorm_bwd")
    return out


def _z_layout(z, n, rows):
    """(token stride, heads per token) of z: dense rows of n, or a [T, heads * n] column slice of a wider row."""
    if z.dim() == 2 and z.shape[1] != n and z.stride(1) == 1:
        heads = z.shape[1] // n
        return z.stride(0), heads
    return 0, 0


def gated_rmsnorm_fwd(x, z, w, *, eps=1e-6, sigmoid=False, out=None, stream=None):
    """x dense [rows, n]; z either dense like x or a [T, heads * n] view (row r = token r // heads)."""
    n = x.shape[-1]
    rows = x.numel() // n
    zts, zh = _z_layout(z, n, rows)
    out = torch.empty_like(x) if out is None else out
    check(lib().r97b_gated_rmsnorm_fwd(_ptr(x), _ptr(z), zts, zh, _ptr(w), _ptr(out), rows, n, eps, int(sigmoid),
                                       _stream(stream)), "r97b_gated_rmsnorm_fwd")
    return out


def gated_rmsnorm_bwd(x, z, w, dout, *, eps=1e-6, sigmoid=False, dx=None, dz=None, stream=None):
    """dz has z's layout (dense, or the same column slice of a wider buffer)."""
    n = x.shape[-1]
    rows = x.numel() // n
    zts, zh = _z_layout(z, n, rows)
    dx = torch.empty_like(x) if dx is None else dx
    dz = torch.empty_like(z) if dz is None else dz
    if zh and (dz.stride(0) != zts):
        raise R97bError("dz must share z's token stride")
    check(lib().r97b_gated_rmsnorm_bwd(_ptr(x), _ptr(z), zts, zh, _ptr(w), _ptr(dout), _ptr(dx), _ptr(dz), rows, n,
                                       eps, int(sigmoid), _stream(stream)), "r97b_gated_rmsnorm_bwd")
    return dx, dz


# ------------------------------------------------------------------------------------------ loss

def ce_kld(logits, targets=None, teacher=None, *, grad=None, grad_scale=1.0, w_ce=1.0, w_kl=1.0, loss_ce=None,
           loss_kl=None, stream=None):
    """Per-row CE / KL losses and the bf16 gradient (in place when grad is logits)."""
    _need(logits, torch.bfloat16, "logits")
    rows, vocab = logits.shape
    if loss_ce is None and targets is not None:
        loss_ce = torch.empty(rows, dtype=torch.float32, device=logits.device)
    if loss_kl is None and teacher is not None:
        loss_kl = torch.empty(rows, dtype=torch.float32, device=logits.device)
    check(lib().r97b_ce_kld(_ptr(logits), _ptr(teacher), _ptr(targets), _ptr(grad), _ptr(loss_ce), _ptr(loss_kl),
                            rows, vocab, logits.stride(0), teacher.stride(0) if teacher is not None else 0,
                            grad_scale, w_ce, w_kl, _stream(stream)), "r97b_ce_kld")
    return loss_ce, loss_kl


# ------------------------------------------------------------------------------------------ AdamW

def adamw_step(w, m, v, g, *, lr, beta1, beta2, eps, weight_decay, bc1, bc2, inv_k=1.0, clip_scale=None,
               zero_grad=False, stream=None):
    for t, nm in ((w, "w"), (m, "m"), (v, "v"), (g, "g")):
        _need(t, torch.float32, nm)
    check(lib().r97b_adamw_step(_ptr(w), _ptr(m), _ptr(v), _ptr(g), w.numel(), lr, beta1, beta2, eps, weight_decay,
                                bc1, bc2, inv_k, _ptr(clip_scale), int(zero_grad), _stream(stream)),
          "r97b_adamw_step")


def adamw_step_dev(w, m, v, g, sched, *, beta1, beta2, eps, weight_decay, inv_k=1.0, clip_scale=None,
                   zero_grad=False, stream=None):
    """AdamW with lr, bc1, bc2 read from the device tensor sched[0:3] when the kernel runs."""
    for t, nm in ((w, "w"), (m, "m"), (v, "v"), (g, "g"), (sched, "sched")):
        _need(t, torch.float32, nm)
    check(lib().r97b_adamw_step_dev(_ptr(w), _ptr(m), _ptr(v), _ptr(g), w.numel(), _ptr(sched), beta1, beta2, eps,
                                    weight_decay, inv_k, _ptr(clip_scale), int(zero_grad), _stream(stream)),
          "r97b_adamw_step_dev")


def global_norm(g, *, inv_k=1.0, max_norm=0.0, scratch=None, stream=None):
    n = g.numel()
    nbytes = lib().r97b_global_norm_scratch_bytes(n)
    if scratch is None:
        scratch = torch.empty(nbytes // 8, dtype=torch.float64, device=g.device)
    out = torch.empty(2, dtype=torch.float32, device=g.device)
    check(lib().r97b_global_norm(_ptr(g), n, inv_k, max_norm, _ptr(scratch), ctypes.c_void_p(out.data_ptr()),
                                 ctypes.c_void_p(out.data_ptr() + 4), _stream(stream)), "r97b_global_norm")
    return out[0], out[1:2]


# ------------------------------------------------------------------------------------------ layer kernels

def conv_prep_fwd(x, conv_w, cu_dev, n_seq, Hg, H, q, k, v, stream=None):
    """q, k (L2-normalised) and v of the causal conv + silu over the first (2 Hg + H) 128 columns of x."""
    T = x.shape[0]
    check(lib().r97b_conv_prep_fwd(_ptr(x), x.stride(0), _ptr(conv_w), _ptr(cu_dev), n_seq, T, Hg, H, _ptr(q),
                                   _ptr(k), _ptr(v), _stream(stream)), "r97b_conv_prep_fwd")


def conv_prep_bwd(x, conv_w, cu_dev, n_seq, Hg, H, dq, dk, dv, dx, stream=None):
    """dq, dk: f32 [T, Hg, 128], or [T, H, 128] per value head (summed over the heads of a key head as read)."""
    T = x.shape[0]
    check(lib().r97b_conv_prep_bwd(_ptr(x), x.stride(0), _ptr(conv_w), _ptr(cu_dev), n_seq, T, Hg, H, _ptr(dq),
                                   _ptr(dk), _ptr(dv), dq.shape[1], _ptr(dx), dx.stride(0), _stream(stream)),
          "r97b_conv_prep_bwd")


def gates_fwd(ba, a_log, dt_bias, plan, g, beta, stream=None):
    check(lib().r97b_gates_fwd(_ptr(ba), ba.stride(0), _ptr(a_log), _ptr(dt_bias), _ptr(plan.tok0), _ptr(plan.len),
                               plan.n_chunks, plan.H, _ptr(g), _ptr(beta), _stream(stream)), "r97b_gates_fwd")


def gates_bwd(ba, a_log, dt_bias, plan, dg, dbeta, dba, stream=None):
    check(lib().r97b_gates_bwd(_ptr(ba), ba.stride(0), _ptr(a_log), _ptr(dt_bias), _ptr(plan.tok0), _ptr(plan.len),
                               plan.n_chunks, plan.H, _ptr(dg), _ptr(dbeta), _ptr(dba), dba.stride(0),
                               _stream(stream)), "r97b_gates_bwd")


def swiglu_fwd(gu, y, stream=None):
    rows, n = y.shape
    check(lib().r97b_swiglu_fwd(_ptr(gu), gu.stride(0), rows, n, _ptr(y), y.stride(0), _stream(stream)),
          "r97b_swiglu_fwd")


def swiglu_bwd(gu, dy, dgu, stream=None):
    rows, n = dy.shape
    check(lib().r97b_swiglu_bwd(_ptr(gu), gu.stride(0), rows, n, _ptr(dy), dy.stride(0), _ptr(dgu), dgu.stride(0),
                                _stream(stream)), "r97b_swiglu_bwd")


def qk_norm_rope_fwd(x, head_stride, heads, head_dim, w, cos_t, sin_t, rot, S, eps, out, stream=None):
    """Per (token, head) row of head_dim: RMSNorm with gain w, NeoX RoPE on the first rot dims, into
    out [B, heads, S, head_dim]."""
    T = x.shape[0]
    check(lib().r97b_qk_norm_rope_fwd(_ptr(x), x.stride(0), head_stride, heads, head_dim, _ptr(w), _ptr(cos_t),
                                      _ptr(sin_t), rot, T, S, eps, _ptr(out), _stream(stream)),
          "r97b_qk_norm_rope_fwd")


def qk_norm_rope_bwd(x, head_stride, heads, head_dim, w, cos_t, sin_t, rot, S, eps, dout, dx, stream=None):
    T = x.shape[0]
    check(lib().r97b_qk_norm_rope_bwd(_ptr(x), x.stride(0), head_stride, heads, head_dim, _ptr(w), _ptr(cos_t),
                                      _ptr(sin_t), rot, T, S, eps, _ptr(dout), _ptr(dx), dx.stride(0),
                                      _stream(stream)), "r97b_qk_norm_rope_bwd")


def to_bhsd(x, head_stride, heads, head_dim, S, out, reverse=False, stream=None):
    T = x.shape[0]
    check(lib().r97b_to_bhsd(_ptr(x), x.stride(0), head_stride, heads, head_dim, T, S, _ptr(out), int(reverse),
                             _stream(stream)), "r97b_to_bhsd")


def gate_mul_fwd(attn, gate, gate_hs, heads, head_dim, S, y, stream=None):
    T = y.shape[0]
    check(lib().r97b_gate_mul_fwd(_ptr(attn), _ptr(gate), gate.stride(0), gate_hs, heads, head_dim, T, S, _ptr(y),
                                  _stream(stream)), "r97b_gate_mul_fwd")


def gate_mul_bwd(attn, gate, gate_hs, heads, head_dim, S, dy, dattn, dgate, stream=None):
    T = dy.shape[0]
    check(lib().r97b_gate_mul_bwd(_ptr(attn), _ptr(gate), gate.stride(0), gate_hs, heads, head_dim, T, S, _ptr(dy),
                                  _ptr(dattn), _ptr(dgate), dgate.stride(0), _stream(stream)), "r97b_gate_mul_bwd")


def qlinear_lora_workspace(M: int, N: int, K: int, rank: int, device) -> torch.Tensor:
    """The zeroed split-K workspace r97b_qlinear_lora_fwd / _bwd need for these shapes."""
    n = int(lib().r97b_qlinear_lora_workspace_bytes(M, N, K, rank))
    if n < 0:
        raise R97bError("r97b_qlinear_lora_workspace_bytes: bad shape")
    return torch.zeros(max(n, 256), dtype=torch.uint8, device=device)


def qlinear_lora_fwd(w, w_bf16, x, A, B, scale, *, t=None, y=None, addend=None, w_decoded=False, ws=None,
                     stream=None):
    """y = x decode(w)^T + (scale x A^T) B^T (+ addend) through r97b_qlinear_lora_fwd; returns (y, t).
    `w` is an iqr.IqrWeight [N, K]; w_bf16 [N, K] receives (or, with w_decoded, holds) its decode."""
    from . import iqr as IQ
    M, K = x.shape
    N, r = B.shape
    t = torch.empty((M, r), dtype=torch.bfloat16, device=x.device) if t is None else t
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device) if y is None else y
    ws = qlinear_lora_workspace(M, N, K, r, x.device) if ws is None else ws
    for u, nm in ((w_bf16, "w_bf16"), (x, "x"), (A, "A"), (B, "B"), (t, "t"), (y, "y")):
        _need(u, torch.bfloat16, nm)
    d = IQ.make_desc(w) if w is not None else None
    a = R97bQLinearLora(M, N, K, r, float(scale), ctypes.cast(ctypes.pointer(d), ctypes.c_void_p) if d else None,
                        _ptr(w_bf16), int(w_decoded), 0, _ptr(x), _ptr(A), _ptr(B), _ptr(t), _ptr(y), _ptr(addend),
                        _ptr(ws), ws.numel())
    check(lib().r97b_qlinear_lora_fwd(ctypes.byref(a), _stream(stream)), "r97b_qlinear_lora_fwd")
    return y, t


def qlinear_lora_bwd(w_bf16, x, A, B, t, dy, scale, dA, dB, *, dx=None, dt=None, ws=None, stream=None):
    """dx = dy W + (scale dy B) A; dA += dt^T x; dB += dy^T t (f32) through r97b_qlinear_lora_bwd; returns dx."""
    M, K = x.shape
    N, r = B.shape
    dx = torch.empty((M, K), dtype=torch.bfloat16, device=x.device) if dx is None else dx
    dt = torch.empty((M, r), dtype=torch.bfloat16, device=x.device) if dt is None else dt
    ws = qlinear_lora_workspace(M, N, K, r, x.device) if ws is None else ws
    _need(dA, torch.float32, "dA")
    _need(dB, torch.float32, "dB")
    a = R97bQLinearLoraBwd(M, N, K, r, float(scale), _ptr(w_bf16), _ptr(x), _ptr(A), _ptr(B), _ptr(t), _ptr(dy),
                           _ptr(dt), _ptr(dx), _ptr(dA), _ptr(dB), _ptr(ws), ws.numel())
    check(lib().r97b_qlinear_lora_bwd(ctypes.byref(a), _stream(stream)), "r97b_qlinear_lora_bwd")
    return dx


def attn_fwd(q, k, v, scale, o=None, lse=None, stream=None):
    """Causal GQA attention softmax(scale q k^T) v on this package's tcgen05 kernel (r97b_attn_fwd): q
    [B, Hq, S, D], k, v [B, Hkv, S, D] bf16 contiguous. Returns (o [B, Hq, S, D] bf16, lse [B, Hq, S] f32, the
    natural-log log-sum-exp r97b_attn_bwd reads)."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    for t, name, shape in ((q, "q", (B, Hq, S, D)), (k, "k", (B, Hkv, S, D)), (v, "v", (B, Hkv, S, D))):
        _need(t, torch.bfloat16, name)
        if tuple(t.shape) != shape or not t.is_contiguous():
            raise R97bError(f"{name} must be a contiguous {shape} bf16 tensor")
    o = torch.empty_like(q) if o is None else o
    lse = torch.empty((B, Hq, S), dtype=torch.float32, device=q.device) if lse is None else lse
    a = R97bAttnFwd(B, Hq, Hkv, S, D, float(scale), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse))
    check(lib().r97b_attn_fwd(ctypes.byref(a), _stream(stream)), "r97b_attn_fwd")
    return o, lse


def attn_bwd_workspace(B: int, Hq: int, S: int, device) -> torch.Tensor:
    """A device buffer of the bytes r97b_attn_bwd needs for (B, Hq, S) (the P and dS tiles, the row sums)."""
    n = int(lib().r97b_attn_bwd_workspace_bytes(B, Hq, S))
    if n < 0:
        raise R97bError("r97b_attn_bwd_workspace_bytes: bad shape")
    return torch.empty(n, dtype=torch.uint8, device=device)


def attn_bwd(q, k, v, o, dout, lse, scale, ws, dq=None, dk=None, dv=None, stream=None):
    """dq, dk, dv of causal GQA attention softmax(scale q k^T) v (r97b_attn_bwd): q, o, dout [B, Hq, S, D],
    k, v [B, Hkv, S, D] bf16 contiguous; lse f32 [B, Hq, S] (the forward's natural-log log-sum-exp)."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    for t, name, shape in ((q, "q", (B, Hq, S, D)), (k, "k", (B, Hkv, S, D)), (v, "v", (B, Hkv, S, D)),
                           (o, "o", (B, Hq, S, D)), (dout, "dout", (B, Hq, S, D))):
        _need(t, torch.bfloat16, name)
        if tuple(t.shape) != shape or not t.is_contiguous():
            raise R97bError(f"{name} must be a contiguous {shape} bf16 tensor")
    if lse.dtype != torch.float32 or lse.dim() != 3 or tuple(lse.shape) != (B, Hq, S) or not lse.is_contiguous():
        raise R97bError("lse must be a contiguous [B, Hq, S] f32 tensor")
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(k) if dk is None else dk
    dv = torch.empty_like(v) if dv is None else dv
    a = R97bAttnBwd(B, Hq, Hkv, S, D, float(scale), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dout), _ptr(lse),
                    _ptr(dq), _ptr(dk), _ptr(dv), _ptr(ws), ws.numel() * ws.element_size())
    check(lib().r97b_attn_bwd(ctypes.byref(a), _stream(stream)), "r97b_attn_bwd")
    return dq, dk, dv


def embed(table, ids, out, stream=None):
    T, n = out.shape
    check(lib().r97b_embed(_ptr(table), table.stride(0), table.shape[0], _ptr(ids), T, n, _ptr(out),
                           _stream(stream)), "r97b_embed")


class CastTable:
    """A fixed list of f32 -> bf16 casts (2-D views, columns a multiple of 8, rows 16-byte aligned) run as one
    launch (r97b_cast_segments); the table lives in device memory, built once."""

    def __init__(self, pairs, device):
        segs = (R97bCastSeg * len(pairs))()
        units = 0
        for i, (src, dst) in enumerate(pairs):
            rows, cols = src.shape
            if tuple(dst.shape) != (rows, cols) or cols % 8 or src.stride(1) != 1 or dst.stride(1) != 1:
                raise R97bError("CastTable: views must be row-major with a multiple of 8 columns")
            if src.data_ptr() % 16 or dst.data_ptr() % 16 or src.stride(0) % 4 or dst.stride(0) % 8:
                raise R97bError("CastTable: rows must start 16-byte aligned")
            segs[i] = R97bCastSeg(src.data_ptr(), src.stride(0), dst.data_ptr(), dst.stride(0), rows, cols, units)
            units += rows * cols // 8
        raw = bytes(segs)
        self.table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(device)
        self.n, self.units = len(pairs), units
        self.keep = pairs

    def run(self, stream=None):
        check(lib().r97b_cast_segments(_ptr(self.table), self.n, self.units, _stream(stream)), "r97b_cast_segments")


def cast_f32_bf16(src, dst, stream=None):
    rows, cols = src.shape
    check(lib().r97b_cast_f32_bf16(_ptr(src), src.stride(0), _ptr(dst), dst.stride(0), rows, cols,
                                   _stream(stream)), "r97b_cast_f32_bf16")


def quant_act_i8g(x, group, rotate=True, codes=None, scale=None, stream=None):
    """The w8a8 trunk's activation quantiser (had_quant_act_i8g when rotate, else quant_act_i8g): x bf16
    [rows, n] -> (codes int8 [rows, n], scale f32 [rows, ceil(n / group)])."""
    rows, n = x.shape
    t = group if (rotate or 0 < group <= n) else n
    ngrp = (n + t - 1) // t
    if codes is None:
        codes = torch.empty((rows, n), dtype=torch.int8, device=x.device)
    if scale is None:
        scale = torch.empty((rows, ngrp), dtype=torch.float32, device=x.device)
    check(lib().r97b_quant_act_i8g(_ptr(x), x.stride(0), rows, n, group, 1 if rotate else 0, _ptr(codes),
                                   codes.stride(0), _ptr(scale), _stream(stream)), "r97b_quant_act_i8g")
    return codes, scale


def quant_act_i8g_bwd(x, group, scale, g, rotate=True, dx=None, accumulate=False, stream=None):
    """Its straight-through adjoint: the codes' cotangent g (f32 [rows, n]) -> dx f32 [rows, n]."""
    rows, n = x.shape
    if dx is None:
        dx = torch.empty((rows, n), dtype=torch.float32, device=x.device)
    check(lib().r97b_quant_act_i8g_bwd(_ptr(x), x.stride(0), rows, n, group, 1 if rotate else 0, _ptr(scale),
                                       _ptr(g), g.stride(0), _ptr(dx), dx.stride(0), 1 if accumulate else 0,
                                       _stream(stream)), "r97b_quant_act_i8g_bwd")
    return dx


def gemm_i8g(a, a_scale, b, b_scale, out_dtype=torch.float32, y=None, stream=None):
    """The w8a8 trunk's int8 product (gemm_nt_q at i8a8h): a int8 [M, K], b int8 [N, K], a_scale f32
    [M, ceil(K / 128)], b_scale f32 [N, ceil(K / 128)] -> y [M, N] = sum_g sa sb (a_g . b_g), f32 or bf16."""
    M, K = a.shape
    N = b.shape[0]
    if y is None:
        y = torch.empty((M, N), dtype=out_dtype, device=a.device)
    check(lib().r97b_gemm_i8g(_ptr(a), a.stride(0), _ptr(a_scale), a_scale.stride(0), _ptr(b), b.stride(0),
                              _ptr(b_scale), b_scale.stride(0), M, N, K, _ptr(y), y.stride(0),
                              1 if y.dtype == torch.bfloat16 else 0, _stream(stream)), "r97b_gemm_i8g")
    return y


def gemm_i8g_gated(a, a_scale, b, b_scale, act="silu", want_bf16=False, stream=None):
    """The gated narrow fold (gemm_nt_q_gated): b int8 [2 n, K] = [gate; up] -> (q int8 [M, n], scale f32
    [M, n / 128], and the unrotated product bf16 [M, n] when want_bf16, else None)."""
    M, K = a.shape
    N = b.shape[0]
    n = N // 2
    q = torch.empty((M, n), dtype=torch.int8, device=a.device)
    qs = torch.empty((M, max(1, n // 128)), dtype=torch.float32, device=a.device)
    ob = torch.empty((M, n), dtype=torch.bfloat16, device=a.device) if want_bf16 else None
    check(lib().r97b_gemm_i8g_gated(_ptr(a), a.stride(0), _ptr(a_scale), a_scale.stride(0), _ptr(b), b.stride(0),
                                    _ptr(b_scale), b_scale.stride(0), M, N, K, 1 if act == "sigmoid" else 0,
                                    _ptr(q), q.stride(0), _ptr(qs), qs.stride(0), _ptr(ob),
                                    ob.stride(0) if ob is not None else 0, _stream(stream)), "r97b_gemm_i8g_gated")
    return q, qs, ob


FUSED_PARTS = {"rmsnorm": 0, "silu_mul": 1, "sigmoid_mul": 2}


def fused_quant_i8g(part, x, group, x2=None, w=None, eps=1e-6, wadd=0.0, mult=1.0, want_out=True, stream=None):
    """The int8 trunk's fused producers (rmsnorm / silu_mul / sigmoid_mul, then the rotated quantiser): x bf16
    [rows, n] (gate_up [rows, 2 n] for silu_mul), x2 bf16 [rows, n] (sigmoid_mul's b), w f32 [n] (rmsnorm's
    gain) -> (codes int8 [rows, n], scale f32 [rows, n / group], the part's value bf16 [rows, n] or None)."""
    pid = FUSED_PARTS[part]
    rows = x.shape[0]
    n = x.shape[1] // 2 if pid == 1 else x.shape[1]
    codes = torch.empty((rows, n), dtype=torch.int8, device=x.device)
    scale = torch.empty((rows, n // group), dtype=torch.float32, device=x.device)
    out = torch.empty((rows, n), dtype=torch.bfloat16, device=x.device) if want_out else None
    check(lib().r97b_fused_quant_i8g(pid, _ptr(x), x.stride(0), _ptr(x2), x2.stride(0) if x2 is not None else 0,
                                     _ptr(w), eps, wadd, mult, rows, n, group, _ptr(codes), codes.stride(0),
                                     _ptr(scale), scale.stride(0), _ptr(out), out.stride(0) if out is not None else 0,
                                     _stream(stream)), "r97b_fused_quant_i8g")
    return codes, scale, out


def fused_quant_i8g_bwd(part, x, group, scale, g, g_out=None, x2=None, w=None, eps=1e-6, wadd=0.0, mult=1.0,
                        stream=None):
    """Its adjoint: the codes' cotangent g (f32 [rows, n]) and the part value's g_out -> dx (f32, x's shape) and,
    for sigmoid_mul, db (f32 [rows, n]); returns (dx, db or None)."""
    pid = FUSED_PARTS[part]
    rows = x.shape[0]
    n = x.shape[1] // 2 if pid == 1 else x.shape[1]
    dx = torch.zeros((rows, x.shape[1]), dtype=torch.float32, device=x.device)
    dx2 = torch.zeros((rows, n), dtype=torch.float32, device=x.device) if pid == 2 else None
    check(lib().r97b_fused_quant_i8g_bwd(pid, _ptr(x), x.stride(0), _ptr(x2), x2.stride(0) if x2 is not None else 0,
                                         _ptr(w), eps, wadd, mult, rows, n, group, _ptr(scale), scale.stride(0),
                                         _ptr(g), g.stride(0), _ptr(g_out), g_out.stride(0) if g_out is not None else 0,
                                         _ptr(dx), dx.stride(0), _ptr(dx2), dx2.stride(0) if dx2 is not None else 0,
                                         0, _stream(stream)), "r97b_fused_quant_i8g_bwd")
    return dx, dx2
