"""Torch-facing wrappers over the C ABI of libr97b200.so.

Torch tensors supply device memory and the current CUDA stream; the arithmetic is the library's
sm_100a kernels. Every wrapper checks shapes, dtypes and contiguity, then calls the C entry point and
raises R97bError on a non-zero status. Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import R97bGemm, R97bMat, R97bError, check, lib

EPI_STORE_BF16, EPI_STORE_F32, EPI_ATOMIC_F32, EPI_ATOMIC_F32T = 0, 1, 2, 3


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
         addend=None, beta=1.0, splits=1, bn=0, M=None, N=None, stream=None):
    """out (+)= alpha * (A1 B1^T + A2 B2^T) (+ beta * addend); see include/r97b.h (r97b_gemm).

    A1 is [M, K1] (K-major) or stored [K1, M] (a_mn); B1 is [N, K1] or stored [K1, N] (b_mn); the optional
    tail (a2, b2) has the same majorness with its own K2."""
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
    if mode == EPI_STORE_BF16:
        _need(out, torch.bfloat16, "out")
    else:
        _need(out, torch.float32, "out")
    if out.dim() != 2 or out.stride(1) != 1:
        raise R97bError("out must be a 2-D row-major view")
    g.out, g.ldo = out.data_ptr(), out.stride(0)
    if addend is not None:
        _need(addend, torch.bfloat16, "addend")
        g.addend, g.ld_add = addend.data_ptr(), addend.stride(0)
    check(lib().r97b_gemm(ctypes.byref(g), _stream(stream)), "r97b_gemm")
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


def gated_rmsnorm_fwd(x, z, w, *, eps=1e-6, sigmoid=False, out=None, stream=None):
    n = x.shape[-1]
    rows = x.numel() // n
    out = torch.empty_like(x) if out is None else out
    check(lib().r97b_gated_rmsnorm_fwd(_ptr(x), _ptr(z), _ptr(w), _ptr(out), rows, n, eps, int(sigmoid),
                                       _stream(stream)), "r97b_gated_rmsnorm_fwd")
    return out


def gated_rmsnorm_bwd(x, z, w, dout, *, eps=1e-6, sigmoid=False, dx=None, dz=None, stream=None):
    n = x.shape[-1]
    rows = x.numel() // n
    dx = torch.empty_like(x) if dx is None else dx
    dz = torch.empty_like(z) if dz is None else dz
    check(lib().r97b_gated_rmsnorm_bwd(_ptr(x), _ptr(z), _ptr(w), _ptr(dout), _ptr(dx), _ptr(dz), rows, n, eps,
                                       int(sigmoid), _stream(stream)), "r97b_gated_rmsnorm_bwd")
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


def global_norm(g, *, inv_k=1.0, max_norm=0.0, scratch=None, stream=None):
    n = g.numel()
    nbytes = lib().r97b_global_norm_scratch_bytes(n)
    if scratch is None:
        scratch = torch.empty(nbytes // 8, dtype=torch.float64, device=g.device)
    out = torch.empty(2, dtype=torch.float32, device=g.device)
    check(lib().r97b_global_norm(_ptr(g), n, inv_k, max_norm, _ptr(scratch), ctypes.c_void_p(out.data_ptr()),
                                 ctypes.c_void_p(out.data_ptr() + 4), _stream(stream)), "r97b_global_norm")
    return out[0], out[1:2]
