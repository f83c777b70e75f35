"""TEST INFRASTRUCTURE -- numpy f64 restatements of the reference's host twins and adjoints on the
LoRA-over-IQR hot path. Each function cites the reference lines it restates. Only tests/, bench.py's
cpu_baseline leg and __graft_entry__.smoke() use these, as the checker.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import oracle_lib


# ----------------------------------------------------------------------------- IQR decode (C)

class IqrDesc(ctypes.Structure):
    """The C layout of include/r97b_iqr.h (the reference's R97IqrDecodeDesc)."""
    _fields_ = [
        ("rows_all", ctypes.c_int64), ("cols", ctypes.c_int64), ("row0", ctypes.c_int64), ("rows", ctypes.c_int64),
        ("bits", ctypes.c_int32), ("state_bits", ctypes.c_int32), ("run_rows", ctypes.c_int32), ("rb", ctypes.c_int32),
        ("mad", ctypes.c_int32), ("round_mad", ctypes.c_int32), ("mad_a", ctypes.c_uint32), ("mad_b", ctypes.c_uint32),
        ("lut", ctypes.c_void_p),
        ("codes", ctypes.c_void_p), ("codes_row_bytes", ctypes.c_int64),
        ("scale", ctypes.c_void_p), ("scale_dtype", ctypes.c_int32), ("scale_block_cols", ctypes.c_int64),
        ("scale_row_bytes", ctypes.c_int64),
        ("affine", ctypes.c_int32), ("zero", ctypes.c_void_p), ("zero_bits", ctypes.c_int32),
        ("zero_row_bytes", ctypes.c_int64),
        ("scale2", ctypes.c_void_p), ("scale2_dtype", ctypes.c_int32), ("scale2_row_bytes", ctypes.c_int64),
        ("scale2_block_rows", ctypes.c_int64), ("scale2_block_cols", ctypes.c_int64),
        ("out_codes", ctypes.c_void_p), ("out_scale", ctypes.c_void_p),
    ]


def iqr_form_desc(form: dict, out_codes: np.ndarray, out_scale: np.ndarray, row0=0, rows=None) -> IqrDesc:
    """A description over numpy planes. `form` holds: rows_all, cols, bits, state_bits, run_rows, rb, mad,
    round_mad, mad_a, mad_b, lut (int8 array or None), codes (uint8 [rows_all, row_bytes]), scale (uint8 view
    of the scale plane [rows_all, row_bytes]), scale_dtype, scale_block_cols, and optional affine/zero/
    zero_bits, scale2/scale2_dtype/scale2_block_rows/scale2_block_cols."""
    d = IqrDesc()
    rows_all = form["rows_all"]
    rows = rows_all - row0 if rows is None else rows
    d.rows_all, d.cols, d.row0, d.rows = rows_all, form["cols"], row0, rows
    d.bits, d.state_bits = form.get("bits", 4), form.get("state_bits", 16)
    d.run_rows, d.rb = form.get("run_rows", 256), form.get("rb", 1)
    d.mad, d.round_mad = form.get("mad", 1), form.get("round_mad", 0)
    d.mad_a, d.mad_b = form.get("mad_a", 0), form.get("mad_b", 0)
    lut = form.get("lut")
    d.lut = None if lut is None else lut.ctypes.data
    codes = form["codes"]
    d.codes = codes.ctypes.data + row0 * codes.strides[0]
    d.codes_row_bytes = codes.strides[0]
    sc = form["scale"]
    d.scale = sc.ctypes.data + row0 * sc.strides[0]
    d.scale_dtype = form.get("scale_dtype", 0)
    d.scale_block_cols = form.get("scale_block_cols", 128)
    d.scale_row_bytes = sc.strides[0]
    d.affine = form.get("affine", 0)
    z = form.get("zero")
    if z is not None:
        d.zero = z.ctypes.data + row0 * z.strides[0]
        d.zero_row_bytes = z.strides[0]
        d.zero_bits = form.get("zero_bits", 8)
    s2 = form.get("scale2")
    if s2 is not None:
        d.scale2 = s2.ctypes.data
        d.scale2_dtype = form.get("scale2_dtype", 0)
        d.scale2_row_bytes = s2.strides[0] if s2.ndim > 1 else s2.nbytes
        d.scale2_block_rows = form.get("scale2_block_rows", 0)
        d.scale2_block_cols = form.get("scale2_block_cols", 0)
    d.out_codes = out_codes.ctypes.data
    d.out_scale = out_scale.ctypes.data
    return d


def iqr_decode(form: dict, row0=0, rows=None, lib=None):
    """(int8 codes, uint16 bf16-bit scales) of rows [row0, row0+rows), through the C restatement (or, with
    lib=oracle.ref_lib(), through the reference's own r97_iqr_decode_host)."""
    rows = form["rows_all"] - row0 if rows is None else rows
    codes = np.zeros((rows, form["cols"]), np.int8)
    scale = np.zeros((rows, form["cols"] // 128), np.uint16)
    d = iqr_form_desc(form, codes, scale, row0, rows)
    if lib is None:
        rc = oracle_lib().oracle_iqr_decode(ctypes.byref(d))
    else:
        rc = lib.ref_iqr_decode(ctypes.byref(d))
    if rc != 0:
        raise ValueError("iqr decode rejected the description")
    return codes, scale


def trunk_form(codes: np.ndarray, scale_f32: np.ndarray, mad_a: int, mad_b: int, cols: int) -> dict:
    """The configs' trunk form over numpy planes (u4 codes [rows, cols/2], f32 scale [rows, cols/128])."""
    return dict(rows_all=codes.shape[0], cols=cols, bits=4, state_bits=16, run_rows=256, rb=1, mad=1, round_mad=0,
                mad_a=mad_a, mad_b=mad_b, codes=np.ascontiguousarray(codes),
                scale=np.ascontiguousarray(scale_f32).view(np.uint8).reshape(codes.shape[0], -1),
                scale_dtype=0, scale_block_cols=128)


def bf16_bits_to_f64(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def f64_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round to bf16 (nearest-even through f32, the way the kernels store), returned as f64."""
    f = np.asarray(x, np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


def dequant_value(codes: np.ndarray, scale_bits: np.ndarray) -> np.ndarray:
    """W[n, k] = code[n, k] * bf16 scale[n, k/128] in f64 (reference src/adjoint/host/linear.cpp:155-163)."""
    s = bf16_bits_to_f64(scale_bits)
    return codes.astype(np.float64) * np.repeat(s, 128, axis=1)


# ----------------------------------------------------------------------------- linear + LoRA

def gemm_nt(a, w):
    """y[M,N] = a[M,K] w[N,K]^T (reference src/adjoint/host/linear.cpp:193-218)."""
    return a @ w.T


def gemm_nt_dx(dy, w):
    """dx[M,K] = dy[M,N] w[N,K] (reference src/adjoint/host/linear.cpp:220-243)."""
    return dy @ w


def lora_fwd(x, W, A, B, scale):
    """t = x A^T; y = x W^T + scale * t B^T (reference lora.cpp:290-305 shrink twin, 416-451 expand twin,
    one slot, scale[s, n] = alpha / r)."""
    t = x @ A.T
    return x @ W.T + scale * (t @ B.T), t


def lora_bwd(x, W, A, B, scale, t, dy):
    """The adjoints of gemm_nt + lora_shrink + lora_expand for one slot (reference lora.cpp:320-401 and
    453-521): dt = scale dy B; dB = scale dy^T t; dA = dt^T x; dx = dy W + dt A."""
    dt = scale * (dy @ B)
    dB = scale * (dy.T @ t)
    dA = dt.T @ x
    dx = dy @ W + dt @ A
    return dx, dA, dB, dt


# ----------------------------------------------------------------------------- norms

def rmsnorm_fwd(x, w, eps=1e-6, wadd=0.0, mult=1.0):
    """reference src/adjoint/host/elementwise.cpp:459-528"""
    s = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return x * s * ((w + wadd) if w is not None else 1.0) * mult


def rmsnorm_bwd(x, w, dy, eps=1e-6, wadd=0.0, mult=1.0):
    """dx = mult (s c dy - s^3 x / n sum(dy x c)) (reference src/adjoint/host/elementwise.cpp:531-670)"""
    n = x.shape[-1]
    c = (w + wadd) if w is not None else 1.0
    s = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    t = (dy * x * c).sum(-1, keepdims=True)
    return mult * (s * c * dy - s ** 3 * x * t / n)


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def gated_rmsnorm_fwd(x, z, w, eps=1e-6, sigmoid=False):
    """reference src/adjoint/host/gdn_prep.cpp:501-531"""
    sc = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    g = _sigmoid(z) if sigmoid else z * _sigmoid(z)
    return x * sc * w * g


def gated_rmsnorm_bwd(x, z, w, do, eps=1e-6, sigmoid=False):
    """reference src/adjoint/host/gdn_prep.cpp:541-592"""
    n = x.shape[-1]
    sg = _sigmoid(z)
    g = sg if sigmoid else z * sg
    dg = sg * (1 - sg) if sigmoid else sg * (1 + z * (1 - sg))
    sc = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    a = (x * do * w * g).sum(-1, keepdims=True)
    dx = w * g * sc * do - x * sc ** 3 / n * a
    dz = do * x * sc * w * dg
    return dx, dz


# ----------------------------------------------------------------------------- loss

def ce_rows(logits, targets, grad_scale=1.0):
    """Per row: loss = lse - x[target], grad = (softmax - onehot) * grad_scale; an unscored row (target < 0)
    has zero loss and zero grad (reference src/loss.cpp:21-39 ce_position; include/r97/head.h:28-45)."""
    x = logits.astype(np.float64)
    m = x.max(-1, keepdims=True)
    e = np.exp(x - m)
    s = e.sum(-1, keepdims=True)
    p = e / s
    rows = np.arange(x.shape[0])
    scored = targets >= 0
    tt = np.where(scored, targets, 0)
    # log(s) - (x_t - m): the reference's order, which keeps log(s) when m is large
    loss = np.where(scored, np.log(s[:, 0]) - (x[rows, tt] - m[:, 0]), 0.0)
    grad = p.copy()
    grad[rows, tt] -= 1.0
    grad *= grad_scale
    grad[~scored] = 0.0
    return loss, grad


def kld_rows(logits, teacher, grad_scale=1.0, targets=None):
    """KL(softmax(t) || softmax(s)) per row and its gradient softmax(s) - softmax(t). No reference
    counterpart: the reference has no KL objective, so this restatement is unpinned by it."""
    s = logits.astype(np.float64)
    t = teacher.astype(np.float64)
    ls = s - (s.max(-1, keepdims=True) + np.log(np.exp(s - s.max(-1, keepdims=True)).sum(-1, keepdims=True)))
    lt = t - (t.max(-1, keepdims=True) + np.log(np.exp(t - t.max(-1, keepdims=True)).sum(-1, keepdims=True)))
    pt, ps = np.exp(lt), np.exp(ls)
    loss = (pt * (lt - ls)).sum(-1)
    grad = (ps - pt) * grad_scale
    if targets is not None:
        scored = targets >= 0
        loss = np.where(scored, loss, 0.0)
        grad[~scored] = 0.0
    return loss, grad


# ----------------------------------------------------------------------------- AdamW (f32, exact)

def scheduled_lr(lr, warmup, total, floor_frac, step):
    """reference src/optim.cpp:113-127"""
    import math
    if step <= 0:
        return np.float32(0.0)
    lr32, ff32 = float(np.float32(lr)), float(np.float32(floor_frac))  # the config holds f32 values
    base = lr32 if lr32 > 0 else 0.0
    if warmup > 0 and step <= warmup:
        return np.float32(base * (step / warmup))
    if total <= 0 or total <= warmup:
        return np.float32(lr)
    floor = base * (ff32 if ff32 >= 0 else 0.0)
    horizon = float(total - warmup)
    t = min(float(step - warmup), horizon)
    return np.float32(floor + (base - floor) * 0.5 * (1.0 + math.cos(math.pi * t / horizon)))


def adamw_update(w, m, v, g, lr, b1, b2, eps, wd, t, inv_k=np.float32(1.0), clip_scale=None):
    """One update in f32, operation for operation as the reference (src/optim.cpp:245-290). Arrays are
    updated in place; numpy f32 arithmetic is IEEE-rounded per operation, like the reference's x86 build."""
    f = np.float32
    b1, b2, eps, wd, lr = f(b1), f(b2), f(eps), f(wd), f(lr)
    bc1 = f(1.0) - f(np.power(b1, f(t), dtype=np.float32))
    bc2 = f(1.0) - f(np.power(b2, f(t), dtype=np.float32))
    gi = (g * f(inv_k)).astype(np.float32)
    if clip_scale is not None:
        gi = (gi * f(clip_scale)).astype(np.float32)
    m[:] = b1 * m + (f(1.0) - b1) * gi
    v[:] = b2 * v + (f(1.0) - b2) * gi * gi
    mh = m / bc1
    vh = v / bc2
    w[:] = w - lr * (mh / (np.sqrt(vh) + eps) + wd * w)
    return bc1, bc2


# ----------------------------------------------------------------------------- GDN conv prep + gates

def _silu(x):
    return x / (1.0 + np.exp(-x))


def _silu_grad(x):
    s = 1.0 / (1.0 + np.exp(-x))
    return s * (1.0 + x * (1.0 - s))


def _positions(cu, T):
    pos = np.zeros(T, np.int64)
    for s in range(len(cu) - 1):
        pos[cu[s]:cu[s + 1]] = np.arange(cu[s + 1] - cu[s])
    return pos


def conv_acc(x, w, cu):
    """Causal depthwise conv of width W over each sequence from a cold start (reference
    src/adjoint/host/gdn_prep.cpp:204-229 conv_phase): acc[t, c] = sum_j x[t - W + 1 + j, c] w[c, j]."""
    T, C = x.shape
    W = w.shape[1]
    pos = _positions(cu, T)
    acc = np.zeros((T, C))
    for j in range(W):
        sh = W - 1 - j
        src = np.zeros_like(x)
        src[sh:] = x[:T - sh] if sh else x
        acc += np.where((pos >= sh)[:, None], src, 0.0) * w[:, j][None, :]
    return acc


def conv_prep_fwd(x, w, cu, Hg, H, K=128, eps=1e-6):
    """q, k (L2-normalised per head) and v (reference src/adjoint/host/gdn_prep.cpp:261-318)."""
    T = x.shape[0]
    qk = Hg * K
    u = _silu(conv_acc(x[:, :2 * qk + H * K], w, cu))
    q = u[:, :qk].reshape(T, Hg, K)
    k = u[:, qk:2 * qk].reshape(T, Hg, K)
    q = q / np.sqrt((q * q).sum(-1, keepdims=True) + eps)
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + eps)
    return q, k, u[:, 2 * qk:].reshape(T, H, K)


def conv_prep_bwd(x, w, cu, Hg, H, dq, dk, dv, K=128, eps=1e-6):
    """dx of conv_prep_fwd (reference src/adjoint/host/gdn_prep.cpp:367-455, without the carried state)."""
    T = x.shape[0]
    qk = Hg * K
    C = 2 * qk + H * K
    acc = conv_acc(x[:, :C], w, cu)
    u = _silu(acc)
    dacc = np.zeros((T, C))
    for part, dout in ((slice(0, qk), dq), (slice(qk, 2 * qk), dk)):
        uu = u[:, part].reshape(T, Hg, K)
        ss = (uu * uu).sum(-1, keepdims=True)
        inv = 1.0 / np.sqrt(ss + eps)
        dot = (uu * dout).sum(-1, keepdims=True)
        du = inv * dout - inv ** 3 * uu * dot
        dacc[:, part] = du.reshape(T, qk) * _silu_grad(acc[:, part])
    dacc[:, 2 * qk:] = dv.reshape(T, H * K) * _silu_grad(acc[:, 2 * qk:])
    pos = _positions(cu, T)
    W = w.shape[1]
    dx = np.zeros((T, C))
    for j in range(W):
        sh = W - 1 - j  # output row t reads input row t - sh
        contrib = np.where((pos >= sh)[:, None], dacc, 0.0) * w[:, j][None, :]
        dx[:T - sh] += contrib[sh:] if sh else contrib
    return dx


def _softplus(x):
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def gates_fwd(a, b, a_log, dt_bias, cu, chunk=64):
    """g = within-chunk running sum of -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b)
    (reference src/adjoint/host/gdn_prep.cpp:320-336)."""
    inc = -np.exp(a_log)[None, :] * _softplus(a + dt_bias[None, :])
    g = np.zeros_like(inc)
    for s in range(len(cu) - 1):
        for c0 in range(cu[s], cu[s + 1], chunk):
            r = slice(c0, min(cu[s + 1], c0 + chunk))
            g[r] = np.cumsum(inc[r], axis=0)
    return g, 1.0 / (1.0 + np.exp(-b))


def gates_bwd(a, b, a_log, dt_bias, cu, dg, dbeta, chunk=64):
    """da, db of gates_fwd (reference src/adjoint/host/gdn_prep.cpp:467-488)."""
    tail = np.zeros_like(dg)
    for s in range(len(cu) - 1):
        for c0 in range(cu[s], cu[s + 1], chunk):
            r = slice(c0, min(cu[s + 1], c0 + chunk))
            tail[r] = np.cumsum(dg[r][::-1], axis=0)[::-1]
    av = a + dt_bias[None, :]
    sp = np.where(av > 20.0, 1.0, 1.0 / (1.0 + np.exp(-av)))
    sb = 1.0 / (1.0 + np.exp(-b))
    return tail * (-np.exp(a_log))[None, :] * sp, dbeta * sb * (1.0 - sb)


# ----------------------------------------------------------------------------- gated attention

def rope_fwd(x, positions, rotary_dim, theta, head_dim, scale=1.0):
    """Partial NeoX rotary embedding of every head of x [T, heads * head_dim]: within each head the pairs
    (i, i + rotary_dim/2), i < rotary_dim/2, turn by position * theta^(-2i/rotary_dim); the columns past
    rotary_dim pass through (reference src/adjoint/host/qk.cpp:54-112, rope.cpp:72-90)."""
    T = x.shape[0]
    xh = x.reshape(T, -1, head_dim)
    half = rotary_dim // 2
    inv = theta ** (-2.0 * np.arange(half) / rotary_dim)
    ang = (np.asarray(positions, np.float64) / scale)[:, None] * inv[None, :]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    out = xh.copy()
    x0, x1 = xh[..., :half], xh[..., half:rotary_dim]
    out[..., :half] = x0 * c - x1 * s
    out[..., half:rotary_dim] = x0 * s + x1 * c
    return out.reshape(x.shape)


def rope_bwd(dy, positions, rotary_dim, theta, head_dim, scale=1.0):
    """The transposed rotation (reference src/adjoint/host/qk.cpp:114-150, rope.cpp:92-106)."""
    T = dy.shape[0]
    dh = dy.reshape(T, -1, head_dim)
    half = rotary_dim // 2
    inv = theta ** (-2.0 * np.arange(half) / rotary_dim)
    ang = (np.asarray(positions, np.float64) / scale)[:, None] * inv[None, :]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    out = dh.copy()
    y0, y1 = dh[..., :half], dh[..., half:rotary_dim]
    out[..., :half] = c * y0 + s * y1
    out[..., half:rotary_dim] = -s * y0 + c * y1
    return out.reshape(dy.shape)


def _attn_rows(cu, T):
    return [(int(cu[i]), int(cu[i + 1])) for i in range(len(cu) - 1)] if cu is not None else [(0, T)]


def attention_fwd(q, k, v, scale=None, cu=None):
    """Causal grouped-query softmax attention per sequence: q [T, Hq, D], k, v [T, Hkv, D], query head h
    reads key/value head h // (Hq / Hkv); out[t, h] = sum_{j <= t} softmax_j(scale q_t . k_j) v_j (reference
    src/adjoint/host/attention.cpp:261-313, the `attn_paged` twin over a pool that holds each sequence's
    keys at their positions)."""
    T, Hq, D = q.shape
    grp = Hq // k.shape[1]
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    out = np.zeros_like(q, dtype=np.float64)
    for a, b in _attn_rows(cu, T):
        n = b - a
        mask = np.triu(np.ones((n, n), bool), 1)
        for h in range(Hq):
            s = (q[a:b, h] @ k[a:b, h // grp].T) * scale
            s = np.where(mask, -np.inf, s)
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            out[a:b, h] = p @ v[a:b, h // grp]
    return out


def attention_bwd(q, k, v, dy, scale=None, cu=None):
    """The adjoint: with p the row's weights and G_j = dy . v_j, ds_j = p_j (G_j - sum_k p_k G_k); dq = scale
    ds k, dk = scale ds^T q, dv = p^T dy, the key/value cotangents summed over the query heads of a group
    (reference src/adjoint/host/attention.cpp:322-407)."""
    T, Hq, D = q.shape
    grp = Hq // k.shape[1]
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    dq, dk, dv = np.zeros_like(q, np.float64), np.zeros_like(k, np.float64), np.zeros_like(v, np.float64)
    for a, b in _attn_rows(cu, T):
        n = b - a
        mask = np.triu(np.ones((n, n), bool), 1)
        for h in range(Hq):
            kh = h // grp
            s = (q[a:b, h] @ k[a:b, kh].T) * scale
            s = np.where(mask, -np.inf, s)
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            G = dy[a:b, h] @ v[a:b, kh].T
            ds = p * (G - (p * G).sum(-1, keepdims=True))
            dq[a:b, h] += scale * ds @ k[a:b, kh]
            dk[a:b, kh] += scale * ds.T @ q[a:b, h]
            dv[a:b, kh] += p.T @ dy[a:b, h]
    return dq, dk, dv


def gate_fwd(o, gate):
    """The attention output gate: o * sigmoid(gate) (reference elementwise.cpp `sigmoid` then `mul`,
    :234-242 and :169-183)."""
    return o * _sigmoid(gate)


def gate_bwd(o, gate, dy):
    """d o = dy sigmoid(gate); d gate = dy o s (1 - s) (reference elementwise.cpp:185-251)."""
    s = _sigmoid(gate)
    return dy * s, dy * o * s * (1.0 - s)
