"""The chunked GatedDeltaNet recurrence (kkt solve + chunk scan) on the GPU, through the C ABI.

``GdnPlan`` holds one call's geometry: the ragged sequence table (cu_seqlens) turned into the chunk
table the kernels index, on the device. ``forward`` returns the output, the final state and the saved
tensors the backward reads; ``backward`` returns the input cotangents, with the kkt solve's adjoint
already composed in (reference: gdn_kkt_solve + gdn_chunk_scan, src/adjoint/host/gdn_kkt.cpp and
gdn_scan.cpp).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from ._lib import R97bError, check, lib

c_vp = ctypes.c_void_p


class R97bGdnDims(ctypes.Structure):
    _fields_ = [("n_seq", ctypes.c_int32), ("H", ctypes.c_int32), ("Hg", ctypes.c_int32),
                ("n_chunks", ctypes.c_int32), ("head_k", ctypes.c_int32), ("head_v", ctypes.c_int32),
                ("chunk", ctypes.c_int32), ("flags", ctypes.c_int32), ("T", ctypes.c_int64),
                ("scale", ctypes.c_float), ("_pad2", ctypes.c_int32), ("chunk_tok0", c_vp),
                ("chunk_len", c_vp), ("seq_chunk0", c_vp)]


class R97bGdnFwd(ctypes.Structure):
    _fields_ = [(n, c_vp) for n in ("q", "k", "v", "g", "beta", "h0", "A", "w", "u", "S", "Vp", "P", "o", "ht")]


class R97bGdnBwd(ctypes.Structure):
    _fields_ = [(n, c_vp) for n in ("q", "k", "v", "g", "beta", "A", "w", "S", "Vp", "P", "dO", "dht", "dS", "dVp",
                                     "dw", "pdq", "pdk", "pdg", "dq", "dk", "dv", "dbeta", "dg", "dh0", "dA")]


def _p(t):
    return None if t is None else t.data_ptr()


class GdnPlan:
    """Chunk table of a ragged batch (cu_seqlens, host ints) for H value heads over Hg key heads."""

    def __init__(self, cu_seqlens, H: int, Hg: int, device, scale: float | None = None, K: int = 128):
        cu = np.ascontiguousarray(np.asarray(cu_seqlens, dtype=np.int32))
        n_seq = len(cu) - 1
        T = int(cu[-1])
        n = int(lib().r97b_gdn_chunk_table(cu.ctypes.data, n_seq, 64, None, None, None))
        if n < 0:
            raise R97bError("bad cu_seqlens")
        tok0 = np.zeros(max(n, 1), np.int32)
        ln = np.zeros(max(n, 1), np.int32)
        sc0 = np.zeros(n_seq + 1, np.int32)
        lib().r97b_gdn_chunk_table(cu.ctypes.data, n_seq, 64, tok0.ctypes.data, ln.ctypes.data, sc0.ctypes.data)
        self.n_seq, self.T, self.H, self.Hg, self.n_chunks = n_seq, T, H, Hg, n
        self.device = device
        self.tok0 = torch.from_numpy(tok0).to(device)
        self.len = torch.from_numpy(ln).to(device)
        self.seq_c0 = torch.from_numpy(sc0).to(device)
        self.dims = R97bGdnDims(n_seq, H, Hg, n, K, K, 64, 0, T, scale if scale is not None else 1.0 / math.sqrt(K),
                                0, self.tok0.data_ptr(), self.len.data_ptr(), self.seq_c0.data_ptr())

    def _f32(self, *shape):
        return torch.empty(shape, dtype=torch.float32, device=self.device)

    def forward(self, q, k, v, g, beta, h0=None, want_ht=False, out=None, stream=None):
        T, H, n = self.T, self.H, self.n_chunks
        sv = dict(q=q, k=k, v=v, g=g, beta=beta, h0=h0)
        sv["A"] = self._f32(T, H, 64)
        sv["w"] = self._f32(T, H, 128)
        u = self._f32(T, H, 128)
        sv["S"] = self._f32(max(n, 1), H, 128, 128)
        sv["Vp"] = self._f32(T, H, 128)
        sv["P"] = self._f32(max(n, 1), H, 64, 64)
        o = torch.empty((T, H, 128), dtype=torch.bfloat16, device=self.device) if out is None else out
        ht = self._f32(self.n_seq, H, 128, 128) if want_ht else None
        a = R97bGdnFwd(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(h0), _p(sv["A"]), _p(sv["w"]), _p(u), _p(sv["S"]),
                       _p(sv["Vp"]), _p(sv["P"]), _p(o), _p(ht))
        s = (stream or torch.cuda.current_stream()).cuda_stream
        check(lib().r97b_gdn_fwd(ctypes.byref(self.dims), ctypes.byref(a), c_vp(s)), "r97b_gdn_fwd")
        return o, ht, sv

    def backward(self, sv, dO, dht=None, want_dh0=False, stream=None, sum_heads=True):
        T, H, n = self.T, self.H, self.n_chunks
        dS = self._f32(max(n, 1), H, 128, 128)
        dVp, dw = (self._f32(T, H, 128) for _ in range(2))
        dq, dk, dv = (self._f32(T, H, 128) for _ in range(3))
        dbeta, dg = self._f32(T, H), self._f32(T, H)
        dh0 = self._f32(self.n_seq, H, 128, 128) if want_dh0 else None
        a = R97bGdnBwd(_p(sv["q"]), _p(sv["k"]), _p(sv["v"]), _p(sv["g"]), _p(sv["beta"]), _p(sv["A"]), _p(sv["w"]),
                       _p(sv["S"]), _p(sv["Vp"]), _p(sv["P"]), _p(dO), _p(dht), _p(dS), _p(dVp), _p(dw), None,
                       None, None, _p(dq), _p(dk), _p(dv), _p(dbeta), _p(dg), _p(dh0))
        s = (stream or torch.cuda.current_stream()).cuda_stream
        check(lib().r97b_gdn_bwd(ctypes.byref(self.dims), ctypes.byref(a), c_vp(s)), "r97b_gdn_bwd")
        if sum_heads and self.H != self.Hg:
            dq2, dk2 = self._f32(T, self.Hg, 128), self._f32(T, self.Hg, 128)
            check(lib().r97b_gdn_sum_heads(_p(dq), _p(dq2), T, H, self.Hg, c_vp(s)), "r97b_gdn_sum_heads")
            check(lib().r97b_gdn_sum_heads(_p(dk), _p(dk2), T, H, self.Hg, c_vp(s)), "r97b_gdn_sum_heads")
            dq, dk = dq2, dk2
        return dict(dq=dq, dk=dk, dv=dv, dbeta=dbeta, dg=dg, dh0=dh0)
