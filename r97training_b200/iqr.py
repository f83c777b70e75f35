"""Stored IQR weights: the synthetic trunk form of the configs, and the decode entry points.

The trunk form (u4 codes, 16 state bits, runs of 256 rows, rb 1, computed "mad" codebook, one f32
scale per row and 128 columns, no second level, no transform) follows the reference's trunk-like test
form (reference tests/host/iqr_decode.cpp:82-213, 465-472): codes are uniform random bits, the mad
constants A = (rand & 0xFFFFFF) | 1 and B = rand, the scales |N(0, 0.02)|.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import R97IqrDecodeDesc, check, lib

R97_IQR_F32, R97_IQR_BF16, R97_IQR_F8E4M3, R97_IQR_F16 = 0, 1, 2, 3


@dataclass
class IqrWeight:
    """One stored weight [rows, cols] in the trunk form. Tensors live on one device (CPU or CUDA)."""
    rows: int
    cols: int
    codes: torch.Tensor      # uint8 [rows, cols * bits / 8], codes packed lowest bits first
    scale: torch.Tensor      # float32 [rows, cols / 128]
    mad_a: int
    mad_b: int
    bits: int = 4
    state_bits: int = 16
    run_rows: int = 256

    def to(self, device) -> "IqrWeight":
        return IqrWeight(self.rows, self.cols, self.codes.to(device), self.scale.to(device), self.mad_a, self.mad_b,
                         self.bits, self.state_bits, self.run_rows)

    @property
    def nbytes(self) -> int:
        return self.codes.numel() + self.scale.numel() * 4


def synth_weight(rows: int, cols: int, seed: int, device="cpu", scale_std: float = 0.02) -> IqrWeight:
    """A seeded synthetic IQR weight (trunk form). Generated with numpy on CPU for small weights and
    torch's generator on the target device for large ones; the same (rows, cols, seed) always gives the
    same bytes on a given path."""
    assert cols % 128 == 0
    rs = np.random.RandomState(seed & 0x7FFFFFFF)
    a = int(rs.randint(0, 2**31)) & 0xFFFFFF | 1
    b = int(rs.randint(0, 2**31)) * 2 + int(rs.randint(0, 2))
    b &= 0xFFFFFFFF
    if rows * cols <= (1 << 26) or str(device) == "cpu":
        codes = torch.from_numpy(rs.randint(0, 256, size=(rows, cols // 2), dtype=np.uint8))
        scale = torch.from_numpy(np.abs(rs.normal(0.0, scale_std, size=(rows, cols // 128))).astype(np.float32))
        return IqrWeight(rows, cols, codes.to(device), scale.to(device), a, b)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    codes = torch.randint(0, 256, (rows, cols // 2), dtype=torch.uint8, device=device, generator=gen)
    scale = torch.randn((rows, cols // 128), dtype=torch.float32, device=device, generator=gen).abs_().mul_(scale_std)
    return IqrWeight(rows, cols, codes, scale, a, b)


def make_desc(w: IqrWeight, row0: int = 0, rows: int | None = None, out_codes=None, out_scale=None) -> R97IqrDecodeDesc:
    """The decode description of rows [row0, row0 + rows) of `w`, pointing at w's own buffers."""
    rows = w.rows - row0 if rows is None else rows
    d = R97IqrDecodeDesc()
    d.rows_all, d.cols, d.row0, d.rows = w.rows, w.cols, row0, rows
    d.bits, d.state_bits, d.run_rows, d.rb = w.bits, w.state_bits, w.run_rows, 1
    d.mad, d.round_mad, d.mad_a, d.mad_b = 1, 0, w.mad_a, w.mad_b
    rb = w.codes.stride(0)
    d.codes = w.codes.data_ptr() + row0 * rb
    d.codes_row_bytes = rb
    d.scale = w.scale.data_ptr() + row0 * w.scale.stride(0) * 4
    d.scale_dtype = R97_IQR_F32
    d.scale_block_cols = 128
    d.scale_row_bytes = w.scale.stride(0) * 4
    d.out_codes = None if out_codes is None else out_codes.data_ptr()
    d.out_scale = None if out_scale is None else out_scale.data_ptr()
    return d


def decode(w: IqrWeight, stream=None):
    """The reference-compatible decode on the GPU: (int8 codes [rows, cols], bf16-bit scale [rows, cols/128])."""
    codes = torch.empty((w.rows, w.cols), dtype=torch.int8, device=w.codes.device)
    scale = torch.empty((w.rows, w.cols // 128), dtype=torch.int16, device=w.codes.device)
    d = make_desc(w, out_codes=codes, out_scale=scale)
    s = (stream or torch.cuda.current_stream()).cuda_stream
    rc = lib().r97_iqr_decode(ctypes.byref(d), ctypes.c_void_p(s))
    check(rc, "r97_iqr_decode")
    return codes, scale


def dequant_bf16(w: IqrWeight, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """W = bf16(code * bf16(scale)) [rows, cols] on the GPU (the GEMM operand)."""
    if out is None:
        out = torch.empty((w.rows, w.cols), dtype=torch.bfloat16, device=w.codes.device)
    d = make_desc(w)
    s = (stream or torch.cuda.current_stream()).cuda_stream
    check(lib().r97b_iqr_dequant_bf16(ctypes.byref(d), ctypes.c_void_p(out.data_ptr()), out.stride(0),
                                      ctypes.c_void_p(s)), "r97b_iqr_dequant_bf16")
    return out
