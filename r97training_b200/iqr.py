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

from ._lib import R97bEncoding, R97bStoredPlane, R97IqrDecodeDesc, check, lib

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


# ------------------------------------------------------------------------------- encodings -> descriptions
# The container's encoding of a stored weight (radiance's RadEncoding; here its fields the derivation reads)
# and the planes it names, turned into the decode's description by r97b_iqr_desc_from_planes (the reference's
# src/iqr_form.h). Element types: ENC_U(bits) packed codes, ENC_I8, ENC_U32, ENC_F32, ENC_BF16, ENC_F16,
# ENC_F8E4M3.
ENC_I8, ENC_U32, ENC_F32, ENC_BF16, ENC_F16, ENC_F8E4M3 = 20, 21, 30, 31, 32, 33


def ENC_U(bits: int) -> int:
    return bits


def enc_bits(dtype: int) -> int:
    if 1 <= dtype <= 12:
        return dtype
    return {ENC_I8: 8, ENC_F8E4M3: 8, ENC_BF16: 16, ENC_F16: 16, ENC_F32: 32, ENC_U32: 32}[dtype]


def enc_row_bytes(dtype: int, n: int) -> int:
    """Bytes of a stored row of n elements: packed bits, rounded up to a byte."""
    return (n * enc_bits(dtype) + 7) // 8


class Encoding:
    """An encoding under construction: planes (an element a block[0] rows x block[1] columns of the weight,
    0 = the whole extent) and tables (extent[0] x extent[1] elements)."""

    def __init__(self):
        self.c = R97bEncoding()
        self.c.n_planes = 0

    def _add(self, role, dtype):
        i = self.c.n_planes
        if i >= 8:
            raise ValueError("an encoding holds at most 8 planes")
        p = self.c.plane[i]
        p.role = role.encode()
        p.dtype = dtype
        self.c.n_planes = i + 1
        return i

    def add_plane(self, role, dtype, block_rows, block_cols):
        i = self._add(role, dtype)
        self.c.plane[i].block[0], self.c.plane[i].block[1] = block_rows, block_cols
        return i

    def add_table(self, role, dtype, n0, n1):
        i = self._add(role, dtype)
        self.c.plane[i].extent[0], self.c.plane[i].extent[1] = n0, n1
        return i

    def index(self, role):
        for i in range(self.c.n_planes):
            if self.c.plane[i].role.decode() == role:
                return i
        return -1

    def plane_shape(self, i, rows, cols):
        """(stored rows, elements a stored row) of plane i over a [rows, cols] weight."""
        p = self.c.plane[i]
        if p.extent[0] > 0:
            return 1, p.extent[0] * max(1, p.extent[1])
        prows = 1 if p.block[0] == 0 else -(-rows // p.block[0])
        pcols = 1 if p.block[1] == 0 else -(-cols // p.block[1])
        return prows, pcols

    def plane_bytes(self, i, rows, cols):
        prows, pcols = self.plane_shape(i, rows, cols)
        return prows * enc_row_bytes(self.c.plane[i].dtype, pcols)


def stored_planes(planes):
    """A ctypes array of R97bStoredPlane over host numpy arrays or device torch tensors (None: not held)."""
    arr = (R97bStoredPlane * max(1, len(planes)))()
    for i, p in enumerate(planes):
        if p is None:
            continue
        if isinstance(p, torch.Tensor):
            arr[i].data, arr[i].bytes = p.data_ptr(), p.numel() * p.element_size()
        else:
            arr[i].data, arr[i].bytes = p.ctypes.data, p.nbytes
    return arr


def desc_from_planes(enc: Encoding, planes, rows: int, cols: int, on_device: bool = False):
    """The decode's description derived from the encoding's planes, or None when it is refused."""
    d = R97IqrDecodeDesc()
    rc = lib().r97b_iqr_desc_from_planes(ctypes.byref(enc.c), stored_planes(planes), rows, cols,
                                         1 if on_device else 0, ctypes.byref(d))
    return d if rc == 0 else None


def decode_planes(enc: Encoding, planes, rows: int, cols: int, stream=None):
    """The whole weight decoded on the device from its device planes: (int8 codes [rows, cols], bf16-bit
    scale [rows, cols / 128] as int16), or None when the encoding is refused."""
    dev = next(p.device for p in planes if p is not None)
    codes = torch.empty((rows, cols), dtype=torch.int8, device=dev)
    scale = torch.empty((rows, cols // 128), dtype=torch.int16, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream if stream is None else stream
    rc = lib().r97b_iqr_decode_planes(ctypes.byref(enc.c), stored_planes(planes), rows, cols,
                                      ctypes.c_void_p(codes.data_ptr()), ctypes.c_void_p(scale.data_ptr()),
                                      ctypes.c_void_p(s))
    return (codes, scale) if rc == 0 else None
