"""The encodings of the reference's form test (tests/host/iqr_form.cpp:54-190), built plane by plane with the
same contents: the trunk form (u6 codes, one f32 scale a row, a 2^16-state trellis table with a 256-row run,
the computed codebook's A and B, the per-128 factor scale.col), the stored bf16 form (a bf16 scale a 128
columns), and the affine grid (u4 codes, a u8 zero and a bf16 scale a 128 columns). Planes are numpy byte
arrays; a test moves them to the device for the decode."""
import numpy as np

from r97training_b200 import iqr as I


def _bf16_bits(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def _alloc(enc, rows, cols):
    return [np.zeros(enc.plane_bytes(i, rows, cols), np.uint8) for i in range(enc.c.n_planes)]


def trunk_form(rows, cols, with_mad=True, with_scale_col=True):
    nkb = cols // 128
    e = I.Encoding()
    e.add_plane("codes", I.ENC_U(6), 1, 1)
    e.add_plane("scale", I.ENC_F32, 1, 0)
    it = e.add_table("trellis", I.ENC_I8, 65536, 1)
    e.c.plane[it].block[0], e.c.plane[it].block[1] = 256, 1
    if with_mad:
        e.add_table("trellis.mad", I.ENC_U32, 2, 1)
    if with_scale_col:
        e.add_plane("scale.col", I.ENC_F32, 0, 128)
    p = _alloc(e, rows, cols)
    p[it][:] = ((np.arange(p[it].size) * 37 + 11) & 0xFF).astype(np.uint8)
    if with_mad:
        p[e.index("trellis.mad")][:] = np.array([0x00ABCDEF, 7], np.uint32).view(np.uint8)
    rb = I.enc_row_bytes(I.ENC_U(6), cols)
    codes = p[0].reshape(rows, rb)
    r, j = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
    v = ((r * 13 + j * 7) % 64).astype(np.uint32)
    o = j * 6
    np.bitwise_or.at(codes, (r, o >> 3), ((v << (o & 7)) & 0xFF).astype(np.uint8))
    spill = (o & 7) + 6 > 8
    np.bitwise_or.at(codes, (r[spill], (o[spill] >> 3) + 1), (v[spill] >> (8 - (o[spill] & 7))).astype(np.uint8))
    p[e.index("scale")][:] = (0.0001 * (np.arange(rows) + 1)).astype(np.float32).view(np.uint8)
    if with_scale_col:
        p[e.index("scale.col")][:] = (2.0 + np.arange(nkb)).astype(np.float32).view(np.uint8)
    return e, p


def bf16_form(rows, cols):
    nkb = cols // 128
    e = I.Encoding()
    e.add_plane("codes", I.ENC_U(6), 1, 1)
    e.add_plane("scale", I.ENC_BF16, 1, 128)
    it = e.add_table("trellis", I.ENC_I8, 65536, 1)
    e.c.plane[it].block[0], e.c.plane[it].block[1] = 256, 1
    e.add_table("trellis.mad", I.ENC_U32, 2, 1)
    p = _alloc(e, rows, cols)
    p[it][:] = ((np.arange(p[it].size) * 29 + 5) & 0xFF).astype(np.uint8)
    p[e.index("scale")][:] = _bf16_bits(0.5 + 0.25 * np.arange(rows * nkb)).view(np.uint8)
    return e, p


def affine_form(rows, cols):
    nkb = cols // 128
    e = I.Encoding()
    e.add_plane("codes", I.ENC_U(4), 1, 1)
    e.add_plane("scale", I.ENC_BF16, 1, 128)
    e.add_plane("zero", I.ENC_U(8), 1, 128)
    p = _alloc(e, rows, cols)
    r, j = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
    v = ((r * 5 + j * 3) & 15).astype(np.uint8)
    codes = p[0].reshape(rows, cols // 2)
    np.bitwise_or.at(codes, (r, j >> 1), (v << ((j & 1) * 4)).astype(np.uint8))
    p[e.index("zero")].reshape(rows, nkb)[:] = (np.arange(nkb) + 1).astype(np.uint8)[None, :]
    p[e.index("scale")][:] = _bf16_bits(0.125 * (np.arange(rows * nkb) + 1)).view(np.uint8)
    return e, p


def host_decode(desc, rows, cols):
    """The oracle's C restatement of the decode on a description over host planes."""
    import ctypes
    from oracle import oracle_lib
    codes = np.zeros((rows, cols), np.int8)
    scale = np.zeros((rows, cols // 128), np.uint16)
    desc.out_codes, desc.out_scale = codes.ctypes.data, scale.ctypes.data
    assert oracle_lib().oracle_iqr_decode(ctypes.byref(desc)) == 0
    return codes, scale
