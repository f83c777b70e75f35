"""The stored form derived from an encoding (r97b_iqr_desc_from_planes, csrc/iqr_form.cu) against the reference's
own form test, tests/host/iqr_form.cpp: which plane is what, the trellis's state count and run, the scale's
layout, the computed codebook and its rounding, the affine grid, and every refusal that test names. The
derived description then decodes through the oracle's C restatement (and, where the reference's host decode is
built, through it) with the same codes. CPU only: the planes are host memory."""
import ctypes

import numpy as np
import pytest

import oracle
from r97training_b200 import iqr as I
from tests.iqr_encodings import affine_form, bf16_form, host_decode, trunk_form

ROWS, COLS = 512, 256


def test_trunk_form_description():
    e, p = trunk_form(ROWS, COLS)
    d = I.desc_from_planes(e, p, ROWS, COLS)
    assert d is not None
    assert d.bits == 6 and d.state_bits == 16 and d.run_rows == 256 and d.rb == 1
    assert d.mad == 1 and d.round_mad == 1
    assert (d.mad_a, d.mad_b) == (0x00ABCDEF, 7)
    assert d.scale_dtype == 0 and d.scale_block_cols == 0 and d.scale_row_bytes == 4
    assert not d.scale2 and d.affine == 0
    assert d.codes_row_bytes == COLS * 6 // 8
    codes, scale = host_decode(d, ROWS, COLS)
    assert codes.min() >= -127 and codes.max() <= 127 and np.abs(codes).sum() > 0
    if oracle.ref_available():  # the reference's own host decode of the same description
        c2 = np.zeros_like(codes)
        s2 = np.zeros_like(scale)
        d.out_codes, d.out_scale = c2.ctypes.data, s2.ctypes.data
        assert oracle.ref_lib().ref_iqr_decode(ctypes.byref(d)) == 0
        assert np.array_equal(c2, codes) and np.array_equal(s2, scale)


def test_rounding_follows_mad_or_scale_col():
    e, p = trunk_form(ROWS, COLS, with_mad=True, with_scale_col=False)
    d = I.desc_from_planes(e, p, ROWS, COLS)
    assert d is not None and d.round_mad == 1  # a computed codebook rounds without scale.col too
    e, p = trunk_form(ROWS, COLS, with_mad=False, with_scale_col=True)
    d = I.desc_from_planes(e, p, ROWS, COLS)
    assert d is not None and d.mad == 0 and d.round_mad == 1  # scale.col makes a stored codebook round
    assert d.lut  # the stored codebook is the trellis table


def test_bf16_form_description():
    e, p = bf16_form(ROWS, COLS)
    d = I.desc_from_planes(e, p, ROWS, COLS)
    assert d is not None
    assert d.scale_dtype == 1 and d.scale_block_cols == 128 and d.scale_row_bytes == (COLS // 128) * 2
    assert d.affine == 0 and not d.scale2
    codes, scale = host_decode(d, ROWS, COLS)
    assert np.array_equal(scale.view(np.uint8).reshape(-1), p[e.index("scale")])  # the plane's own bits
    assert codes.min() >= -127 and codes.max() <= 127


def test_affine_form_description():
    rows = 256
    e, p = affine_form(rows, COLS)
    d = I.desc_from_planes(e, p, rows, COLS)
    assert d is not None
    assert d.affine == 1 and d.bits == 4 and d.zero_bits == 8 and d.zero_row_bytes == COLS // 128
    assert d.run_rows == 1 and d.rb == 1 and not d.scale2
    codes, _ = host_decode(d, rows, COLS)
    r, j = np.meshgrid(np.arange(rows), np.arange(COLS), indexing="ij")
    want = ((r * 5 + j * 3) & 15) - (j // 128 + 1)
    assert np.array_equal(codes.astype(np.int64), want)  # every code is its stored code less the block's zero


def test_refusals():
    e, p = trunk_form(256, COLS)
    e.c.n_planes = 2  # codes and scale only: no trellis and no zero
    assert I.desc_from_planes(e, p, 256, COLS) is None
    e, p = trunk_form(256, COLS)
    e.c.plane[e.index("trellis")].extent[0] = 1000  # not a power of two
    assert I.desc_from_planes(e, p, 256, COLS) is None
    e, p = trunk_form(256, COLS)
    p[0] = p[0][: p[0].size // 2]  # a codes plane shorter than the weight
    assert I.desc_from_planes(e, p, 256, COLS) is None
    e, p = trunk_form(256, COLS)
    assert I.desc_from_planes(e, p, 256, 250) is None  # a column count the decode does not tile
    e, p = affine_form(256, COLS)
    e.add_table("trellis", I.ENC_I8, 65536, 1)  # zero and trellis together
    p.append(np.zeros(65536, np.uint8))
    assert I.desc_from_planes(e, p, 256, COLS) is None
    e, p = trunk_form(256, COLS)
    p[e.index("trellis.mad")] = None  # a computed codebook whose A and B are not held
    assert I.desc_from_planes(e, p, 256, COLS) is None
    e, p = trunk_form(256, COLS)
    assert oracle is not None and I.lib().r97b_iqr_desc_from_planes(None, I.stored_planes(p), 256, COLS, 0,
                                                                    ctypes.byref(I.R97IqrDecodeDesc())) == 1


@pytest.mark.parametrize("second", [False, True])
def test_second_scale_level(second):
    """A scale.1 plane (one f32 for the weight) becomes the description's second level."""
    e, p = trunk_form(256, COLS, with_scale_col=False)
    if second:
        e.add_plane("scale.1", I.ENC_F32, 0, 0)
        p.append(np.array([1.5], np.float32).view(np.uint8))
    d = I.desc_from_planes(e, p, 256, COLS)
    assert d is not None
    assert bool(d.scale2) == second
    if second:
        assert d.scale2_dtype == 0 and d.scale2_block_rows == 0 and d.scale2_block_cols == 0
