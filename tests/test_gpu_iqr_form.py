"""The whole-weight device decode from an encoding's planes (r97b_iqr_decode_planes, csrc/iqr_form.cu) against
the reference's form test (tests/host/iqr_form.cpp): codes bit-identical to the oracle's host decode of the
same description, the stored scale the plane's own bits, and the scale.col fold the description cannot carry
-- bf16(row f32 x the block's factor), one rounding -- bit for bit; a bf16 block scale beside scale.col is
refused."""
import numpy as np
import pytest
import torch

from r97training_b200 import iqr as I
from tests.iqr_encodings import _bf16_bits, affine_form, bf16_form, host_decode, trunk_form

pytestmark = pytest.mark.gpu
ROWS, COLS = 512, 256


def _dev(planes, cuda):
    return [None if p is None else torch.from_numpy(p.copy()).to(cuda) for p in planes]


def _decode(e, p, rows, cols, cuda):
    out = I.decode_planes(e, _dev(p, cuda), rows, cols)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("with_scale_col", [True, False])
def test_trunk_form_decodes_on_device(cuda, with_scale_col):
    e, p = trunk_form(ROWS, COLS, with_scale_col=with_scale_col)
    codes, scale = _decode(e, p, ROWS, COLS, cuda)
    want_c, want_s = host_decode(I.desc_from_planes(e, p, ROWS, COLS), ROWS, COLS)
    assert np.array_equal(codes.cpu().numpy(), want_c)
    got_s = scale.cpu().numpy().view(np.uint16)
    if with_scale_col:
        row = p[e.index("scale")].view(np.float32)
        factor = p[e.index("scale.col")].view(np.float32)
        want = _bf16_bits((row[:, None] * factor[None, :]).astype(np.float32))
        assert np.array_equal(got_s, want)  # bf16(row x factor), one rounding
        assert got_s[0, 0] != _bf16_bits(row[:1])[0]  # the factor is not a no-op at these values
    else:
        assert np.array_equal(got_s, want_s)


def test_bf16_form_decodes_on_device(cuda):
    e, p = bf16_form(ROWS, COLS)
    codes, scale = _decode(e, p, ROWS, COLS, cuda)
    want_c, _ = host_decode(I.desc_from_planes(e, p, ROWS, COLS), ROWS, COLS)
    assert np.array_equal(codes.cpu().numpy(), want_c)
    assert np.array_equal(scale.cpu().numpy().view(np.uint8).reshape(-1), p[e.index("scale")])


def test_affine_form_decodes_on_device(cuda):
    e, p = affine_form(256, COLS)
    codes, _ = _decode(e, p, 256, COLS, cuda)
    r, j = np.meshgrid(np.arange(256), np.arange(COLS), indexing="ij")
    assert np.array_equal(codes.cpu().numpy().astype(np.int64), ((r * 5 + j * 3) & 15) - (j // 128 + 1))


def test_bf16_block_scale_beside_scale_col_is_refused(cuda):
    e, p = bf16_form(256, COLS)
    e.add_plane("scale.col", I.ENC_F32, 0, 128)
    p.append(np.zeros(COLS // 128 * 4, np.uint8))
    assert _decode(e, p, 256, COLS, cuda) is None
