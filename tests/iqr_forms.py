"""Synthetic stored IQR weights in every form the decode accepts, for the parity tests.

Mirrors the coverage of the reference's own decode test (reference tests/host/iqr_decode.cpp:82-213,
236-320, 465-492): computed and stored codebooks, f32 / bf16 / e4m3 / f16 scales, a second scale
level, tcq_rb row blocks, a short last run, a chunk that starts at a run boundary, the affine grid.
"""
import numpy as np


def _pack(vals: np.ndarray, bits: int) -> np.ndarray:
    rows, cols = vals.shape
    row_bytes = (cols * bits + 7) // 8
    out = np.zeros((rows, row_bytes + 4), np.uint8)  # slack so multi-byte reads stay in bounds
    for j in range(cols):
        bit = j * bits
        for b in range(bits):
            on = (vals[:, j] >> b) & 1
            out[:, (bit + b) >> 3] |= (on << ((bit + b) & 7)).astype(np.uint8)
    return out


def _scale_plane(rs, rows, groups, dtype):
    v = np.abs(rs.normal(0.0, 0.02, size=(rows, groups))).astype(np.float32)
    if dtype == 0:
        return v.view(np.uint8).reshape(rows, -1)
    if dtype == 1:
        u = v.view(np.uint32)
        b = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        return b.view(np.uint8).reshape(rows, -1)
    if dtype == 2:  # e4m3: random finite positive bytes (not the NaN 0x7F)
        b = rs.randint(0x08, 0x78, size=(rows, groups)).astype(np.uint8)
        return b.reshape(rows, -1)
    if dtype == 3:
        return v.astype(np.float16).view(np.uint8).reshape(rows, -1)
    raise ValueError(dtype)


def make_form(seed=0, rows=512, cols=256, bits=4, state_bits=16, run_rows=256, rb=1, mad=True, scale_dtype=0,
              rowf=False, second=False, affine=False, round_mad=0):
    rs = np.random.RandomState(seed)
    codes = rs.randint(0, 1 << bits, size=(rows, cols)).astype(np.int64)
    form = dict(rows_all=rows, cols=cols, bits=bits, state_bits=state_bits, run_rows=run_rows, rb=rb,
                mad=int(mad), round_mad=round_mad, scale_dtype=scale_dtype, scale_block_cols=cols if rowf else 128)
    form["codes"] = _pack(codes, bits)
    groups = 1 if rowf else cols // 128
    form["scale"] = _scale_plane(rs, rows, groups, scale_dtype)
    if affine:
        form.update(affine=1, run_rows=1, rb=1, mad=0)
        zb = 8
        z = rs.randint(0, 1 << (bits - 1), size=(rows, groups)).astype(np.int64)
        form["zero"] = _pack(z, zb)
        form["zero_bits"] = zb
        return form
    if mad:
        form["mad_a"] = int(rs.randint(0, 2 ** 31)) & 0xFFFFFF | 1
        form["mad_b"] = int(rs.randint(0, 2 ** 31)) * 2 + 1
    else:
        form["lut"] = rs.randint(-127, 128, size=(1 << state_bits,)).astype(np.int8)
    if second:
        form["scale2"] = np.array([1.7], np.float32).view(np.uint8)
        form["scale2_dtype"] = 0
    return form


FORMS = [
    dict(),                                     # the trunk form (u4, L16, mad, f32 scales)
    dict(scale_dtype=1),                        # bf16 scales
    dict(scale_dtype=2, second=True),           # e4m3 + scale.1
    dict(scale_dtype=3),                        # f16 scales
    dict(mad=False, state_bits=12, bits=3),     # stored LUT, u3
    dict(bits=5, state_bits=15),
    dict(bits=6, state_bits=18, run_rows=128),
    dict(rb=2, run_rows=256),                   # tcq_rb blocks
    dict(rb=4, run_rows=128, round_mad=1),
    dict(rows=300),                             # a short last run (44 rows)
    dict(rowf=True),                            # one scale a row (scale.col form)
    dict(affine=True, bits=4),                  # the affine grid
    dict(cols=384, rows=640, seed=7),
]
