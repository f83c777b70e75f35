"""Helpers shared by the GPU tests: device copies of numpy IQR forms, tolerance checks."""
import numpy as np
import torch

from r97training_b200._lib import R97IqrDecodeDesc


def device_form_desc(form: dict, dev, row0=0, rows=None):
    """The product's R97IqrDecodeDesc over DEVICE copies of a numpy form's planes, plus the output
    tensors; returns (desc, out_codes, out_scale, keepalive)."""
    keep = []

    def up(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        keep.append(t)
        return t

    rows_all, cols = form["rows_all"], form["cols"]
    rows = rows_all - row0 if rows is None else rows
    d = R97IqrDecodeDesc()
    d.rows_all, d.cols, d.row0, d.rows = rows_all, cols, row0, rows
    d.bits, d.state_bits = form.get("bits", 4), form.get("state_bits", 16)
    d.run_rows, d.rb = form.get("run_rows", 256), form.get("rb", 1)
    d.mad, d.round_mad = form.get("mad", 1), form.get("round_mad", 0)
    d.mad_a, d.mad_b = form.get("mad_a", 0), form.get("mad_b", 0)
    if form.get("lut") is not None:
        d.lut = up(form["lut"]).data_ptr()
    codes = up(form["codes"])
    d.codes = codes.data_ptr() + row0 * codes.stride(0)
    d.codes_row_bytes = codes.stride(0)
    sc = up(form["scale"])
    d.scale = sc.data_ptr() + row0 * sc.stride(0)
    d.scale_dtype = form.get("scale_dtype", 0)
    d.scale_block_cols = form.get("scale_block_cols", 128)
    d.scale_row_bytes = sc.stride(0)
    d.affine = form.get("affine", 0)
    if form.get("zero") is not None:
        z = up(form["zero"])
        d.zero = z.data_ptr() + row0 * z.stride(0)
        d.zero_row_bytes = z.stride(0)
        d.zero_bits = form.get("zero_bits", 8)
    if form.get("scale2") is not None:
        s2 = up(form["scale2"])
        d.scale2 = s2.data_ptr()
        d.scale2_dtype = form.get("scale2_dtype", 0)
        d.scale2_row_bytes = s2.numel()
        d.scale2_block_rows = form.get("scale2_block_rows", 0)
        d.scale2_block_cols = form.get("scale2_block_cols", 0)
    oc = torch.zeros((rows, cols), dtype=torch.int8, device=dev)
    os_ = torch.zeros((rows, cols // 128), dtype=torch.int16, device=dev)
    d.out_codes, d.out_scale = oc.data_ptr(), os_.data_ptr()
    return d, oc, os_, keep


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))


# The per-tensor bar of the north star for bf16 results: relative L2 <= 1e-2 and cosine >= 0.999.
REL_L2_MAX = 1e-2
COS_MIN = 0.999


def assert_close_bf16(got, want, rel=REL_L2_MAX, cos=COS_MIN, what=""):
    r, c = rel_l2(got, want), cosine(got, want)
    assert r <= rel and c >= cos, f"{what}: rel_l2={r:.3e} cos={c:.6f}"


def to_np(t):
    return t.detach().float().cpu().numpy().astype(np.float64)
