"""TEST INFRASTRUCTURE -- the CPU oracle for the LoRA-over-IQR hot path.

Only ``tests/``, ``bench.py``'s ``cpu_baseline`` leg and ``__graft_entry__.smoke()`` import this
package, and only as the checker (or the timed CPU baseline). The product path never imports it.

Two checkers live here:

* ``liboracle.so`` -- this repository's plain-C restatement of the IQR decode (``iqr_oracle.c``),
  and numpy restatements of the floating-point rows (``oracle/rows.py``). Both cite the reference
  lines they restate.
* ``_ref/libr97ref.so`` -- the reference's OWN radiance-free host rows (adjoint registry, twins and
  host adjoints, loss.cpp, optim.cpp, iqr_decode.h), compiled in place from the reference tree by
  ``oracle/Makefile`` with the flat ABI of ``ref_shim.cpp``. It pins the restatements (see
  ``tests/test_oracle_pin.py``) and is the "reference" CPU baseline.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_TREE = os.environ.get("R97_REFERENCE", "/root/reference")

_oracle = None
_ref = None


def build(ref: bool = True) -> None:
    """Builds liboracle.so, and libr97ref.so when the reference tree is present."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
    if ref and os.path.isdir(os.path.join(REF_TREE, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REF_TREE}"], check=True)


def oracle_lib():
    global _oracle
    if _oracle is None:
        path = os.path.join(HERE, "_build", "liboracle.so")
        if not os.path.exists(path):
            build(ref=False)
        lib = ctypes.CDLL(path)
        lib.oracle_iqr_decode.restype = ctypes.c_int32
        lib.oracle_iqr_validate.restype = ctypes.c_int32
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libr97ref.so")) or os.path.isdir(
        os.path.join(REF_TREE, "src"))


def ref_lib():
    """The reference's own host rows; raises when neither the built library nor the tree exists."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libr97ref.so")
        if not os.path.exists(path):
            if not os.path.isdir(os.path.join(REF_TREE, "src")):
                raise FileNotFoundError("oracle/_ref/libr97ref.so is not built and the reference tree is absent")
            build(ref=True)
        # global: a device-row plugin loaded after it binds to this registry by name
        lib = ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
        lib.ref_last_error.restype = ctypes.c_char_p
        lib.ref_iqr_decode.restype = ctypes.c_int
        lib.ref_twin.restype = ctypes.c_int
        lib.ref_adjoint.restype = ctypes.c_int
        lib.ref_adjoint_on.restype = ctypes.c_int
        lib.ref_op_rows.restype = ctypes.c_int
        lib.ref_paramset.restype = ctypes.c_void_p
        lib.ref_grad_count.restype = ctypes.c_int
        lib.ref_grad_name.restype = ctypes.c_char_p
        lib.ref_grad_numel.restype = ctypes.c_int64
        lib.ref_ce_position.restype = ctypes.c_double
        lib.ref_ce_position.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
                                        ctypes.c_double]
        lib.ref_adamw.restype = ctypes.c_int
        lib.ref_adamw.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int] + \
            [ctypes.c_float] * 6 + [ctypes.c_int] * 3
        lib.ref_scheduled_lr.restype = ctypes.c_float
        lib.ref_scheduled_lr.argtypes = [ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int]
        _ref = lib
    return _ref


# ----------------------------------------------------------------------------- generic row driver

class _RefOperand(ctypes.Structure):
    _fields_ = [("buffer", ctypes.c_char_p), ("dtype", ctypes.c_char_p), ("ndim", ctypes.c_int32),
                ("shape", ctypes.POINTER(ctypes.c_int64)), ("written", ctypes.c_int32),
                ("in_place", ctypes.c_int32), ("stored_codes", ctypes.c_void_p),
                ("stored_scale", ctypes.c_void_p)]


class _RefParam(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("is_int", ctypes.c_int32), ("ival", ctypes.c_int64),
                ("sval", ctypes.c_char_p)]


class Operand:
    """One operand of a record: its buffer name, dtype, shape, whether the op writes it, and for a
    stored IQR weight the decoded (codes int8 [N,K], scale bf16-bits uint16 [N,K/128]) pair."""

    def __init__(self, buffer, dtype, shape, written=False, in_place=False, stored=None):
        self.buffer, self.dtype, self.shape = buffer, dtype, tuple(int(s) for s in shape)
        self.written, self.in_place, self.stored = written, in_place, stored

    @property
    def numel(self):
        n = 1
        for s in self.shape:
            n *= s
        return n


def _pack(op_name, params, operands):
    keep = []
    ps = (_RefParam * max(1, len(params)))()
    for i, (k, v) in enumerate(params.items()):
        kb = k.encode()
        keep.append(kb)
        if isinstance(v, (int, np.integer)):
            ps[i] = _RefParam(kb, 1, int(v), None)
        else:
            sb = str(v).encode()
            keep.append(sb)
            ps[i] = _RefParam(kb, 0, 0, sb)
    os_ = (_RefOperand * len(operands))()
    for i, o in enumerate(operands):
        shp = (ctypes.c_int64 * max(1, len(o.shape)))(*o.shape)
        b, d = o.buffer.encode(), o.dtype.encode()
        keep += [shp, b, d]
        codes = scale = None
        if o.stored is not None:
            c = np.ascontiguousarray(o.stored[0], dtype=np.int8)
            s = np.ascontiguousarray(o.stored[1], dtype=np.uint16)
            keep += [c, s]
            codes, scale = c.ctypes.data, s.ctypes.data
        os_[i] = _RefOperand(b, d, len(o.shape), shp, int(o.written), int(o.in_place), codes, scale)
    return ps, os_, keep


def _dptrs(arrays, keep):
    arr = (ctypes.c_void_p * max(1, len(arrays)))()
    for i, a in enumerate(arrays):
        if a is None:
            arr[i] = None
        else:
            keep.append(a)
            arr[i] = a.ctypes.data
    return arr


def ref_twin(op, params, operands, reads):
    """Runs the reference twin; ``reads`` maps each read operand's buffer to an f64 array (None for a
    stored operand). Returns {written buffer: f64 array shaped as its operand}."""
    lib = ref_lib()
    ps, os_, keep = _pack(op, params, operands)
    rlist = []
    for o in operands:
        if o.written and not o.in_place:
            continue
        v = reads.get(o.buffer)
        rlist.append(None if v is None else np.ascontiguousarray(v, dtype=np.float64).reshape(-1))
    outs = [np.zeros(o.numel, np.float64) for o in operands if o.written]
    rc = lib.ref_twin(op.encode(), ps, len(params), os_, len(operands), _dptrs(rlist, keep),
                      _dptrs(outs, keep))
    if rc != 0:
        raise RuntimeError(f"ref_twin({op}) rc={rc}: {lib.ref_last_error().decode()}")
    res, w = {}, 0
    for o in operands:
        if o.written:
            res[o.buffer] = outs[w].reshape(o.shape)
            w += 1
    return res


def op_rows(op):
    """What the reference registry holds for ``op``: {"twin", "host", "device": bool, "host_frozen",
    "device_frozen": lists}."""
    lib = ref_lib()
    hf, df = (ctypes.c_int * 16)(), (ctypes.c_int * 16)()
    nh, nd = ctypes.c_int(), ctypes.c_int()
    bits = lib.ref_op_rows(op.encode(), hf, ctypes.byref(nh), df, ctypes.byref(nd))
    return {"twin": bool(bits & 1), "host": bool(bits & 2), "device": bool(bits & 4),
            "host_frozen": list(hf[:nh.value]), "device_frozen": list(df[:nd.value])}


def ref_adjoint(op, params, operands, fwd, cots, prefix="m", fused_slots=False, side="host", flush=None):
    """Runs the adjoint row the reference registry serves for ``op`` on ``side`` ("host": the reference's
    own f64 row; "device": whatever device row a loaded plugin registered). ``fwd`` maps buffer -> forward
    value (None for stored), ``cots`` maps each written buffer -> its cotangent. ``flush``, when given, is
    called with the call's ParamSet pointer before the gradients are read (a device row's gradients wait
    in its stage until flushed). Returns (dc dict, grads dict)."""
    lib = ref_lib()
    ps, os_, keep = _pack(op, params, operands)
    flist = [None if fwd.get(o.buffer) is None else np.ascontiguousarray(fwd[o.buffer], np.float64).reshape(-1)
             for o in operands]
    clist = [np.ascontiguousarray(cots[o.buffer], np.float64).reshape(-1) for o in operands if o.written]
    dcs = [np.zeros(o.numel, np.float64) for o in operands]
    pb = prefix.encode()
    rc = lib.ref_adjoint_on(op.encode(), ps, len(params), os_, len(operands), _dptrs(flist, keep),
                            _dptrs(clist, keep), _dptrs(dcs, keep), pb, int(fused_slots), int(side == "device"))
    if rc != 0:
        raise RuntimeError(f"ref_adjoint({op}, {side}) rc={rc}: {lib.ref_last_error().decode()}")
    if flush is not None:
        flush(lib.ref_paramset())
    dc = {o.buffer: dcs[i].reshape(o.shape) for i, o in enumerate(operands)}
    grads = {}
    for i in range(lib.ref_grad_count()):
        n = lib.ref_grad_numel(i)
        g = np.zeros(n, np.float32)
        lib.ref_grad_copy(i, ctypes.c_void_p(g.ctypes.data))
        grads[lib.ref_grad_name(i).decode()] = g
    return dc, grads
