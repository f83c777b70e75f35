"""Loads the adjoint-row plugin (libr97host.so) into this process after the reference's registry
(oracle/_ref/libr97ref.so), so its rows register there, and compares two rows' results under the
north star's tolerance."""
import ctypes
import os

import numpy as np
import pytest

import oracle
from r97training_b200 import build as B

_plugin = None


def plugin():
    """The plugin, registered into the reference registry (which is loaded first, RTLD_GLOBAL)."""
    global _plugin
    if _plugin is None:
        if not oracle.ref_available():
            pytest.skip("reference host library not built and reference tree absent")
        oracle.ref_lib()
        if not os.path.exists(B.HOSTLIB):
            B.build_all()
        lib = ctypes.CDLL(B.HOSTLIB, mode=ctypes.RTLD_GLOBAL)
        lib.r97host_registered.restype = ctypes.c_int
        lib.r97host_head_ce.restype = ctypes.c_int
        lib.r97host_grad_stage_flush.restype = ctypes.c_int
        lib.r97host_grad_stage_flush.argtypes = [ctypes.c_void_p]
        lib.r97host_sync.restype = ctypes.c_int
        _plugin = lib
    return _plugin


def flush(paramset_ptr):
    assert plugin().r97host_grad_stage_flush(ctypes.c_void_p(paramset_ptr)) == 0


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def cosine(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / max(na * nb, 1e-300))


def assert_parity(mine, ref, what, rel=1e-2, cos=0.999):
    """The north star's bar for gradients and cotangents: per-tensor relative L2 <= 1e-2 and cosine
    >= 0.999."""
    r, c = rel_l2(mine, ref), cosine(mine, ref)
    assert r <= rel and c >= cos, f"{what}: rel_l2 {r:.3e} cosine {c:.6f}"
