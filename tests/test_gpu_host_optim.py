"""The device Optimiser of libr97host.so (r97host_optim_*) against the reference's own r97::Optimiser
(src/optim.cpp, compiled into oracle/_ref): after the same step() calls -- gradient accumulation, global-norm
clipping, warm-up and cosine schedule, weight decay skipped by name -- both serialise to the same bytes
(bit-identical weights, moments and accumulation buffer, in the reference's "R97OPT" checkpoint format),
and each restores the other's checkpoint."""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from r97training_b200 import build as B

pytestmark = pytest.mark.gpu


class AdamW(ctypes.Structure):
    _fields_ = [("lr", ctypes.c_float), ("beta1", ctypes.c_float), ("beta2", ctypes.c_float), ("eps", ctypes.c_float),
                ("weight_decay", ctypes.c_float), ("clip_norm", ctypes.c_float), ("warmup_steps", ctypes.c_int32),
                ("total_steps", ctypes.c_int32), ("lr_floor_frac", ctypes.c_float), ("accum_steps", ctypes.c_int32)]


def _host():
    if not os.path.exists(B.HOSTLIB):
        B.build_all()
    lib = ctypes.CDLL(B.HOSTLIB)
    lib.r97host_optim_create.restype = ctypes.c_void_p
    lib.r97host_optim_create.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
    lib.r97host_optim_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.r97host_optim_serialise.restype = ctypes.c_int64
    lib.r97host_optim_serialise.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    lib.r97host_optim_restore.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    lib.r97host_optim_state.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.r97host_optim_destroy.argtypes = [ctypes.c_void_p]
    lib.r97host_optim_error.restype = ctypes.c_char_p
    return lib


def _bind_ref(ref):
    f = ref.ref_optim_serialised
    f.restype = ctypes.c_int64
    f.argtypes = ([ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int] +
                  [ctypes.c_float] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64])


def _cstrs(xs):
    arr = (ctypes.c_char_p * len(xs))(*[x.encode() for x in xs])
    return arr


CASES = [
    dict(lr=2e-3, wd=0.01, clip=0.5, warmup=2, total=7, floor=0.1, accum=2, calls=10),   # clip bites, cosine
    dict(lr=1e-3, wd=0.0, clip=0.0, warmup=0, total=0, floor=0.1, accum=1, calls=3),     # plain AdamW
    dict(lr=5e-4, wd=0.1, clip=1e3, warmup=1, total=4, floor=0.0, accum=3, calls=8),     # clip never bites; ends pending
]


@pytest.mark.parametrize("case", CASES, ids=["accum2_clip_cosine", "plain", "accum3_pending"])
def test_device_optimiser_matches_reference_bytes(cuda, case):
    if not oracle.ref_available():
        pytest.skip("reference host library not built and reference tree absent")
    ref = oracle.ref_lib()
    _bind_ref(ref)
    host = _host()
    names = ["model.layers.0.q_proj.lora_A", "model.layers.0.q_proj.lora_B", "model.norm.bias",
             "model.layers.1.down_proj.lora_A"]
    counts = [5000, 3000, 257, 70000]   # one set over 65536 elements: the reference norms it on threads
    no_decay = ["bias", "norm"]
    n = sum(counts)
    rs = np.random.RandomState(17 + case["calls"])
    w0 = (rs.normal(size=n) * 0.05).astype(np.float32)
    grads = (rs.normal(size=(case["calls"], n)) * 0.02).astype(np.float32)
    grads[:, :100] *= 50.0  # a few large entries so the clip (when set) bites
    cfg = AdamW(case["lr"], 0.9, 0.999, 1e-8, case["wd"], case["clip"], case["warmup"], case["total"], case["floor"],
                case["accum"])
    # the reference
    cnt = (ctypes.c_int64 * 4)(*counts)
    args = (4, _cstrs(names), cnt, w0.ctypes.data, grads.ctypes.data, case["calls"], cfg.lr, 0.9, 0.999, 1e-8,
            cfg.weight_decay, cfg.clip_norm, cfg.warmup_steps, cfg.total_steps, cfg.lr_floor_frac, cfg.accum_steps,
            _cstrs(no_decay), 2, 4)
    size = ref.ref_optim_serialised(*args, None, 0)
    assert size > 0
    want = (ctypes.c_uint8 * size)()
    assert ref.ref_optim_serialised(*args, want, size) == size
    # the device optimiser on the same parameters and gradients
    stream = torch.cuda.current_stream().cuda_stream
    w = torch.from_numpy(w0.copy()).to(cuda)
    g_dev = torch.from_numpy(grads).to(cuda)
    opt = host.r97host_optim_create(ctypes.byref(cfg), 4, _cstrs(names), cnt, w.data_ptr(), _cstrs(no_decay), 2,
                                    ctypes.c_void_p(stream))
    assert opt, host.r97host_optim_error()
    try:
        applied = 0
        for s in range(case["calls"]):
            rc = host.r97host_optim_step(opt, g_dev[s].data_ptr())
            assert rc in (0, 1), host.r97host_optim_error()
            applied += rc
        done, pend = ctypes.c_int32(), ctypes.c_int32()
        host.r97host_optim_state(opt, ctypes.byref(done), ctypes.byref(pend))
        assert done.value == applied == case["calls"] // case["accum"]
        assert pend.value == case["calls"] % case["accum"]
        got_size = host.r97host_optim_serialise(opt, None, 0)
        assert got_size == size
        got = (ctypes.c_uint8 * got_size)()
        assert host.r97host_optim_serialise(opt, got, got_size) == size
        assert bytes(got) == bytes(want), "serialised state differs from the reference optimiser's"
        # restore: the reference's checkpoint into a fresh device optimiser reproduces it exactly
        w2 = torch.zeros_like(w)
        opt2 = host.r97host_optim_create(ctypes.byref(cfg), 4, _cstrs(names), cnt, w2.data_ptr(), _cstrs(no_decay), 2,
                                         ctypes.c_void_p(stream))
        assert host.r97host_optim_restore(opt2, want, size) == 0, host.r97host_optim_error()
        back = (ctypes.c_uint8 * size)()
        host.r97host_optim_serialise(opt2, back, size)
        assert bytes(back) == bytes(want)
        assert torch.equal(w2, w)
        # bad bytes leave the state unchanged
        bad = bytearray(bytes(want))
        bad[0] = ord("X")
        bad_buf = (ctypes.c_uint8 * len(bad)).from_buffer(bad)
        assert host.r97host_optim_restore(opt2, bad_buf, len(bad)) == 1
        host.r97host_optim_serialise(opt2, back, size)
        assert bytes(back) == bytes(want)
        host.r97host_optim_destroy(opt2)
    finally:
        host.r97host_optim_destroy(opt)
