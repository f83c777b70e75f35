"""The trained adapter on disk in PEFT's layout (adapter_config.json + adapter_model.safetensors), written
and read by the C++ host library (libr97host.so, r97host_adapter_write / r97host_adapter_read) -- the
layout the reference's trainer writes and its server loads (reference include/r97/adapter_io.h,
src/adapter_io.cpp)."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from . import build as _build

_host = None


class R97hostAdapterConfig(ctypes.Structure):
    _fields_ = [("base_model", ctypes.c_char_p), ("rank", ctypes.c_int64), ("alpha", ctypes.c_double),
                ("targets", ctypes.c_void_p), ("n_targets", ctypes.c_int32), ("input_basis", ctypes.c_char_p),
                ("dtype", ctypes.c_int32)]


def host():
    """libr97host.so, bound for the adapter entry points (it loads without the reference's registry)."""
    global _host
    if _host is None:
        if not os.path.exists(_build.HOSTLIB):
            _build.build_all()
        lib = ctypes.CDLL(_build.HOSTLIB)
        lib.r97host_adapter_write.restype = ctypes.c_int
        lib.r97host_adapter_write.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
        lib.r97host_adapter_read.restype = ctypes.c_int
        lib.r97host_adapter_read.argtypes = [ctypes.c_char_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.r97host_adapter_error.restype = ctypes.c_char_p
        _host = lib
    return _host


def _strs(xs):
    return (ctypes.c_char_p * max(len(xs), 1))(*[x.encode() for x in xs])


def write(directory: str, names, shapes, values, *, base_model: str = "", rank: int, alpha: float, targets=(),
          dtype: str = "f32", input_basis: str | None = None) -> None:
    """Writes the adapter directory: `names` (`<module>.lora_A` / `.lora_B`), `shapes` ([rows, cols] each)
    and `values`, their f32 values concatenated in that order -- a numpy array or a torch tensor (a CUDA
    tensor is copied on its current stream by the library)."""
    nm = _strs(list(names))
    sh = np.ascontiguousarray(np.asarray(shapes, dtype=np.int64).reshape(-1, 2))
    tg = _strs(list(targets))
    cfg = R97hostAdapterConfig(base_model.encode(), rank, float(alpha), ctypes.cast(tg, ctypes.c_void_p),
                               len(targets), (input_basis or "").encode(), 1 if dtype == "bf16" else 0)
    on_dev, stream, keep = 0, None, values
    if isinstance(values, torch.Tensor):
        keep = values.detach().float().contiguous()
        ptr = keep.data_ptr()
        if keep.is_cuda:
            on_dev, stream = 1, ctypes.c_void_p(torch.cuda.current_stream(keep.device).cuda_stream)
    else:
        keep = np.ascontiguousarray(np.asarray(values, dtype=np.float32))
        ptr = keep.ctypes.data
    if int(sh.prod(axis=1).sum()) > (keep.numel() if isinstance(keep, torch.Tensor) else keep.size):
        raise ValueError("values hold fewer elements than the shapes name")
    rc = host().r97host_adapter_write(directory.encode(), ctypes.byref(cfg), len(sh), nm, sh.ctypes.data, ptr, on_dev,
                                      stream)
    if rc != 0:
        raise RuntimeError(host().r97host_adapter_error().decode())


def read(directory: str, names, shapes):
    """(values f32 numpy, rank, alpha, dtype name) of an adapter directory, the values laid out as the named
    parameters in order."""
    nm = _strs(list(names))
    sh = np.ascontiguousarray(np.asarray(shapes, dtype=np.int64).reshape(-1, 2))
    out = np.empty(int(sh.prod(axis=1).sum()), dtype=np.float32)
    rank, alpha, dt = ctypes.c_int64(), ctypes.c_double(), ctypes.c_int32()
    rc = host().r97host_adapter_read(directory.encode(), len(sh), nm, sh.ctypes.data, out.ctypes.data,
                                     ctypes.byref(rank), ctypes.byref(alpha), ctypes.byref(dt))
    if rc != 0:
        raise RuntimeError(host().r97host_adapter_error().decode())
    return out, rank.value, alpha.value, "bf16" if dt.value == 1 else "f32"


def save_adapter(adapter, directory: str, *, base_model: str = "", dtype: str = "f32", input_basis=None) -> None:
    """A model's trained adapter (model.Adapter: the flat f32 master buffer on the device) as a PEFT
    directory; target_modules are the projections' leaf names."""
    targets = sorted({n.rsplit(".", 2)[0].rsplit(".", 1)[1] for n in adapter.names})
    write(directory, adapter.names, adapter.shapes, adapter.w, base_model=base_model, rank=adapter.cfg.rank,
          alpha=adapter.cfg.alpha, targets=targets, dtype=dtype, input_basis=input_basis)


def load_adapter(adapter, directory: str):
    """Loads a PEFT directory into a model.Adapter (master weights, then its bf16 mirrors); returns the
    file's (rank, alpha, dtype)."""
    values, rank, alpha, dt = read(directory, adapter.names, adapter.shapes)
    if rank != adapter.cfg.rank:
        raise ValueError(f"the adapter has rank {rank}, the model {adapter.cfg.rank}")
    adapter.w.copy_(torch.from_numpy(values).to(adapter.w.device))
    adapter.refresh_mirrors()
    return rank, alpha, dt
