"""Loads libr97b200.so (the sm_100a kernels) through its C ABI (include/r97b.h).

There is no fallback: if the library cannot be built or loaded, every op raises. The library is
built in-tree by ``r97training_b200.build`` (``__graft_entry__.build()``); when it is missing on a
machine that has nvcc it is built on first use.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_lock = threading.Lock()
_lib = None

c_i32, c_i64, c_f32, c_vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class R97bError(RuntimeError):
    pass


class R97bMat(ctypes.Structure):
    _fields_ = [("ptr", c_vp), ("ld", c_i64), ("mn_major", c_i32), ("_pad", c_i32)]


class R97bGemm(ctypes.Structure):
    _fields_ = [("M", c_i64), ("N", c_i64), ("K1", c_i64), ("K2", c_i64),
                ("a1", R97bMat), ("b1", R97bMat), ("a2", R97bMat), ("b2", R97bMat),
                ("mode", c_i32), ("splits", c_i32), ("alpha", c_f32), ("beta", c_f32),
                ("out", c_vp), ("ldo", c_i64), ("addend", c_vp), ("ld_add", c_i64),
                ("bn", c_i32), ("_pad", c_i32), ("ws", c_vp), ("ws_bytes", c_i64),
                ("out2", c_vp), ("ldo2", c_i64)]


class R97bAttnBwd(ctypes.Structure):
    _fields_ = [("B", c_i32), ("Hq", c_i32), ("Hkv", c_i32), ("S", c_i32), ("D", c_i32), ("scale", c_f32),
                ("q", c_vp), ("k", c_vp), ("v", c_vp), ("o", c_vp), ("dout", c_vp), ("lse", c_vp),
                ("dq", c_vp), ("dk", c_vp), ("dv", c_vp), ("ws", c_vp), ("ws_bytes", c_i64)]


class R97bAttnFwd(ctypes.Structure):
    _fields_ = [("B", c_i32), ("Hq", c_i32), ("Hkv", c_i32), ("S", c_i32), ("D", c_i32), ("scale", c_f32),
                ("q", c_vp), ("k", c_vp), ("v", c_vp), ("o", c_vp), ("lse", c_vp)]


class R97bCastSeg(ctypes.Structure):
    _fields_ = [("src", c_vp), ("ld_src", c_i64), ("dst", c_vp), ("ld_dst", c_i64), ("rows", c_i64),
                ("cols", c_i64), ("unit0", c_i64)]


class R97bQLinearLora(ctypes.Structure):
    _fields_ = [("M", c_i64), ("N", c_i64), ("K", c_i64), ("rank", c_i32), ("scale", c_f32), ("w", c_vp),
                ("w_bf16", c_vp), ("w_decoded", c_i32), ("_pad", c_i32), ("x", c_vp), ("A", c_vp), ("B", c_vp),
                ("t", c_vp), ("y", c_vp), ("addend", c_vp), ("ws", c_vp), ("ws_bytes", c_i64)]


class R97bQLinearLoraBwd(ctypes.Structure):
    _fields_ = [("M", c_i64), ("N", c_i64), ("K", c_i64), ("rank", c_i32), ("scale", c_f32), ("w_bf16", c_vp),
                ("x", c_vp), ("A", c_vp), ("B", c_vp), ("t", c_vp), ("dy", c_vp), ("dt", c_vp), ("dx", c_vp),
                ("dA", c_vp), ("dB", c_vp), ("ws", c_vp), ("ws_bytes", c_i64)]


class R97IqrDecodeDesc(ctypes.Structure):
    """Field-for-field the C struct of include/r97b_iqr.h (the reference's R97IqrDecodeDesc layout)."""
    _fields_ = [
        ("rows_all", c_i64), ("cols", c_i64), ("row0", c_i64), ("rows", c_i64),
        ("bits", c_i32), ("state_bits", c_i32), ("run_rows", c_i32), ("rb", c_i32),
        ("mad", c_i32), ("round_mad", c_i32), ("mad_a", ctypes.c_uint32), ("mad_b", ctypes.c_uint32),
        ("lut", c_vp),
        ("codes", c_vp), ("codes_row_bytes", c_i64),
        ("scale", c_vp), ("scale_dtype", c_i32), ("scale_block_cols", c_i64), ("scale_row_bytes", c_i64),
        ("affine", c_i32), ("zero", c_vp), ("zero_bits", c_i32), ("zero_row_bytes", c_i64),
        ("scale2", c_vp), ("scale2_dtype", c_i32), ("scale2_row_bytes", c_i64),
        ("scale2_block_rows", c_i64), ("scale2_block_cols", c_i64),
        ("out_codes", c_vp), ("out_scale", c_vp),
    ]


class R97bEncPlane(ctypes.Structure):
    _fields_ = [("role", ctypes.c_char * 24), ("dtype", c_i32), ("block", c_i64 * 2), ("extent", c_i64 * 2)]


class R97bEncoding(ctypes.Structure):
    """include/r97b_iqr.h R97bEncoding: the encoding fields the IQR form derivation reads."""
    _fields_ = [("n_planes", c_i32), ("plane", R97bEncPlane * 8)]


class R97bStoredPlane(ctypes.Structure):
    _fields_ = [("data", c_vp), ("bytes", c_i64)]


_SIGS = {
    "r97b_abi_version": (c_i32, []),
    "r97b_device_error": (c_i32, [c_vp]),
    "r97b_last_launch_error": (c_i32, []),
    "r97b_launch_error_name": (ctypes.c_char_p, [c_i32]),
    "r97_iqr_decode": (c_i32, [c_vp, c_vp]),
    "r97b_iqr_dequant_bf16": (c_i32, [c_vp, c_vp, c_i64, c_vp]),
    "r97b_gemm": (c_i32, [c_vp, c_vp]),
    "r97b_gemm_workspace_bytes": (c_i64, [c_vp]),
    "r97b_attn_bwd": (c_i32, [c_vp, c_vp]),
    "r97b_attn_fwd": (c_i32, [c_vp, c_vp]),
    "r97b_cast_segments": (c_i32, [c_vp, c_i32, c_i64, c_vp]),
    "r97b_add_f32": (c_i32, [c_vp, c_vp, c_i64, c_vp]),
    "r97b_quant_act_i8g": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i32, c_vp, c_i64, c_vp, c_vp]),
    "r97b_quant_act_i8g_bwd": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_i64, c_i32, c_vp, c_vp, c_i64, c_vp, c_i64,
                                       c_i32, c_vp]),
    "r97b_fused_quant_i8g": (c_i32, [c_i32, c_vp, c_i64, c_vp, c_i64, c_vp, c_f32, c_f32, c_f32, c_i64, c_i64, c_i64,
                                     c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp]),
    "r97b_fused_quant_i8g_bwd": (c_i32, [c_i32, c_vp, c_i64, c_vp, c_i64, c_vp, c_f32, c_f32, c_f32, c_i64, c_i64,
                                         c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i32,
                                         c_vp]),
    "r97b_iqr_desc_from_planes": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_i32, c_vp]),
    "r97b_iqr_decode_planes": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "r97b_group_scale": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_i64, c_i32, c_vp]),
    "r97b_gemm_i8g": (c_i32, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64,
                              c_i32, c_vp]),
    "r97b_gemm_i8g_gated": (c_i32, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i32,
                                    c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp]),
    "r97b_qlinear_lora_fwd": (c_i32, [c_vp, c_vp]),
    "r97b_qlinear_lora_bwd": (c_i32, [c_vp, c_vp]),
    "r97b_qlinear_lora_workspace_bytes": (c_i64, [c_i64, c_i64, c_i64, c_i32]),
    "r97b_attn_bwd_workspace_bytes": (c_i64, [c_i32, c_i32, c_i32]),
    "r97b_rmsnorm_fwd": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_f32, c_f32, c_f32, c_vp]),
    "r97b_rmsnorm_bwd": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_f32, c_f32, c_f32, c_vp]),
    "r97b_gated_rmsnorm_fwd": (c_i32, [c_vp, c_vp, c_i64, c_i32, c_vp, c_vp, c_i64, c_i64, c_f32, c_i32, c_vp]),
    "r97b_gated_rmsnorm_bwd": (c_i32, [c_vp, c_vp, c_i64, c_i32, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_f32, c_i32,
                                       c_vp]),
    "r97b_ce_kld": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_f32, c_f32, c_f32,
                            c_vp]),
    "r97b_adamw_step": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i64, c_f32, c_f32, c_f32, c_f32, c_f32, c_f32, c_f32,
                                c_f32, c_vp, c_i32, c_vp]),
    "r97b_global_norm_scratch_bytes": (c_i64, [c_i64]),
    "r97b_global_norm": (c_i32, [c_vp, c_i64, c_f32, c_f32, c_vp, c_vp, c_vp, c_vp]),
    "r97b_gdn_chunk_table": (c_i32, [c_vp, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "r97b_gdn_fwd": (c_i32, [c_vp, c_vp, c_vp]),
    "r97b_gdn_bwd": (c_i32, [c_vp, c_vp, c_vp]),
    "r97b_gdn_sum_heads": (c_i32, [c_vp, c_vp, c_i64, c_i32, c_i32, c_vp]),
    "r97b_codes_dequant_bf16": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp]),
    "r97b_mem_alloc": (c_i32, [c_vp, c_i64]),
    "r97b_mem_free": (c_i32, [c_vp]),
    "r97b_memcpy": (c_i32, [c_vp, c_vp, c_i64, c_i32, c_vp]),
    "r97b_memset": (c_i32, [c_vp, c_i32, c_i64, c_vp]),
    "r97b_stream_create": (c_i32, [c_vp]),
    "r97b_stream_sync": (c_i32, [c_vp]),
    "r97b_last_cuda_error": (ctypes.c_char_p, []),
    "r97b_gdn_kkt_bwd": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "r97b_conv_prep_fwd": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp]),
    "r97b_conv_prep_bwd": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_i32,
                                   c_vp, c_i64, c_vp]),
    "r97b_gates_fwd": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "r97b_gates_bwd": (c_i32, [c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "r97b_swiglu_fwd": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp]),
    "r97b_swiglu_bwd": (c_i32, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp]),
    "r97b_qk_norm_rope_fwd": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_i32, c_i64, c_i32, c_f32,
                                      c_vp, c_vp]),
    "r97b_qk_norm_rope_bwd": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_i32, c_i64, c_i32, c_f32,
                                      c_vp, c_vp, c_i64, c_vp]),
    "r97b_to_bhsd": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_i32, c_i64, c_i32, c_vp, c_i32, c_vp]),
    "r97b_gate_mul_fwd": (c_i32, [c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i64, c_i32, c_vp, c_vp]),
    "r97b_gate_mul_bwd": (c_i32, [c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_i64, c_i32, c_vp, c_vp, c_vp, c_i64,
                                  c_vp]),
    "r97b_embed": (c_i32, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_vp]),
    "r97b_cast_f32_bf16": (c_i32, [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "r97b_launch_count": (ctypes.c_uint64, []),
    "r97b_adamw_step_dev": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_f32, c_f32, c_f32, c_f32, c_f32, c_vp,
                                    c_i32, c_vp]),
    "r97b_global_norm_noalloc": (c_i32, [c_vp, c_i64, c_f32, c_f32, c_vp, c_vp, c_vp]),
}

OPTIONAL = set()


def lib():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_build.LIB):
                _build.build_kernels()
            handle = ctypes.CDLL(_build.LIB, mode=ctypes.RTLD_GLOBAL)
            for name, (res, args) in _SIGS.items():
                try:
                    fn = getattr(handle, name)
                except AttributeError:
                    if name in OPTIONAL:
                        continue
                    raise R97bError(f"{_build.LIB} does not export {name}")
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        detail = ""
        if rc == 2 and _lib is not None:  # R97B_ELAUNCH: name the CUDA error behind it
            code = int(_lib.r97b_last_launch_error())
            detail = f" ({_lib.r97b_launch_error_name(code).decode()})" if code else ""
        raise R97bError(f"{what} returned status {rc}{detail}")


def exported_symbols():
    """Every function name the ABI declares, for the load test."""
    return sorted(_SIGS)
