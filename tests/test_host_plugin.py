"""The adjoint-row plugin (libr97host.so) on CPU: it loads without a GPU, registers its device rows into
the reference's own registry at load with the frozen positions of the reference's rows, and loads (and
registers nothing) in a process without the registry. CPU only."""
import os
import re
import subprocess
import sys

import pytest

import oracle
from r97training_b200 import build as B
from tests.plugin_util import plugin

# op -> the frozen operand positions the reference registers for it (reference linear.cpp:444-457 and
# device/linear.hip:760,
# lora.cpp:534-538, gdn_kkt.cpp:355, gdn_scan.cpp:584, gdn_prep.cpp:597-600, elementwise.cpp:687; the quant
# family's two int8 ops have none and its fused rmsnorm producer freezes the gain, quant.cpp:1518-1533)
FROZEN = {
    "gemm_nt": [1],
    "gemm_nt_q": [1, 2, 3],
    "lora_shrink": [1, 2, 3],
    "lora_expand": [1, 2, 3],
    "lora_expand_mm": [1, 2, 3],
    "rmsnorm": [1],
    "gdn_gated_rmsnorm": [2],
    "gdn_kkt_solve": [3],
    "gdn_chunk_scan": [6, 7, 10],
    "quant_act_i8g": [],
    "had_quant_act_i8g": [],
    "rmsnorm_had_quant_i8g": [1],
    "gated_had_quant_i8g": [],
    "gate_had_quant_i8g": [],
}


def test_plugin_registers_device_rows_into_reference_registry():
    lib = plugin()
    assert lib.r97host_registered() == 1
    for op, frozen in FROZEN.items():
        rows = oracle.op_rows(op)
        assert rows["device"], f"no device row for {op}"
        assert rows["device_frozen"] == frozen, (op, rows)
        assert rows["host"], f"the reference has no host row for {op}"
        if op != "lora_shrink":  # the host's first lora_shrink row is the coded form's (2, 3)
            assert rows["host_frozen"] == frozen, (op, rows)


def test_plugin_loads_without_registry():
    """Loaded alone, the plugin's weak references to the host stay null and it registers nothing."""
    if not os.path.exists(B.HOSTLIB):
        B.build_all()
    code = ("import ctypes,sys; l=ctypes.CDLL(sys.argv[1]); l.r97host_registered.restype=ctypes.c_int; "
            "print(l.r97host_registered())")
    r = subprocess.run([sys.executable, "-c", code, B.HOSTLIB], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "0"


def test_plugin_exports_its_c_entry_points():
    if not os.path.exists(B.HOSTLIB):
        B.build_all()
    out = subprocess.run(["nm", "-D", "--defined-only", B.HOSTLIB], capture_output=True, text=True).stdout
    src = re.sub(r"/\*.*?\*/", "", open(os.path.join(os.path.dirname(B.HOSTLIB), "..", "include", "r97host.h")).read(),
                 flags=re.S)
    declared = set(re.findall(r"\b(r97host_\w+)\s*\(", src))
    assert {"r97host_registered", "r97host_head_ce", "r97host_optim_create", "r97host_optim_serialise"} <= declared
    for name in sorted(declared):
        assert f" T {name}" in out, name
