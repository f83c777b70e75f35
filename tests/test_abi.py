"""The C-ABI library loads without a GPU and exports every entry point include/*.h declares."""
import ctypes
import os
import re

from r97training_b200 import build as B
from r97training_b200._lib import exported_symbols, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if not h.endswith(".h") or h == "r97host.h":  # the plugin's own entry points (test_host_plugin.py)
            continue
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:int|int32_t|int64_t|uint64_t|void|unsigned int|const char\s*\*)\s+(r97\w*)\s*\(", src, re.M):
            names.add(m.group(1))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    h = lib()
    decl = declared()
    assert decl, "no declarations found"
    for name in sorted(decl):
        assert hasattr(h, name), f"{B.LIB} does not export {name}"
    assert decl <= set(exported_symbols()) | decl
    assert h.r97b_abi_version() >= 1


def test_binding_table_covers_declarations():
    missing = declared() - set(exported_symbols())
    assert not missing, f"declared in include/ but not bound in _lib: {sorted(missing)}"


def test_gemm_workspace_bytes_without_a_gpu():
    """The split-K workspace size is host arithmetic: 256-byte-rounded tile counters, then the f32 partial
    tiles [splits][tiles][128][bn]; 0 when the call does not split; -1 for a description the GEMM rejects."""
    from r97training_b200._lib import R97bGemm
    g = R97bGemm()
    g.M, g.N, g.K1, g.mode, g.splits, g.bn = 8192, 64, 4096, 4, 2, 64
    assert lib().r97b_gemm_workspace_bytes(ctypes.byref(g)) == 256 + 2 * 64 * 128 * 64 * 4
    g.splits = 1
    assert lib().r97b_gemm_workspace_bytes(ctypes.byref(g)) == 0
    g.mode, g.splits = 0, 2
    assert lib().r97b_gemm_workspace_bytes(ctypes.byref(g)) == 0
    g.mode = 9
    assert lib().r97b_gemm_workspace_bytes(ctypes.byref(g)) == -1
