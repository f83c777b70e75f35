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


def test_int8_entry_points_reject_bad_arguments_without_a_gpu():
    """The w8a8 entry points check their operand rules on the host and return R97B_EINVAL (1) before any
    device work: null operands, K or a pitch off the 16-byte rule, a fold width off the 128 groups, a rotation
    wider than 256 or not a power of two, a group scale whose pitch is short."""
    h = lib()
    fake = ctypes.c_void_p(1 << 20)  # never dereferenced: every call below fails its checks first
    nul = None
    # r97b_gemm_i8g(a, lda, sa, ld_as, b, ldb, sb, ld_bs, M, N, K, y, ldy, y_bf16, stream)
    assert h.r97b_gemm_i8g(nul, 256, fake, 2, fake, 256, fake, 2, 8, 8, 256, fake, 8, 0, nul) == 1
    assert h.r97b_gemm_i8g(fake, 200, fake, 2, fake, 200, fake, 2, 8, 8, 200, fake, 8, 0, nul) == 1  # K % 16
    assert h.r97b_gemm_i8g(fake, 264, fake, 1, fake, 256, fake, 2, 8, 8, 256, fake, 8, 0, nul) == 1  # ld_as < K/128
    # r97b_gemm_i8g_gated(..., M, N, K, act, q, ldq, qs, ld_qs, ob, ld_ob, stream): n = N / 2 = 96 not a multiple of 128
    assert h.r97b_gemm_i8g_gated(fake, 256, fake, 2, fake, 256, fake, 2, 8, 192, 256, 0, fake, 96, fake, 1, nul, 0,
                                 nul) == 1
    # r97b_fused_quant_i8g(part, x, ldx, x2, ldx2, w, eps, wadd, mult, rows, n, group, codes, ldc, s, lds, out,
    #                      ldo, stream)
    assert h.r97b_fused_quant_i8g(0, fake, 512, nul, 0, fake, 1e-6, 0.0, 1.0, 4, 512, 512, fake, 512, fake, 1, nul,
                                  0, nul) == 1  # group 512 > 256
    assert h.r97b_fused_quant_i8g(1, fake, 512, nul, 0, nul, 1e-6, 0.0, 1.0, 4, 512, 96, fake, 512, fake, 6, nul,
                                  0, nul) == 1  # group 96 not a power of two
    assert h.r97b_fused_quant_i8g(2, fake, 512, nul, 0, nul, 1e-6, 0.0, 1.0, 4, 512, 128, fake, 512, fake, 4, nul,
                                  0, nul) == 1  # sigmoid mul without b
    assert h.r97b_fused_quant_i8g(0, fake, 512, nul, 0, nul, 1e-6, 1.0, 1.0, 4, 512, 128, fake, 512, fake, 4, nul,
                                  0, nul) == 1  # an offset without a gain
    # r97b_group_scale(x, ldx, rows, cols, group, s, lds, y, ldy, y_bf16, stream): lds < ceil(cols / group)
    assert h.r97b_group_scale(fake, 256, 4, 256, 128, fake, 1, fake, 256, 0, nul) == 1
