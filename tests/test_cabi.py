"""CPU checks of the C ABI: the library loads without a GPU, exports every
function include/b200k.h declares, and the ctypes mirror has the C layout."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from compiler import runtime
from compiler.runtime import cabi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b200k.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(b200k_\w+)\s*\(", src, flags=re.M)))


def test_header_declarations_are_exported():
    lib = ctypes.CDLL(runtime.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), f"{name} declared in b200k.h but not exported"
    assert sorted(cabi.EXPORTED) == sorted(n for n in names if n in cabi.EXPORTED)


def test_library_answers_without_gpu():
    lib = cabi.library()
    assert lib.b200k_version() == 1
    assert lib.b200k_status_string(6).decode().startswith("device-side wait")
    n = lib.b200k_gemm_num_configs()
    assert n >= 2
    bm, bn, bk, st = (ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int())
    assert lib.b200k_gemm_config_info(0, ctypes.byref(bm), ctypes.byref(bn), ctypes.byref(bk), ctypes.byref(st)) == 0
    assert bm.value in (128, 256) and bk.value == 64 and bn.value in (128, 192, 256, 512)
    assert lib.b200k_gemm_config_info(n, None, None, None, None) == 1  # B200K_ERR_ARG


def test_tile_config_pick_rules():
    """The picker's documented domains (no GPU needed: 148 SMs assumed):
    CTA-pair tiles only from K = 1536, the 256 x 512 pair tile only from
    K = 12288, and a config inside the table for every shape."""
    lib = cabi.library()
    n = lib.b200k_gemm_num_configs()
    bm, bn = ctypes.c_int(), ctypes.c_int()
    info = {}
    for c in range(n):
        assert lib.b200k_gemm_config_info(c, ctypes.byref(bm), ctypes.byref(bn), None, None) == 0
        info[c] = (bm.value, bn.value)
    for M, N, K in [(12608, 3072, 768), (12608, 2304, 768), (12608, 768, 768), (4096, 4096, 1024), (512, 512, 512),
                    (1, 8, 8), (16384, 4096, 1535)]:
        c = lib.b200k_gemm_pick_config(M, N, K)
        assert 0 <= c < n and info[c][0] == 128, (M, N, K, c)
    for M, N, K in [(4096, 4096, 4096), (8192, 8192, 8192), (16384, 2048, 2048), (16384, 8192, 2048),
                    (16384, 2048, 8192), (12608, 768, 3072)]:
        c = lib.b200k_gemm_pick_config(M, N, K)
        assert info[c] == (256, 256), (M, N, K, c)
    assert info[lib.b200k_gemm_pick_config(16384, 4096, 14336)] == (256, 512)


def test_host_side_errors_need_no_gpu():
    """Argument errors are caught before any CUDA call."""
    lib = cabi.library()
    assert lib.b200k_pointwise(None, None) == 1
    a = cabi.PointwiseArgs()
    a.n_inputs = 0
    assert lib.b200k_pointwise(ctypes.byref(a), None) == 1
    g = cabi.GemmArgs()
    g.M, g.N, g.K = 4, 4, 8
    assert lib.b200k_gemm_epilogue(ctypes.byref(g), None) == 1  # null pointers
    g.a = g.b = g.out = 16
    g.M, g.N, g.K = 4, 4, 0
    assert lib.b200k_gemm_epilogue(ctypes.byref(g), None) == 3  # K == 0
    g.K = 8
    g.ab_dtype = cabi.F32
    assert lib.b200k_gemm_epilogue(ctypes.byref(g), None) == 4  # fp32 operands unsupported
    g.ab_dtype = cabi.BF16
    g.out_dtype = cabi.BF16
    g.program = cabi.make_program([999], [0.0])
    assert lib.b200k_gemm_epilogue(ctypes.byref(g), None) == 7  # malformed program
    r = cabi.RowNormArgs()
    r.rows, r.cols = 4, 8
    assert lib.b200k_rownorm(ctypes.byref(r), None) == 1  # null x / out
    r.rows = 0
    assert lib.b200k_rownorm(ctypes.byref(r), None) == 0  # empty: nothing to do
    q = cabi.RopeArgs()
    q.sizes[:] = [1, 2, 3, 64]
    assert lib.b200k_rope(ctypes.byref(q), None) == 1  # null pointers
    q.sizes[3] = 0
    assert lib.b200k_rope(ctypes.byref(q), None) == 0  # empty: nothing to do
    q.sizes[3] = -1
    assert lib.b200k_rope(ctypes.byref(q), None) == 3  # B200K_ERR_SHAPE


STRUCTS = {
    "B200kInstr": (cabi.Instr, ["code", "imm"]),
    "B200kProgram": (cabi.Program, ["n", "ins"]),
    "B200kTensorRef": (cabi.TensorRef, ["ptr", "dtype", "strides"]),
    "B200kPointwiseArgs": (cabi.PointwiseArgs, ["rank", "n_inputs", "sizes", "inputs", "out", "out_dtype", "program"]),
    "B200kEpiOperand": (cabi.EpiOperand, ["ptr", "dtype", "stride_m", "stride_n"]),
    "B200kGemmArgs": (cabi.GemmArgs, ["M", "a", "b_stride_n", "ab_dtype", "out", "n_extras", "tile_config",
                                      "extras", "program", "status", "timeout_ns", "form", "test_flags", "trace",
                                      "trace_words"]),
    "B200kEpilogueForm": (cabi.EpilogueForm, ["kind", "bias", "act", "round", "scale", "residual"]),
    "B200kRowNormArgs": (cabi.RowNormArgs, ["rows", "x", "kind", "weight", "flags", "bias", "eps", "out",
                                            "out_dtype", "mean_out", "rstd_out"]),
    "B200kSoftmaxArgs": (cabi.SoftmaxArgs, ["rows", "x", "log_softmax", "out", "out_dtype"]),
    "B200kRopeArgs": (cabi.RopeArgs, ["sizes", "x", "x_strides", "cos", "cos_strides", "sin", "sin_strides", "out",
                                      "out_strides", "dtype"]),
    "B200kRopeTables": (cabi.RopeTables, ["cos", "sin", "stride", "period", "head_dim", "dtype"]),
    "B200kAttentionArgs": (cabi.AttentionArgs, ["batch", "head_dim", "q", "q_strides", "k", "k_strides", "v",
                                                "v_strides", "out", "out_strides", "dtype", "causal", "scale",
                                                "test_flags", "status", "timeout_ns"]),
}


def test_gemm_rope_host_checks():
    """Argument errors of the rotary-epilogue GEMM, reported before any launch."""
    lib = cabi.library()
    g = cabi.GemmArgs()
    g.M, g.N, g.K = 256, 512, 128
    g.a, g.b, g.out = 4096, 8192, 16384
    g.a_stride_m, g.a_stride_k, g.b_stride_k, g.b_stride_n = 128, 1, 1, 128
    g.ab_dtype = g.out_dtype = cabi.BF16
    r = cabi.RopeTables()
    r.cos, r.sin, r.stride, r.period, r.head_dim, r.dtype = 32768, 65536, 64, 2048, 64, cabi.BF16
    assert lib.b200k_gemm_rope(None, ctypes.byref(r), None) == 1
    assert lib.b200k_gemm_rope(ctypes.byref(g), None, None) == 1
    r.head_dim = 128
    assert lib.b200k_gemm_rope(ctypes.byref(g), ctypes.byref(r), None) == 1  # 64-wide heads only
    r.head_dim = 64
    g.N = 520
    assert lib.b200k_gemm_rope(ctypes.byref(g), ctypes.byref(r), None) == 3  # whole heads
    g.N = 512
    r.dtype = cabi.F16
    assert lib.b200k_gemm_rope(ctypes.byref(g), ctypes.byref(r), None) == 4  # tables of the output type
    r.dtype = cabi.BF16
    r.stride = 60
    assert lib.b200k_gemm_rope(ctypes.byref(g), ctypes.byref(r), None) == 2  # 16-byte table rows
    r.stride = 64
    g.n_extras = 1
    assert lib.b200k_gemm_rope(ctypes.byref(g), ctypes.byref(r), None) == 1  # no other epilogue operands


def test_attention_host_checks():
    """Argument errors the library reports before launching anything."""
    lib = cabi.library()
    a = cabi.AttentionArgs()
    a.batch, a.heads, a.kv_heads, a.q_len, a.kv_len, a.head_dim = 1, 4, 2, 16, 16, 64
    assert lib.b200k_attention(None, None) == 1  # B200K_ERR_ARG
    assert lib.b200k_attention(ctypes.byref(a), None) == 1  # null pointers
    a.q = a.k = a.v = a.out = 4096
    for st in (a.q_strides, a.k_strides, a.v_strides, a.out_strides):
        st[0], st[1], st[2], st[3] = 4 * 16 * 64, 16 * 64, 64, 1
    a.head_dim = 128
    assert lib.b200k_attention(ctypes.byref(a), None) == 4  # head_dim 64 only
    a.head_dim = 64
    a.dtype = cabi.F32
    assert lib.b200k_attention(ctypes.byref(a), None) == 4  # 16-bit only
    a.dtype = cabi.BF16
    a.kv_heads = 3
    assert lib.b200k_attention(ctypes.byref(a), None) == 3  # heads % kv_heads
    a.kv_heads = 2
    a.q_strides[3] = 2
    assert lib.b200k_attention(ctypes.byref(a), None) == 4  # unit d stride
    a.q_strides[3] = 1
    a.k_strides[2] = 65
    assert lib.b200k_attention(ctypes.byref(a), None) == 2  # 16-byte rows
    a.k_strides[2] = 64
    a.q = 4098
    assert lib.b200k_attention(ctypes.byref(a), None) == 2  # 16-byte pointers
    a.q_len = 0
    assert lib.b200k_attention(ctypes.byref(a), None) == 0  # empty output: nothing to launch


def test_ctypes_layout_matches_c():
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "b200k.h"', "int main(void) {"]
    for cname, (_, fields) in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for f in fields:
            lines.append(f'  printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("  return 0; }")
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "layout.c")
        exe = os.path.join(d, "layout")
        open(src, "w").write("\n".join(lines))
        r = subprocess.run(["gcc", "-I", os.path.dirname(HEADER), src, "-o", exe], capture_output=True, text=True)
        if r.returncode != 0:
            pytest.fail(r.stderr)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    for line in filter(None, out):
        cname, field, value = line.split()
        cls = STRUCTS[cname][0]
        got = ctypes.sizeof(cls) if field == "size" else getattr(cls, field).offset
        assert got == int(value), f"{cname}.{field}: ctypes {got} vs C {value}"


def test_missing_library_fails_loudly(monkeypatch):
    """Without the built extension the runtime raises instead of falling back
    to anything: there is no CPU or eager path inside the compiled graph."""
    from compiler import runtime

    monkeypatch.setattr(runtime, "_loaded", False)
    monkeypatch.setattr(runtime, "EXT_PATH", "/nonexistent/_b200_ops.so")
    with pytest.raises(runtime.LibraryMissing):
        runtime.load()
