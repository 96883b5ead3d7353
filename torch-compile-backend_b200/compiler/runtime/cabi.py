"""ctypes view of the C ABI in include/b200k.h.

This is the binding a non-PyTorch host would write (plain pointers, sizes,
strides).  The GPU parity tests call the kernels through it, below the torch
binding, and the CPU tests check that every declared symbol is exported.
Tensors passed in must already live on the current CUDA device.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import LIB_PATH

MAX_DIMS = 6
MAX_INPUTS = 8
MAX_INSTR = 64

F32, F16, BF16, F64, I32, I64, BOOL, U8 = range(8)
DTYPE = {
    torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.float64: F64,
    torch.int32: I32, torch.int64: I64, torch.bool: BOOL, torch.uint8: U8,
}
ROW_RMSNORM, ROW_LAYERNORM, ROW_RMSNORM_SWIGLU = 0, 1, 2
GEMM_TEST_WITHHOLD_READY = 1  # include/b200k.h: failure-detection test hook

EXPORTED = [
    "b200k_pointwise", "b200k_gemm_epilogue", "b200k_gemm_num_configs", "b200k_gemm_config_info",
    "b200k_gemm_pick_config", "b200k_rownorm", "b200k_softmax", "b200k_status_string", "b200k_version",
    "b200k_gemm_epilogue_noalloc", "b200k_gemm_noalloc_status", "b200k_rope", "b200k_pointwise_jit_stats",
    "b200k_pointwise_jit_compile", "b200k_attention", "b200k_gemm_rope",
]


class Instr(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int32), ("imm", ctypes.c_float)]


class Program(ctypes.Structure):
    _fields_ = [("n", ctypes.c_int32), ("pad", ctypes.c_int32), ("ins", Instr * MAX_INSTR)]


class TensorRef(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("pad", ctypes.c_int32),
                ("strides", ctypes.c_int64 * MAX_DIMS)]


class PointwiseArgs(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("n_inputs", ctypes.c_int32), ("sizes", ctypes.c_int64 * MAX_DIMS),
                ("inputs", TensorRef * MAX_INPUTS), ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int32),
                ("pad", ctypes.c_int32), ("program", Program)]


class EpiOperand(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("pad", ctypes.c_int32),
                ("stride_m", ctypes.c_int64), ("stride_n", ctypes.c_int64)]


class EpilogueForm(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("bias", ctypes.c_int32), ("act", ctypes.c_int32),
                ("round", ctypes.c_int32), ("scale", ctypes.c_int32), ("residual", ctypes.c_int32)]


class GemmArgs(ctypes.Structure):
    _fields_ = [("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("a", ctypes.c_void_p), ("a_stride_m", ctypes.c_int64), ("a_stride_k", ctypes.c_int64),
                ("b", ctypes.c_void_p), ("b_stride_k", ctypes.c_int64), ("b_stride_n", ctypes.c_int64),
                ("ab_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
                ("out", ctypes.c_void_p), ("out_stride_m", ctypes.c_int64), ("out_stride_n", ctypes.c_int64),
                ("n_extras", ctypes.c_int32), ("tile_config", ctypes.c_int32),
                ("extras", EpiOperand * (MAX_INPUTS - 1)), ("program", Program),
                ("status", ctypes.c_void_p), ("timeout_ns", ctypes.c_int64), ("form", EpilogueForm),
                ("test_flags", ctypes.c_int32), ("trace", ctypes.c_void_p), ("trace_words", ctypes.c_int64)]

TRACE_WORDS = 256


class RowNormArgs(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("x", ctypes.c_void_p),
                ("x_row_stride", ctypes.c_int64), ("x_dtype", ctypes.c_int32), ("kind", ctypes.c_int32),
                ("weight", ctypes.c_void_p), ("w_dtype", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("bias", ctypes.c_void_p), ("b_dtype", ctypes.c_int32), ("eps", ctypes.c_float),
                ("out", ctypes.c_void_p), ("out_row_stride", ctypes.c_int64), ("out_dtype", ctypes.c_int32),
                ("pad", ctypes.c_int32), ("mean_out", ctypes.c_void_p), ("rstd_out", ctypes.c_void_p)]


class SoftmaxArgs(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("x", ctypes.c_void_p),
                ("x_row_stride", ctypes.c_int64), ("x_dtype", ctypes.c_int32), ("log_softmax", ctypes.c_int32),
                ("out", ctypes.c_void_p), ("out_row_stride", ctypes.c_int64), ("out_dtype", ctypes.c_int32),
                ("pad", ctypes.c_int32)]


class RopeArgs(ctypes.Structure):
    _fields_ = [("sizes", ctypes.c_int64 * 4), ("x", ctypes.c_void_p), ("x_strides", ctypes.c_int64 * 4),
                ("cos", ctypes.c_void_p), ("cos_strides", ctypes.c_int64 * 4), ("sin", ctypes.c_void_p),
                ("sin_strides", ctypes.c_int64 * 4), ("out", ctypes.c_void_p), ("out_strides", ctypes.c_int64 * 4),
                ("dtype", ctypes.c_int32), ("pad", ctypes.c_int32)]


class RopeTables(ctypes.Structure):
    _fields_ = [("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("stride", ctypes.c_int64),
                ("period", ctypes.c_int64), ("head_dim", ctypes.c_int32), ("dtype", ctypes.c_int32)]


class AttentionArgs(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("kv_heads", ctypes.c_int64),
                ("q_len", ctypes.c_int64), ("kv_len", ctypes.c_int64), ("head_dim", ctypes.c_int64),
                ("q", ctypes.c_void_p), ("q_strides", ctypes.c_int64 * 4),
                ("k", ctypes.c_void_p), ("k_strides", ctypes.c_int64 * 4),
                ("v", ctypes.c_void_p), ("v_strides", ctypes.c_int64 * 4),
                ("out", ctypes.c_void_p), ("out_strides", ctypes.c_int64 * 4),
                ("dtype", ctypes.c_int32), ("causal", ctypes.c_int32), ("scale", ctypes.c_float),
                ("test_flags", ctypes.c_int32), ("status", ctypes.c_void_p), ("timeout_ns", ctypes.c_int64)]


ATTN_TEST_WITHHOLD_SCORES = 1  # include/b200k.h: failure-detection test hook

_lib = None


def library() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run torch-compile-backend_b200/csrc/build.py")
        lib = ctypes.CDLL(LIB_PATH)
        for name, argt in [
            ("b200k_pointwise", [ctypes.POINTER(PointwiseArgs), ctypes.c_void_p]),
            ("b200k_gemm_epilogue", [ctypes.POINTER(GemmArgs), ctypes.c_void_p]),
            ("b200k_gemm_epilogue_noalloc", [ctypes.POINTER(GemmArgs), ctypes.c_void_p]),
            ("b200k_gemm_noalloc_status", [ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p]),
            ("b200k_rownorm", [ctypes.POINTER(RowNormArgs), ctypes.c_void_p]),
            ("b200k_softmax", [ctypes.POINTER(SoftmaxArgs), ctypes.c_void_p]),
            ("b200k_rope", [ctypes.POINTER(RopeArgs), ctypes.c_void_p]),
            ("b200k_attention", [ctypes.POINTER(AttentionArgs), ctypes.c_void_p]),
            ("b200k_gemm_pick_config", [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]),
            ("b200k_gemm_config_info", [ctypes.c_int] + [ctypes.POINTER(ctypes.c_int)] * 4),
            ("b200k_gemm_num_configs", []),
            ("b200k_version", []),
            ("b200k_pointwise_jit_stats", [ctypes.POINTER(ctypes.c_int64)] * 3),
            ("b200k_pointwise_jit_compile", [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int32),
                                             ctypes.POINTER(ctypes.c_int32), ctypes.c_int32,
                                             ctypes.POINTER(Program), ctypes.c_char_p, ctypes.c_int64]),
        ]:
            fn = getattr(lib, name)
            fn.argtypes = argt
            fn.restype = ctypes.c_int
        lib.b200k_status_string.argtypes = [ctypes.c_int]
        lib.b200k_status_string.restype = ctypes.c_char_p
        _lib = lib
    return _lib


class CError(RuntimeError):
    def __init__(self, what: str, code: int):
        super().__init__(f"{what}: {library().b200k_status_string(code).decode()} (code {code})")
        self.code = code


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check(what: str, rc: int) -> None:
    if rc != 0:
        raise CError(what, rc)


def make_program(code, imm) -> Program:
    p = Program()
    if len(code) > MAX_INSTR:
        raise ValueError("program too long")
    p.n = len(code)
    for i, (c, v) in enumerate(zip(code, imm)):
        p.ins[i].code = int(c)
        p.ins[i].imm = float(v)
    return p


def pointwise(inputs: list[torch.Tensor], code, imm, out: torch.Tensor) -> None:
    a = PointwiseArgs()
    shape = list(out.shape)
    a.rank = len(shape)
    a.n_inputs = len(inputs)
    for d, s in enumerate(shape):
        a.sizes[d] = s
    for i, t in enumerate(inputs):
        e = t.expand(shape)
        a.inputs[i].ptr = e.data_ptr()
        a.inputs[i].dtype = DTYPE[e.dtype]
        for d in range(len(shape)):
            a.inputs[i].strides[d] = e.stride(d)
    a.out = out.data_ptr()
    a.out_dtype = DTYPE[out.dtype]
    a.program = make_program(code, imm)
    _check("b200k_pointwise", library().b200k_pointwise(ctypes.byref(a), _stream()))


def pointwise_jit_stats() -> dict:
    """This process's generated pointwise kernels: compiled, failed, launches."""
    v = [ctypes.c_int64() for _ in range(3)]
    _check("b200k_pointwise_jit_stats", library().b200k_pointwise_jit_stats(*[ctypes.byref(x) for x in v]))
    return {"compiled": v[0].value, "failed": v[1].value, "launches": v[2].value}


def pointwise_jit_compile(rank: int, dtypes: list[int], unit_stride: list[bool], out_dtype: int, code,
                          imm) -> tuple[int, str]:
    """Generates and compiles (no GPU needed) the kernel of a program; returns
    (status code, NVRTC log)."""
    n = len(dtypes)
    dt = (ctypes.c_int32 * max(n, 1))(*dtypes)
    us = (ctypes.c_int32 * max(n, 1))(*[int(bool(u)) for u in unit_stride])
    prog = make_program(code, imm)
    log = ctypes.create_string_buffer(8192)
    rc = library().b200k_pointwise_jit_compile(rank, n, dt, us, out_dtype, ctypes.byref(prog), log, len(log))
    return rc, log.value.decode(errors="replace")


def gemm_epilogue(a: torch.Tensor, b: torch.Tensor, extras: list[torch.Tensor], code, imm, out: torch.Tensor,
                  tile_config: int = -1, status: torch.Tensor | None = None, timeout_ns: int = 0,
                  form=None, noalloc: bool = False, trace: torch.Tensor | None = None, test_flags: int = 0) -> None:
    """out[M,N] = program(a @ b, extras) with extras given as [M,N]-broadcastable tensors.
    noalloc=True calls b200k_gemm_epilogue_noalloc, which ignores `status` and
    uses the library's own status scratch (for hosts that cannot allocate)."""
    g = GemmArgs()
    M, K = a.shape
    N = b.shape[1]
    g.M, g.N, g.K = M, N, K
    g.a, g.a_stride_m, g.a_stride_k = a.data_ptr(), a.stride(0), a.stride(1)
    g.b, g.b_stride_k, g.b_stride_n = b.data_ptr(), b.stride(0), b.stride(1)
    g.ab_dtype = DTYPE[a.dtype]
    g.out_dtype = DTYPE[out.dtype]
    g.out, g.out_stride_m, g.out_stride_n = out.data_ptr(), out.stride(0), out.stride(1)
    g.n_extras = len(extras)
    g.tile_config = tile_config
    for i, t in enumerate(extras):
        e = t.expand(M, N)
        g.extras[i].ptr = e.data_ptr()
        g.extras[i].dtype = DTYPE[e.dtype]
        g.extras[i].stride_m = e.stride(0)
        g.extras[i].stride_n = e.stride(1)
    g.program = make_program(code, imm)
    g.status = status.data_ptr() if status is not None else None
    g.timeout_ns = timeout_ns
    g.test_flags = test_flags
    if form:
        (g.form.kind, g.form.bias, g.form.act, g.form.round, g.form.scale, g.form.residual) = form
    if trace is not None:  # int64 device tensor, TRACE_WORDS per CTA
        g.trace, g.trace_words = trace.data_ptr(), trace.numel()
    if noalloc:
        _check("b200k_gemm_epilogue_noalloc", library().b200k_gemm_epilogue_noalloc(ctypes.byref(g), _stream()))
    else:
        _check("b200k_gemm_epilogue", library().b200k_gemm_epilogue(ctypes.byref(g), _stream()))


def gemm_rope(a: torch.Tensor, b: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, out: torch.Tensor,
              tile_config: int = -1, status: torch.Tensor | None = None) -> None:
    """out[M,N] = rope(round(a @ b)) per 64-column head, output row m rotated
    by cos / sin row m % cos.shape[0] (b200k_gemm_rope)."""
    g = GemmArgs()
    M, K = a.shape
    N = b.shape[1]
    g.M, g.N, g.K = M, N, K
    g.a, g.a_stride_m, g.a_stride_k = a.data_ptr(), a.stride(0), a.stride(1)
    g.b, g.b_stride_k, g.b_stride_n = b.data_ptr(), b.stride(0), b.stride(1)
    g.ab_dtype = g.out_dtype = DTYPE[a.dtype]
    g.out, g.out_stride_m, g.out_stride_n = out.data_ptr(), out.stride(0), out.stride(1)
    g.tile_config = tile_config
    g.status = status.data_ptr() if status is not None else None
    r = RopeTables()
    r.cos, r.sin, r.stride, r.period = cos.data_ptr(), sin.data_ptr(), cos.stride(0), cos.shape[0]
    r.head_dim, r.dtype = cos.shape[1], DTYPE[cos.dtype]
    _check("b200k_gemm_rope", library().b200k_gemm_rope(ctypes.byref(g), ctypes.byref(r), _stream()))


def gemm_noalloc_status() -> int:
    """Status word of the last allocation-free GEMM on the current device
    (0 = ok, 6 = a device-side wait timed out); synchronises with the current
    stream."""
    v = ctypes.c_int32(-1)
    _check("b200k_gemm_noalloc_status", library().b200k_gemm_noalloc_status(ctypes.byref(v), _stream()))
    return int(v.value)


def rownorm(x: torch.Tensor, kind: int, weight, bias, eps: float, flags: int, out: torch.Tensor,
            mean_out=None, rstd_out=None) -> None:
    a = RowNormArgs()
    a.cols = x.shape[-1]
    a.rows = x.numel() // a.cols
    a.x = x.data_ptr()
    a.x_row_stride = x.stride(-2) if x.dim() > 1 else a.cols
    a.x_dtype = DTYPE[x.dtype]
    a.kind = kind
    if weight is not None:
        a.weight, a.w_dtype = weight.data_ptr(), DTYPE[weight.dtype]
    if bias is not None:
        a.bias, a.b_dtype = bias.data_ptr(), DTYPE[bias.dtype]
    a.flags = flags
    a.eps = eps
    a.out = out.data_ptr()
    a.out_row_stride = out.stride(-2) if out.dim() > 1 else out.shape[-1]
    a.out_dtype = DTYPE[out.dtype]
    a.mean_out = mean_out.data_ptr() if mean_out is not None else None
    a.rstd_out = rstd_out.data_ptr() if rstd_out is not None else None
    _check("b200k_rownorm", library().b200k_rownorm(ctypes.byref(a), _stream()))


def softmax(x: torch.Tensor, out: torch.Tensor, log: bool = False) -> None:
    a = SoftmaxArgs()
    a.cols = x.shape[-1]
    a.rows = x.numel() // a.cols
    a.x, a.x_row_stride, a.x_dtype = x.data_ptr(), (x.stride(-2) if x.dim() > 1 else a.cols), DTYPE[x.dtype]
    a.log_softmax = 1 if log else 0
    a.out, a.out_row_stride, a.out_dtype = out.data_ptr(), (out.stride(-2) if out.dim() > 1 else a.cols), DTYPE[out.dtype]
    _check("b200k_softmax", library().b200k_softmax(ctypes.byref(a), _stream()))


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, out: torch.Tensor) -> None:
    """out = x * cos + rotate_half(x) * sin (rank <= 4; cos / sin broadcast to x)."""
    c, sn = cos.expand(x.shape), sin.expand(x.shape)
    a = RopeArgs()
    pad = 4 - x.dim()
    for d in range(4):
        real = d >= pad
        a.sizes[d] = x.shape[d - pad] if real else 1
        a.x_strides[d] = x.stride(d - pad) if real else 0
        a.cos_strides[d] = c.stride(d - pad) if real else 0
        a.sin_strides[d] = sn.stride(d - pad) if real else 0
        a.out_strides[d] = out.stride(d - pad) if real else 0
    a.x, a.cos, a.sin, a.out = x.data_ptr(), c.data_ptr(), sn.data_ptr(), out.data_ptr()
    a.dtype = DTYPE[x.dtype]
    _check("b200k_rope", library().b200k_rope(ctypes.byref(a), _stream()))


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, causal: bool = False,
              scale: float = 0.0, status: torch.Tensor | None = None, timeout_ns: int = 0,
              test_flags: int = 0) -> None:
    """out = softmax(scale q k^T [causal mask]) v over [B, H, S, D] views
    (k, v with H / G heads)."""
    a = AttentionArgs()
    a.batch, a.heads, a.q_len, a.head_dim = q.shape
    a.kv_heads, a.kv_len = k.shape[1], k.shape[2]
    for dst, t in ((a.q_strides, q), (a.k_strides, k), (a.v_strides, v), (a.out_strides, out)):
        for d in range(4):
            dst[d] = t.stride(d)
    a.q, a.k, a.v, a.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    a.dtype = DTYPE[q.dtype]
    a.causal = 1 if causal else 0
    a.scale = scale
    a.test_flags = test_flags
    a.status = status.data_ptr() if status is not None else None
    a.timeout_ns = timeout_ns
    _check("b200k_attention", library().b200k_attention(ctypes.byref(a), _stream()))
