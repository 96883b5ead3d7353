"""GEMM + epilogue fusion pass: folds a pointwise group that consumes a matmul
into the matmul's epilogue, so the matmul result never goes to memory.

Same names, anchor rules and operand order as the reference
(compiler/optimization/fusion_epilogue.py): MATMUL_OPS / DOT_DTYPES (:22-23),
_is_static_cuda (:41-42), find_epilogue_anchor (:45-69), build_epilogue_op
(:154-180), _epilogue_is_faster (:207-234), fuse_epilogue (:237-265); the
rewritten node takes (mat1, mat2, bias?, *externals) like the reference's
closure (:247-256).  The lowering differs: the group becomes an
accumulator-machine program run by the persistent tcgen05 GEMM kernel in
libb200k.so (``torch.ops.b200.gemm_epilogue``), and the Triton autotuner is
replaced by the library's B200 tile table.

Documented extension (config.EXTENSIONS): the anchor may sit behind a
``view``/``_unsafe_view`` that only unflattens the matmul's rows, which is how
AOTAutograd lowers 3-d ``nn.Linear`` calls ([B,S,K] -> view -> mm -> view ->
pointwise).  The reference cannot anchor those (its anchor must be the
matmul itself and 2-d), so ViT/Llama-style models get no epilogue fusion
there.
"""
from __future__ import annotations

import math

import torch
import torch.fx as fx

from compiler import runtime

from . import config
from .fusion_pointwise import _tensor_meta, external_inputs, find_fusion_groups, new_kernel_name
from .program import ProgramError, canonical_form, compile_group

aten = torch.ops.aten
runtime.load()

MATMUL_OPS = (aten.addmm.default, aten.mm.default)
DOT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)
VIEW_OPS = (aten.view.default, aten._unsafe_view.default)


def _is_static_cuda(val) -> bool:
    return config.on_target_device(val) and all(isinstance(s, int) for s in val.shape)


def _kernel_supports(mat1, mat2, out_meta, extras_meta, out_shape) -> bool:
    """Layouts the sm_100a GEMM kernel accepts (checked on the fake values; a
    mismatch leaves the group to ATen at compile time, as the reference does
    for anything it cannot anchor)."""
    a, b = _tensor_meta(mat1), _tensor_meta(mat2)
    if a.dtype not in config.gemm_ab_dtypes() or out_meta.dtype not in config.GEMM_OUT_DTYPES:
        return False
    M, K = a.shape
    N = b.shape[1]
    if min(M, N, K) == 0:
        return False
    eb = a.element_size()
    a_k_major = a.stride(1) == 1 and (a.stride(0) * eb) % 16 == 0
    # M-major A (the transposed gradient of a weight-gradient GEMM in a
    # backward graph): 16-bit only, interpreted epilogue
    a_m_major = a.stride(0) == 1 and (a.stride(1) * eb) % 16 == 0 and eb == 2
    if not (a_k_major or a_m_major):
        return False
    k_major = b.stride(0) == 1 and (b.stride(1) * eb) % 16 == 0
    n_major = b.stride(1) == 1 and (b.stride(0) * eb) % 16 == 0 and eb == 2  # TF32 runs K-major B only
    if not (k_major or n_major):
        return False
    if len(extras_meta) > config.MAX_INPUTS - 1:
        return False
    for v in extras_meta:
        if v is None or not config.on_target_device(v) or v.dtype not in config.LOADABLE_DTYPES:
            return False
        if not _flattens(v, out_shape):
            return False
    return True


def _flattens(v: torch.Tensor, out_shape) -> bool:
    """True when v broadcast to out_shape indexes as [m, n] with the leading
    dims merged into m (what the kernel's (stride_m, stride_n) can express)."""
    try:
        e = v.expand(out_shape)
    except RuntimeError:
        return False
    r = len(out_shape)
    if r <= 2:
        return True
    expect = e.stride(r - 2) * out_shape[r - 2]
    for d in range(r - 3, -1, -1):
        if out_shape[d] != 1 and e.stride(d) != expect:
            return False
        expect *= out_shape[d]
    return True


def _anchor(group: list[fx.Node], inputs: list[fx.Node]):
    """(anchor input, matmul): the input through which the group reads the
    matmul result (the matmul itself, or with the extension a row-unflattening
    view of it), or (None, None)."""
    members = set(group)
    out_shape = _tensor_meta(group[-1]).shape
    for node in inputs:
        view = None
        mm = node
        if (
            config.EXTENSIONS
            and node.op == "call_function"
            and node.target in VIEW_OPS
            and isinstance(node.args[0], fx.Node)
            and node.args[0].op == "call_function"
            and node.args[0].target in MATMUL_OPS
        ):
            view, mm = node, node.args[0]
        if mm.op != "call_function" or mm.target not in MATMUL_OPS or mm.kwargs:
            continue  # kwargs means beta/alpha scaling; not handled
        mat1, mat2 = mm.args[-2:]
        val, a, b = _tensor_meta(mm), _tensor_meta(mat1), _tensor_meta(mat2)
        if val is None or a is None or b is None:
            continue
        if view is not None:
            vval = _tensor_meta(view)
            ok_view = (
                vval is not None
                and set(mm.users) == {view}
                and all(u in members for u in view.users)
                and val.dim() == 2
                and vval.dim() >= 2
                and vval.shape[-1] == val.shape[1]
                and math.prod(vval.shape[:-1]) == val.shape[0]
                and vval.shape == out_shape
            )
            if not ok_view:
                continue
        elif not (all(u in members for u in mm.users) and val.dim() == 2 and val.shape == out_shape):
            continue
        if (
            all(_is_static_cuda(t) for t in (val, a, b))
            and a.dtype == b.dtype
            and a.dtype in DOT_DTYPES
        ):
            return (view if view is not None else mm), mm
    return None, None


def find_epilogue_anchor(group: list[fx.Node], inputs: list[fx.Node]):
    """Return the matmul node whose output this group can consume straight
    from the accumulator, or None (reference :45-69)."""
    return _anchor(group, inputs)[1]


def build_epilogue_op(group, matmul, inputs, anchor=None):
    """Lower the group to (program, out_shape, out_dtype) for
    ``torch.ops.b200.gemm_epilogue``.  Slot 0 is the accumulator, slots 1..
    are ``inputs`` (bias first for addmm).  Raises ProgramError when the
    group does not fit the kernel's program limits."""
    anchor = matmul if anchor is None else anchor
    out_meta = _tensor_meta(group[-1])
    operands = [anchor] + list(inputs)
    prologue = None
    if matmul.target == aten.addmm.default:
        prologue = [("ADD", matmul.args[0])]  # acc + bias first (reference :142-143)
    prog = compile_group(group, operands, prologue=prologue, prologue_target=anchor,
                         rounding_casts=config.EXTENSIONS)
    return prog, [int(s) for s in out_meta.shape], out_meta.dtype


def _row_vector(n) -> bool:
    """An epilogue operand that broadcasts along the rows of the [M, N] output."""
    v = _tensor_meta(n) if isinstance(n, fx.Node) else None
    if v is None:
        return False
    shape = list(v.shape)
    return len(shape) <= 1 or all(s == 1 for s in shape[:-1])


def epilogue_form(prog, n_operands: int, operands=None) -> list[int]:
    """The kernel's compiled-path descriptor for this program ([] = interpret).
    ``operands`` (the extras, in slot order 1..) lets only row vectors take the
    bias role."""
    rv = None if operands is None else [False] + [_row_vector(n) for n in operands]
    form = canonical_form(prog, n_operands, rv) if config.FAST_EPILOGUE else None
    return form or []


# Cost model of the profitability rule, measured on one B200 (bf16, device
# time with CUDA-graph replay).  The library's GEMM against cuBLAS on the
# same plain problems: 16384x2048x2048 95.4 vs 97.4 us, 16384x8192x2048
# 364.8 vs 360.9, 12608x2304x768 (+bias) 42.2 vs 38.3, 8192^3 723.5 vs
# 681.6, 16384x128256x2048 6281 vs 6014.
GEMM_FLOPS = 1.5e15  # cuBLAS bf16 on large problems, FLOP/s
HBM_BYTES = 6.5e12   # measured copy bandwidth, B/s
LAUNCH_S = 4e-6      # one more kernel in a replayed graph


def library_over_cublas(K: int) -> float:
    """Measured time ratio of the library GEMM to cuBLAS by reduction depth:
    short main loops (K <= 1024) leave the library's per-tile latencies
    unhidden; from K = 4096 cuBLAS's 2x1 CTA-pair clusters share operands
    the library's pairs do not."""
    if K <= 1024:
        return 1.10
    return 1.0 if K < 4096 else 1.06


def fusion_pays(M: int, N: int, K: int, acc_bytes: int, out_bytes: int, extra_bytes: int) -> bool:
    """Predicted fused time <= predicted unfused time.  Unfused, ATen runs
    the GEMM (cuBLAS), which writes the M x N product, and then the
    pointwise group's kernel, which reads it back with the extra operands
    and writes the output.  Fused, the library's GEMM (its time ratio to
    cuBLAS above) applies the group in its epilogue; the extra operands are
    read under the MMAs."""
    # fp32 operands run at the TF32 rate, half the 16-bit one
    t_mm = 2.0 * M * N * K / (GEMM_FLOPS / 2 if acc_bytes == 4 else GEMM_FLOPS)
    tail = (2.0 * M * N * acc_bytes + M * N * out_bytes + extra_bytes) / HBM_BYTES + LAUNCH_S
    return library_over_cublas(K) * t_mm <= t_mm + tail


def _epilogue_is_faster(group, matmul, inputs) -> bool:
    """Profitability rule standing in for the reference's compile-time
    wall-clock race (:207-234): the cost model of ``fusion_pays`` on the
    group's shapes and dtypes."""
    mat1, mat2 = matmul.args[-2:]
    a, b, acc = _tensor_meta(mat1), _tensor_meta(mat2), _tensor_meta(matmul)
    out = _tensor_meta(group[-1])
    M, K = a.shape
    N = b.shape[1]
    extra = 0
    for n in inputs:
        v = _tensor_meta(n)
        if v is not None:
            extra += v.numel() * v.element_size()
    return fusion_pays(int(M), int(N), int(K), acc.element_size(), out.element_size(), extra)


def fuse_epilogue(gm: fx.GraphModule) -> fx.GraphModule:
    for group in find_fusion_groups(gm.graph):
        group_inputs = external_inputs(group)
        anchor, matmul = _anchor(group, group_inputs)
        if matmul is None:
            continue
        bias = [matmul.args[0]] if matmul.target == aten.addmm.default else []
        inputs = list(dict.fromkeys(bias + [n for n in group_inputs if n is not anchor]))
        mat1, mat2 = matmul.args[-2:]
        root = group[-1]
        out_meta = _tensor_meta(root)
        if not out_meta.is_contiguous():
            continue  # the kernel writes a row-major [M, N] output
        if not _kernel_supports(mat1, mat2, out_meta, [_tensor_meta(n) for n in inputs], out_meta.shape):
            continue
        try:
            prog, shape, dtype = build_epilogue_op(group, matmul, inputs, anchor)
        except ProgramError:
            continue
        if not _epilogue_is_faster(group, matmul, inputs):
            continue
        with gm.graph.inserting_before(root):
            new_node = gm.graph.call_function(
                torch.ops.b200.gemm_epilogue.default,
                (mat1, mat2, list(inputs), prog.code, prog.imm, shape, dtype,
                 epilogue_form(prog, 1 + len(inputs), list(inputs))),
            )
        new_node.meta = dict(root.meta)
        new_node.meta["b200_kernel"] = new_kernel_name("gemm_epilogue")
        new_node.meta["b200_group"] = [str(matmul.target)] + [str(n.target) for n in group]
        new_node.meta["b200_program"] = prog.listing()
        root.replace_all_uses_with(new_node)
        for n in reversed(group):  # consumers before producers
            gm.graph.erase_node(n)
        if anchor is not matmul:
            gm.graph.erase_node(anchor)
        gm.graph.erase_node(matmul)
    gm.graph.lint()
    gm.recompile()
    return gm
