"""Pointwise fusion pass: groups chains of elementwise ATen ops and replaces
each group of >= 2 ops with one call of the sm_100a pointwise kernel.

Same public names, grouping rules and argument order as the reference
(compiler/optimization/fusion_pointwise.py): POINTWISE_OPS (:12-30),
_is_float_cast / _is_fusible (:44-73), find_fusion_groups (:76-105),
external_inputs (:108-113), build_fused_op (:189-210), fuse_pointwise
(:213-231).  What differs is the lowering: instead of writing Triton source to
a temp file and importing it (:132-186), a group becomes an accumulator-machine
program (optimization/program.py) passed as data to
``torch.ops.b200.pointwise``.  The kernel library turns that program into
straight-line CUDA C and compiles it for sm_100a with NVRTC on first use
(csrc/pointwise_jit.cu), or interprets it where a launch is outside the
generated kernels' scope (csrc/pointwise.cu).
"""
from __future__ import annotations

import torch
import torch.fx as fx

from compiler import runtime

from . import config
from .program import BINARY, CAST, UNARY, ProgramError, compile_group

aten = torch.ops.aten
runtime.load()

# The fusible ops, as in the reference; the value is the kernel-side op name.
POINTWISE_OPS = {
    aten.add.Tensor: "ADD",
    aten.sub.Tensor: "SUB",
    aten.mul.Tensor: "MUL",
    aten.div.Tensor: "DIV",
    aten.neg.default: "NEG",
    aten.abs.default: "ABS",
    aten.relu.default: "RELU",
    aten.exp.default: "EXP",
    aten.log.default: "LOG",
    aten.sqrt.default: "SQRT",
    aten.rsqrt.default: "RSQRT",
    aten.erf.default: "ERF",
    aten.sigmoid.default: "SIGMOID",
    aten.tanh.default: "TANH",  # 2*sigmoid(2x)-1, as the reference computes it
    aten.maximum.default: "MAX",
    aten.minimum.default: "MIN",
    aten._to_copy.default: "CAST",
}
assert set(POINTWISE_OPS) == set(BINARY) | set(UNARY) | {CAST}

_fused_counter = 0


def _tensor_meta(node):
    val = node.meta.get("val") if isinstance(node, fx.Node) else None
    return val if isinstance(val, torch.Tensor) else None


def _is_float_cast(node: fx.Node) -> bool:
    """A dtype conversion between floats that fit in fp32.  In the reference a
    cast below fp32 must end its group: only the final store rounds, so ops
    after it would see the unrounded value (reference :67-79).  With the
    extensions on, the kernel rounds at the cast itself (ROUND_BF16/F16), so
    such a cast may sit inside a group and bf16 chains like
    cast -> gelu -> cast -> +residual stay one kernel with eager's rounding."""
    src, dst = _tensor_meta(node.args[0]), _tensor_meta(node)
    return (
        set(node.kwargs) == {"dtype"}
        and src is not None
        and dst is not None
        and src.is_floating_point()
        and torch.float64 not in (src.dtype, dst.dtype)
        and (
            dst.dtype == torch.float32
            or config.EXTENSIONS
            or not any(_is_fusible(u) for u in node.users)
        )
    )


def _is_fusible(node: fx.Node) -> bool:
    if node.op != "call_function" or node.target not in POINTWISE_OPS:
        return False
    if node.target == aten._to_copy.default:
        if not _is_float_cast(node):
            return False
    elif node.kwargs:
        return False
    val = _tensor_meta(node)
    return (
        val is not None
        and config.on_target_device(val)
        and val.is_floating_point()
        and all(isinstance(s, int) for s in val.shape)  # static shapes only
    )


def find_fusion_groups(graph: fx.Graph) -> list[list[fx.Node]]:
    """Walk the graph backwards and pull each fusible node into its
    consumers' group when (a) all of its users are in that one group and
    (b) it has the group's output shape.  (a) keeps every group
    single-output.  Groups come back in topological order (reference
    :99-128)."""
    group_of: dict[fx.Node, list[fx.Node]] = {}
    for node in reversed(graph.nodes):
        if not _is_fusible(node):
            continue
        consumer_groups = [group_of.get(u) for u in node.users]
        group = consumer_groups[0] if consumer_groups else None
        if (
            group is not None
            and all(g is group for g in consumer_groups)
            and _tensor_meta(node).shape == _tensor_meta(group[0]).shape
        ):
            group.append(node)
        else:
            group = [node]
        group_of[node] = group

    order = {n: i for i, n in enumerate(graph.nodes)}
    groups = {id(g): g for g in group_of.values()}.values()
    return [sorted(g, key=order.__getitem__) for g in groups]


def external_inputs(group: list[fx.Node]) -> list[fx.Node]:
    """Nodes the group reads from outside, deduplicated, in first-use order."""
    members = set(group)
    return list(dict.fromkeys(arg for node in group for arg in node.all_input_nodes if arg not in members))


def new_kernel_name(prefix: str) -> str:
    global _fused_counter
    _fused_counter += 1
    return f"{prefix}_{_fused_counter - 1}"


def _inputs_supported(inputs: list[fx.Node], out_rank: int) -> bool:
    if len(inputs) > config.MAX_INPUTS or out_rank > config.MAX_DIMS:
        return False
    for n in inputs:
        v = _tensor_meta(n)
        if v is None or not config.on_target_device(v) or v.dtype not in config.LOADABLE_DTYPES:
            return False
    return True


def _dense(v: torch.Tensor) -> bool:
    """Non-overlapping and dense: a permutation of a contiguous layout."""
    dims = sorted((d for d in range(v.dim()) if v.shape[d] != 1), key=lambda d: v.stride(d))
    expect = 1
    for d in dims:
        if v.stride(d) != expect:
            return False
        expect *= v.shape[d]
    return True


def build_fused_op(group: list[fx.Node], inputs: list[fx.Node]):
    """The lowered form of a group: (target op, constant args) for
    ``torch.ops.b200.pointwise(inputs, code, imm, out_shape, out_dtype)``.
    Raises ProgramError when the group does not fit the kernel."""
    out_meta = _tensor_meta(group[-1])
    prog = compile_group(group, inputs, rounding_casts=config.EXTENSIONS)
    shape, dtype = [int(s) for s in out_meta.shape], out_meta.dtype
    return prog, shape, dtype


def fuse_pointwise(gm: fx.GraphModule) -> fx.GraphModule:
    for group in find_fusion_groups(gm.graph):
        if len(group) < 2:  # a single op gains nothing; leave it to ATen
            continue
        inputs = external_inputs(group)
        root = group[-1]
        out_meta = _tensor_meta(root)
        if out_meta.dtype not in config.STORABLE_DTYPES or not _inputs_supported(inputs, out_meta.dim()):
            continue
        try:
            prog, shape, dtype = build_fused_op(group, inputs)
        except ProgramError:
            continue
        # Keep the layout the ATen ops would have produced (they follow their
        # inputs' memory order); later views in the graph may rely on it.
        if out_meta.is_contiguous():
            stride = []
        elif _dense(out_meta):
            stride = [int(s) for s in out_meta.stride()]
        else:
            continue
        with gm.graph.inserting_before(root):
            new_node = gm.graph.call_function(
                torch.ops.b200.pointwise.default, (list(inputs), prog.code, prog.imm, shape, dtype, stride)
            )
        new_node.meta = dict(root.meta)
        new_node.meta["b200_kernel"] = new_kernel_name("fused")
        new_node.meta["b200_group"] = [str(n.target) for n in group]
        new_node.meta["b200_program"] = prog.listing()
        root.replace_all_uses_with(new_node)
        for n in reversed(group):  # consumers before producers
            gm.graph.erase_node(n)
    gm.graph.lint()
    gm.recompile()
    return gm
