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
    """The FakeTensor value AOTAutograd recorded for `node`, or None."""
    if not isinstance(node, fx.Node):
        return None
    val = node.meta.get("val")
    return val if isinstance(val, torch.Tensor) else None


def _is_float_cast(node: fx.Node) -> bool:
    """True for an ``aten._to_copy`` that only changes the dtype between two
    floating types no wider than fp32.

    The reference ends a group at a cast below fp32, because its kernel
    rounds only when it stores the result and ops after the cast would see
    the unrounded value (fusion_pointwise.py:44-58).  With the extensions on,
    the program rounds at the cast itself (ROUND_BF16/F16), so a narrowing
    cast may sit inside a group: bf16 chains such as cast -> gelu -> cast ->
    +residual become one kernel with eager's rounding."""
    if set(node.kwargs) != {"dtype"}:
        return False
    src, dst = _tensor_meta(node.args[0]), _tensor_meta(node)
    if src is None or dst is None or not src.is_floating_point():
        return False
    if src.dtype == torch.float64 or dst.dtype == torch.float64:
        return False
    if dst.dtype == torch.float32 or config.EXTENSIONS:
        return True
    # A narrowing cast must be the last node of its group.
    return all(not _is_fusible(user) for user in node.users)


def _is_fusible(node: fx.Node) -> bool:
    """An op of POINTWISE_OPS with a floating, statically shaped result on the
    target device (CUDA unless a test injects another predicate)."""
    if node.op != "call_function" or node.target not in POINTWISE_OPS:
        return False
    args_ok = _is_float_cast(node) if node.target == aten._to_copy.default else not node.kwargs
    if not args_ok:
        return False
    val = _tensor_meta(node)
    if val is None or not val.is_floating_point() or not config.on_target_device(val):
        return False
    return not any(isinstance(d, torch.SymInt) or not isinstance(d, int) for d in val.shape)


def find_fusion_groups(graph: fx.Graph) -> list[list[fx.Node]]:
    """Partition the fusible nodes of `graph` into single-output groups.

    Nodes are visited from the graph's end, so every consumer is placed
    before its producers.  A node joins the group that holds all of its
    users when there is exactly one such group and the node's shape equals
    that group's output shape; otherwise it opens a new group.  Because a
    node joins only when every user is already inside, no value but the
    group's last one is read outside it.  The grouping decisions, the order
    of the groups (by their output node, last first) and the order inside a
    group (graph order) are the reference's (fusion_pointwise.py:76-105);
    tests/test_passes.py checks them against its recorded groupings.
    """
    group_id: dict[fx.Node, int] = {}
    groups: list[list[fx.Node]] = []  # each filled consumers first
    for node in reversed(list(graph.nodes)):
        if not _is_fusible(node):
            continue
        user_groups = {group_id.get(user, -1) for user in node.users}
        joined = -1
        if len(user_groups) == 1:
            (gid,) = user_groups
            if gid >= 0 and _tensor_meta(node).shape == _tensor_meta(groups[gid][0]).shape:
                joined = gid
        if joined < 0:
            joined = len(groups)
            groups.append([])
        groups[joined].append(node)
        group_id[node] = joined
    return [g[::-1] for g in groups]


def external_inputs(group: list[fx.Node]) -> list[fx.Node]:
    """The values the group reads but does not compute, each listed once, in
    the order the group first reads them.  This order is the fused op's
    argument order (reference fusion_pointwise.py:108-113)."""
    inside = set(group)
    order: list[fx.Node] = []
    listed: set[fx.Node] = set()
    for node in group:
        for arg in node.all_input_nodes:
            if arg not in inside and arg not in listed:
                listed.add(arg)
                order.append(arg)
    return order


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
