"""Test helpers: run the backend's passes on a model's ATen graph without
executing the fused ops (so graph-level tests run on a CPU-only machine)."""
from __future__ import annotations

import contextlib
import copy

import torch
from torch._decomp import get_decompositions
from torch._dynamo.backends.common import aot_autograd
from torch._functorch.aot_autograd import make_boxed_func

from compiler import backend as B
from compiler.optimization import config


@contextlib.contextmanager
def cpu_target(extensions: bool = True):
    """Let the passes fire on CPU tensors (the device predicate) and pick the
    extension setting; restores both afterwards."""
    old_pred = config.set_device_predicate(lambda v: True)
    old_ext = config.EXTENSIONS
    config.EXTENSIONS = extensions
    try:
        yield
    finally:
        config.set_device_predicate(old_pred)
        config.EXTENSIONS = old_ext


def fused_graphs(model, inputs, extensions: bool = True):
    """Compile `model` with a backend that runs the passes on a copy of each
    graph and executes the original graph eagerly.  Returns the rewritten
    forward graphs."""
    captured = []

    def cap(gm, example_inputs):
        g2 = copy.deepcopy(gm)
        B.compiler(g2, example_inputs)
        captured.append(g2)
        return make_boxed_func(gm.forward)

    be = aot_autograd(fw_compiler=cap, decompositions=get_decompositions([torch.ops.aten.gelu, torch.ops.aten.silu]))
    torch._dynamo.reset()
    with cpu_target(extensions), torch.no_grad():
        torch.compile(model, backend=be)(*inputs)
    return captured


def kernels_of(gm) -> list[tuple[str, list[str], object]]:
    """(kind, group op names, node) for every fused node, in creation order."""
    out = []
    for n in gm.graph.nodes:
        name = n.meta.get("b200_kernel")
        if not name:
            continue
        kind, idx = name.rsplit("_", 1)
        ops = n.meta.get("b200_group", [])
        if kind == "gemm_epilogue":
            ops = ops[1:]  # drop the matmul itself
        out.append((int(idx), "pointwise" if kind == "fused" else kind, ops, n))
    return [(k, o, n) for _, k, o, n in sorted(out, key=lambda t: t[0])]


def capturing_backend():
    """A backend identical to custom_backend that also keeps each compiled
    (rewritten) graph, for tests that run on the GPU and inspect the graph."""
    graphs = []

    def comp(gm, example_inputs):
        f = B.compiler(gm, example_inputs)
        graphs.append(gm)
        return f

    be = aot_autograd(fw_compiler=comp, bw_compiler=comp,
                      decompositions=get_decompositions([torch.ops.aten.gelu, torch.ops.aten.silu]))
    return be, graphs


def b200_targets(graphs) -> list:
    return [n.target for gm in graphs for n in gm.graph.nodes
            if n.op == "call_function" and str(n.target).startswith("b200.")]
