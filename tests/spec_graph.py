"""Rebuild an FX group from a recorded spec (tests/golden/reference_kernels.json)
so the product's lowering (compile_group) can be applied to it."""
from __future__ import annotations

import torch
import torch.fx as fx

aten = torch.ops.aten


def target_of(name: str):
    op, overload = name.split(".")
    return getattr(getattr(aten, op), overload)


def build(spec, n_inputs: int, with_acc: bool = False):
    """Returns (group nodes, operand nodes).  For a GEMM-epilogue spec the
    accumulator is operand 0 and inputs follow (slot i+1)."""
    g = fx.Graph()
    acc = g.placeholder("acc") if with_acc else None
    ins = [g.placeholder(f"in{i}") for i in range(n_inputs)]
    nodes = []
    for op, args in spec:
        fargs = []
        kwargs = {}
        for a in args:
            if isinstance(a, list) and a[0] == "in":
                fargs.append(ins[a[1]])
            elif isinstance(a, list) and a[0] == "node":
                fargs.append(nodes[a[1]])
            elif isinstance(a, list) and a[0] == "acc":
                fargs.append(acc)
            elif isinstance(a, str):
                kwargs["dtype"] = getattr(torch, a)
            else:
                fargs.append(a)
        nodes.append(g.call_function(target_of(op), tuple(fargs), kwargs))
    g.output(nodes[-1])
    operands = ([acc] if with_acc else []) + ins
    return nodes, operands
