"""Rotary position embedding pass (an extension: the reference has none).

The rotate-half form of RoPE, ``x * cos + rotate_half(x) * sin`` with
``rotate_half(x) = cat(-x[..., D/2:], x[..., :D/2])``, decomposes into

    split(x, D/2, -1) | slice(x, -1, 0, D/2), slice(x, -1, D/2, end)
      -> neg(second half) -> cat([neg, first half], -1)
      -> mul(x, cos), mul(cat, sin) -> add

The reference's pointwise pass cannot take aten.cat (it is not in
POINTWISE_OPS, compiler/optimization/fusion_pointwise.py:12-30), so eager
execution and the reference run neg and cat as separate kernels and the
fused multiply-add reads the materialised rotation.  This pass replaces the
whole group with ``torch.ops.b200.rope``, one kernel that reads x, cos and
sin once and applies the same roundings (each product and the sum rounded to
the 16-bit type), so its result equals eager PyTorch bit for bit.  The
output keeps the decomposed graph's layout (``out_stride``).
"""
from __future__ import annotations

import operator

import torch
import torch.fx as fx

from compiler import runtime

from . import config
from .fusion_pointwise import _tensor_meta, new_kernel_name

aten = torch.ops.aten
runtime.load()

_END = 2**63 - 1


def _is(n, target) -> bool:
    return isinstance(n, fx.Node) and n.op == "call_function" and n.target == target


def _last_dim(dim, rank: int) -> bool:
    return dim in (-1, rank - 1)


def _halves(cat: fx.Node):
    """For cat([-x2, x1], -1) with x1, x2 the two halves of one x: (x, removed)."""
    if not (_is(cat, aten.cat.default) and len(cat.args) == 2 and not cat.kwargs):
        return None
    parts, dim = cat.args
    if not (isinstance(parts, (list, tuple)) and len(parts) == 2):
        return None
    neg, x1 = parts
    if not (_is(neg, aten.neg.default) and len(neg.users) == 1):
        return None
    x2 = neg.args[0]
    if not (isinstance(x1, fx.Node) and isinstance(x2, fx.Node)):
        return None
    # split(x, half, -1) -> getitem 0 (x1), getitem 1 (x2)
    if (x1.op == x2.op == "call_function" and x1.target is operator.getitem and x2.target is operator.getitem
            and x1.args[0] is x2.args[0] and x1.args[1] == 0 and x2.args[1] == 1):
        sp = x1.args[0]
        if not _is(sp, aten.split.Tensor) or len(sp.users) != 2:
            return None
        x = sp.args[0]
        xv = _tensor_meta(x)
        if xv is None or xv.dim() < 1:
            return None
        d = xv.shape[-1]
        sp_dim = sp.args[2] if len(sp.args) > 2 else 0
        if not (_last_dim(sp_dim, xv.dim()) and _last_dim(dim, xv.dim()) and d % 2 == 0 and sp.args[1] == d // 2):
            return None
        if len(x1.users) != 1 or len(x2.users) != 1:
            return None
        return x, [cat, neg, x1, x2, sp]
    # slice(x, -1, 0, half), slice(x, -1, half, end)
    if _is(x1, aten.slice.Tensor) and _is(x2, aten.slice.Tensor) and x1.args[0] is x2.args[0]:
        x = x1.args[0]
        xv = _tensor_meta(x)
        if xv is None or xv.dim() < 1:
            return None
        d = xv.shape[-1]
        a1 = list(x1.args) + [None] * (4 - len(x1.args))
        a2 = list(x2.args) + [None] * (4 - len(x2.args))
        ok = (
            _last_dim(a1[1], xv.dim()) and _last_dim(a2[1], xv.dim()) and _last_dim(dim, xv.dim())
            and d % 2 == 0 and a1[2] in (0, None) and a1[3] == d // 2
            and a2[2] == d // 2 and a2[3] in (d, _END, None)
        )
        if not ok or len(x1.users) != 1 or len(x2.users) != 1:
            return None
        return x, [cat, neg, x1, x2]
    return None


def _operands(mul: fx.Node, known: fx.Node):
    a, b = mul.args[:2]
    if a is known:
        return b
    if b is known:
        return a
    return None


def _supported(x, cos, sin, out) -> bool:
    vs = [_tensor_meta(n) for n in (x, cos, sin, out)]
    if any(v is None for v in vs):
        return False
    xv, cv, sv, ov = vs
    if xv.dtype not in (torch.bfloat16, torch.float16) or any(v.dtype != xv.dtype for v in (cv, sv, ov)):
        return False
    if not all(config.on_target_device(v) for v in vs):
        return False
    if xv.dim() > 4 or tuple(ov.shape) != tuple(xv.shape):
        return False
    for v in (cv, sv):  # broadcast to x
        if v.dim() > xv.dim() or any(a not in (1, b) for a, b in zip(reversed(v.shape), reversed(xv.shape))):
            return False
        if v.shape[-1] != xv.shape[-1]:
            return False
    return True


def fuse_rope(gm: fx.GraphModule) -> fx.GraphModule:
    order = {n: i for i, n in enumerate(gm.graph.nodes)}
    for add in list(gm.graph.nodes):
        if add.graph is not gm.graph or not _is(add, aten.add.Tensor) or add.kwargs or len(add.args) != 2:
            continue
        for m_cos, m_sin in (tuple(add.args), tuple(reversed(add.args))):
            if not (_is(m_cos, aten.mul.Tensor) and _is(m_sin, aten.mul.Tensor)) or m_cos is m_sin:
                continue
            if m_cos.kwargs or m_sin.kwargs or len(m_cos.users) != 1 or len(m_sin.users) != 1:
                continue
            cat = next((a for a in m_sin.args[:2] if _is(a, aten.cat.default)), None)
            h = _halves(cat) if cat is not None and len(cat.users) == 1 else None
            if h is None:
                continue
            x, removed = h
            sin = _operands(m_sin, cat)
            cos = _operands(m_cos, x)
            if not isinstance(sin, fx.Node) or not isinstance(cos, fx.Node) or not _supported(x, cos, sin, add):
                continue
            out_stride = [int(s) for s in _tensor_meta(add).stride()]
            with gm.graph.inserting_before(add):
                new = gm.graph.call_function(torch.ops.b200.rope.default, (x, cos, sin, out_stride))
            new.meta = dict(add.meta)
            new.meta["b200_kernel"] = new_kernel_name("rope")
            add.replace_all_uses_with(new)
            for n in sorted([add, m_cos, m_sin] + removed, key=lambda n: -order[n]):
                if not n.users:
                    gm.graph.erase_node(n)
            break
    gm.graph.lint()
    gm.recompile()
    return gm
