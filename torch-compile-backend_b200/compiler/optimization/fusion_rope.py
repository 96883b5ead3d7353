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


# ---------------------------------------------------------------- projection
# A rotation whose input is a projection viewed as heads,
#
#     mm(h, t(W)) -> [_unsafe_]view [B, S, H*64] -> view [B, S, H, 64]
#       -> transpose(1, 2) -> b200.rope(., cos [S, 64], sin [S, 64])
#
# (a Llama-style q or k projection), becomes one GEMM with the rotation as its
# epilogue, ``torch.ops.b200.gemm_rope`` (csrc/gemm_kernel.cuh, ROW_ROPE):
# the projection's 16-bit product is rotated in registers before its only
# store, so neither the product nor the rotation's input is written and read
# back.  The reference leaves the projection to ATen (its anchor needs a
# pointwise consumer, compiler/optimization/fusion_epilogue.py:45-69) and has
# no rotation kernel.  Taken when the library's cost model predicts the fused
# launch no slower than cuBLAS plus the rotation kernel.
_VIEWS = (aten.view.default, aten._unsafe_view.default, aten.reshape.default)


def _single_user(n: fx.Node) -> bool:
    return len(n.users) == 1


def _projection_of(x: fx.Node):
    """(mm node, removed nodes, B, S, H) when x = transpose(view(...mm...), 1, 2)."""
    if not (_is(x, aten.transpose.int) and _single_user(x) and tuple(x.args[1:]) in ((1, 2), (2, 1))):
        return None
    removed = [x]
    n = x.args[0]
    while isinstance(n, fx.Node) and any(_is(n, v) for v in _VIEWS) and _single_user(n):
        removed.append(n)
        n = n.args[0]
    if not (isinstance(n, fx.Node) and _is(n, aten.mm.default) and _single_user(n) and len(removed) >= 2):
        return None
    v4 = _tensor_meta(removed[1])  # the [B, S, H, 64] view
    if v4 is None or v4.dim() != 4:
        return None
    B, S, H, D = (int(d) for d in v4.shape)
    return n, removed, B, S, H, D


def _table2d(t: fx.Node, S: int):
    """The [S, 64] table behind a cos / sin operand broadcast over batch and heads."""
    v = _tensor_meta(t)
    if v is None or v.dim() < 2 or tuple(v.shape[-2:]) != (S, 64) or any(d != 1 for d in v.shape[:-2]):
        return None
    if v.stride(-1) != 1 or v.stride(-2) % 8 or v.storage_offset() % 8:
        return None
    return v


def fuse_gemm_rope(gm: fx.GraphModule) -> fx.GraphModule:
    from .fusion_epilogue import fusion_pays

    for node in list(gm.graph.nodes):
        if node.graph is not gm.graph or not _is(node, torch.ops.b200.rope.default):
            continue
        x, cos, sin = node.args[:3]
        proj = _projection_of(x) if isinstance(x, fx.Node) else None
        if proj is None:
            continue
        mm, removed, B, S, H, D = proj
        a, b = mm.args
        av, bv, outv = _tensor_meta(a), _tensor_meta(b), _tensor_meta(node)
        if av is None or bv is None or outv is None or D != 64:
            continue
        M, K = (int(d) for d in av.shape)
        N = int(bv.shape[1])
        if M != B * S or N != H * D or av.dtype not in (torch.bfloat16, torch.float16) or bv.dtype != av.dtype:
            continue
        if not (config.on_target_device(av) and config.on_target_device(bv)):
            continue
        if av.stride(1) != 1 or (av.stride(0) * 2) % 16 or bv.stride(0) != 1 or (bv.stride(1) * 2) % 16:
            continue
        if tuple(outv.stride()) != (S * N, D, N, 1):  # the rotation keeps the heads view of a row-major product
            continue
        cv, sv = _table2d(cos, S), _table2d(sin, S)
        if cv is None or sv is None or cv.dtype != av.dtype or sv.dtype != av.dtype or cv.stride(-2) != sv.stride(-2):
            continue
        if not fusion_pays(M, N, K, 2, 2, 2 * S * 64 * 2):
            continue
        with gm.graph.inserting_before(node):
            c2 = cos if cv.dim() == 2 else gm.graph.call_function(aten.view.default, (cos, [S, 64]))
            s2 = sin if sv.dim() == 2 else gm.graph.call_function(aten.view.default, (sin, [S, 64]))
            g = gm.graph.call_function(torch.ops.b200.gemm_rope.default, (a, b, c2, s2, S, [B, S, N]))
            v = gm.graph.call_function(aten.view.default, (g, [B, S, H, D]))
            t = gm.graph.call_function(aten.transpose.int, (v, 1, 2))
        for n_new in (c2, s2):
            if n_new is not cos and n_new is not sin:
                n_new.meta["val"] = _tensor_meta(n_new.args[0]).view(S, 64)
        g.meta["val"] = av.new_empty((B, S, N))
        g.meta["b200_kernel"] = new_kernel_name("gemm_rope")
        g.meta["b200_group"] = [str(mm.target), str(node.target)]
        v.meta["val"] = g.meta["val"].view(B, S, H, D)
        t.meta = dict(node.meta)
        t.meta.pop("b200_kernel", None)
        t.meta["val"] = v.meta["val"].transpose(1, 2)
        node.replace_all_uses_with(t)
        gm.graph.erase_node(node)
        for n in removed:
            if not n.users:
                gm.graph.erase_node(n)
        if not mm.users:
            gm.graph.erase_node(mm)
    gm.graph.lint()
    gm.recompile()
    return gm
