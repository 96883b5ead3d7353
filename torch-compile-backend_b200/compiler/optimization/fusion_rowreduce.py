"""Row-reduction fusion pass (an extension: the reference has none).

The reference's POINTWISE_OPS (compiler/optimization/fusion_pointwise.py:12-30)
has no reductions and its groups must share one output shape (:93-97), so
RMSNorm, LayerNorm and softmax stay in ATen with only their pointwise
fragments fused (e.g. RMSNorm -> ATen pow, ATen mean, fused add+rsqrt,
fused x*r*w).  This pass recognises whole row groups in the decomposed ATen
graph and replaces each with one single-pass kernel from libb200k.so:

  RMSNorm      [_to_copy f32] -> pow 2 -> mean(-1, keepdim) -> add eps -> rsqrt
               -> mul x -> [_to_copy x.dtype] -> [mul weight]
                                        => torch.ops.b200.rms_norm
  RMSNorm + SwiGLU  the above -> split in halves g, u -> [_to_copy f32] ->
               sigmoid -> mul g -> [_to_copy] -> mul u
                                        => torch.ops.b200.rms_norm_swiglu
  LayerNorm    aten.native_layer_norm over the last dim
                                        => torch.ops.b200.layer_norm
  softmax      aten._softmax / aten._log_softmax over the last dim
                                        => torch.ops.b200.softmax / log_softmax

Rounding points of the decomposed graph (the casts to bf16/f16 between the
ops) are reproduced by the kernel's flags, so the fused result matches eager
PyTorch op for op.  A pattern fires only when every intermediate it removes
has no reader outside the pattern (training graphs that save them for the
backward keep the ATen ops).
"""
from __future__ import annotations

import torch
import torch.fx as fx

from compiler import runtime

from . import config
from .fusion_pointwise import _tensor_meta, new_kernel_name

aten = torch.ops.aten
runtime.load()

ROWF_ROUND_NORMED = 1
ROWF_ROUND_AFFINE = 2
ROWF_ROUND_SILU = 4

_CAST = aten._to_copy.default


def _only_user(n: fx.Node):
    return next(iter(n.users)) if len(n.users) == 1 else None


def _is(n, target) -> bool:
    return isinstance(n, fx.Node) and n.op == "call_function" and n.target == target


def _is_cast_to(n, dtype) -> bool:
    return _is(n, _CAST) and set(n.kwargs) == {"dtype"} and n.kwargs["dtype"] == dtype


def _last_dim_arg(dims, rank) -> bool:
    return isinstance(dims, (list, tuple)) and len(dims) == 1 and dims[0] in (-1, rank - 1)


def _rows_ok(v: torch.Tensor) -> bool:
    """On device, supported dtype, unit last-dim stride, leading dims flatten,
    row short enough for the register-resident kernels."""
    if v is None or not config.on_target_device(v) or v.dtype not in config.ROW_DTYPES or v.dim() < 1:
        return False
    if not all(isinstance(s, int) for s in v.shape):
        return False
    cols = v.shape[-1]
    if cols == 0 or (v.stride(-1) != 1 and cols != 1):
        return False
    if v.dim() >= 2:
        expect = v.stride(-2) * v.shape[-2]
        for d in range(v.dim() - 3, -1, -1):
            if v.shape[d] != 1 and v.stride(d) != expect:
                return False
            expect *= v.shape[d]
    return cols <= (32768 if cols % 8 == 0 else 4096)


def _other(node: fx.Node, known: fx.Node):
    a, b = node.args[:2]
    if a is known:
        return b
    if b is known:
        return a
    return None


def _match_rmsnorm(mean: fx.Node):
    """Returns (x, weight, eps, flags, out_node, removed_nodes) or None."""
    if not (_is(mean, aten.mean.dim) and len(mean.args) >= 3 and mean.args[2] is True and not mean.kwargs):
        return None
    p = mean.args[0]
    if not isinstance(p, fx.Node) or _only_user(p) is not mean:
        return None
    if _is(p, aten.pow.Tensor_Scalar) and p.args[1] == 2:
        x32 = p.args[0]
    elif _is(p, aten.mul.Tensor) and p.args[0] is p.args[1]:
        x32 = p.args[0]
    else:
        return None
    xv = _tensor_meta(x32)
    if xv is None or not _last_dim_arg(mean.args[1], xv.dim()):
        return None
    add = _only_user(mean)
    if not (_is(add, aten.add.Tensor) and add.args[0] is mean and isinstance(add.args[1], (int, float)) and not add.kwargs):
        return None
    eps = float(add.args[1])
    rs = _only_user(add)
    if not _is(rs, aten.rsqrt.default):
        return None
    n = _only_user(rs)
    if not (_is(n, aten.mul.Tensor) and _other(n, rs) is x32 and not n.kwargs):
        return None
    removed = [p, mean, add, rs, n]
    # x32 is either the input itself (fp32) or a cast of it read only here.
    if _is_cast_to(x32, torch.float32) and set(x32.users) <= {p, n}:
        x = x32.args[0]
        removed.insert(0, x32)
    else:
        x = x32
    xin = _tensor_meta(x)
    if not _rows_ok(xin) or xv.dtype != torch.float32:
        return None
    flags = 0
    out = n
    nxt = _only_user(n)
    if nxt is not None and _is_cast_to(nxt, xin.dtype) and xin.dtype != torch.float32:
        flags |= ROWF_ROUND_NORMED
        out = nxt
        removed.append(nxt)
        nxt = _only_user(nxt)
    weight = None
    if nxt is not None and _is(nxt, aten.mul.Tensor) and not nxt.kwargs:
        w = _other(nxt, out)
        wv = _tensor_meta(w) if isinstance(w, fx.Node) else None
        if (
            wv is not None
            and wv.dim() == 1
            and wv.shape[0] == xin.shape[-1]
            and wv.stride(0) == 1
            and wv.dtype in config.ROW_DTYPES
            and config.on_target_device(wv)
        ):
            weight = w
            out = nxt
            removed.append(nxt)
    if _tensor_meta(out).dtype not in config.ROW_DTYPES or not _tensor_meta(out).is_contiguous():
        return None
    return x, weight, eps, flags, out, removed


def _match_swiglu(y: fx.Node):
    """y -> split halves -> silu(g) * u.  Returns (out_node, flags, removed)."""
    yv = _tensor_meta(y)
    sp = _only_user(y)
    if sp is None or yv is None:
        return None
    cols = yv.shape[-1]
    if cols % 2:
        return None
    half = cols // 2
    if _is(sp, aten.split.Tensor):
        if not (sp.args[1] == half and (len(sp.args) < 3 or sp.args[2] in (-1, yv.dim() - 1))):
            return None
    elif _is(sp, aten.split_with_sizes.default):
        if not (list(sp.args[1]) == [half, half] and (len(sp.args) < 3 or sp.args[2] in (-1, yv.dim() - 1))):
            return None
    else:
        return None
    if len(sp.users) != 2:
        return None
    items = {}
    for u in sp.users:
        if not (u.op == "call_function" and u.target.__name__ == "getitem" and u.args[1] in (0, 1)):
            return None
        items[u.args[1]] = u
    g, up = items.get(0), items.get(1)
    if g is None or up is None or len(up.users) != 1:
        return None
    removed = [sp, g, up]
    flags = 0
    g32 = g
    if _is_cast_to(_only_user(g), torch.float32) and yv.dtype != torch.float32:
        g32 = _only_user(g)
        removed.append(g32)
    elif len(g.users) != 2:
        return None
    users = set(g32.users)
    sig = next((u for u in users if _is(u, aten.sigmoid.default)), None)
    if sig is None:
        return None
    mul = _only_user(sig)
    if not (_is(mul, aten.mul.Tensor) and _other(mul, sig) is g32 and users == {sig, mul}):
        return None
    removed += [sig, mul]
    s_out = mul
    nxt = _only_user(mul)
    if nxt is not None and _is_cast_to(nxt, yv.dtype) and yv.dtype != torch.float32:
        flags |= ROWF_ROUND_SILU
        s_out = nxt
        removed.append(nxt)
        nxt = _only_user(nxt)
    if not (nxt is not None and _is(nxt, aten.mul.Tensor) and _other(nxt, s_out) is up and _only_user(up) is nxt):
        return None
    out_v = _tensor_meta(nxt)
    if out_v is None or out_v.dtype != yv.dtype or not out_v.is_contiguous():
        return None
    if yv.dtype != torch.float32:
        flags |= ROWF_ROUND_AFFINE
    removed.append(nxt)
    return nxt, flags, removed


def _replace(gm: fx.GraphModule, out: fx.Node, target, args, removed, kind: str) -> None:
    with gm.graph.inserting_before(out):
        new = gm.graph.call_function(target, args)
    new.meta = dict(out.meta)
    new.meta["b200_kernel"] = new_kernel_name(kind)
    out.replace_all_uses_with(new)
    for n in sorted(set(removed), key=lambda n: -_order[n]):
        if not n.users:
            gm.graph.erase_node(n)


_order: dict[fx.Node, int] = {}


def fuse_rowreduce(gm: fx.GraphModule) -> fx.GraphModule:
    global _order
    _order = {n: i for i, n in enumerate(gm.graph.nodes)}
    for node in list(gm.graph.nodes):
        if node.graph is not gm.graph or node.op != "call_function":
            continue
        if node.target == aten.mean.dim:
            m = _match_rmsnorm(node)
            if m is None:
                continue
            x, w, eps, flags, out, removed = m
            sw = _match_swiglu(out)
            if sw is not None:
                sw_out, sw_flags, sw_removed = sw
                _replace(
                    gm, sw_out, torch.ops.b200.rms_norm_swiglu.default,
                    (x, w, eps, flags | sw_flags, _tensor_meta(sw_out).dtype), removed + sw_removed, "rms_norm_swiglu",
                )
            else:
                _replace(gm, out, torch.ops.b200.rms_norm.default, (x, w, eps, flags, _tensor_meta(out).dtype),
                         removed, "rms_norm")
        elif node.target == aten.native_layer_norm.default:
            x, shape, w, b, eps = node.args
            xv = _tensor_meta(x)
            ok = (
                _rows_ok(xv)
                and xv.is_contiguous()
                and list(shape) == [xv.shape[-1]]
                and all(
                    t is None
                    or (
                        _tensor_meta(t) is not None
                        and _tensor_meta(t).dim() == 1
                        and _tensor_meta(t).is_contiguous()
                        and _tensor_meta(t).dtype in config.ROW_DTYPES
                        and config.on_target_device(_tensor_meta(t))
                    )
                    for t in (w, b)
                )
            )
            if ok:
                node.target = torch.ops.b200.layer_norm.default
                node.meta["b200_kernel"] = new_kernel_name("layer_norm")
        elif node.target in (aten._softmax.default, aten._log_softmax.default):
            x, dim, half_to_float = node.args
            xv = _tensor_meta(x)
            if (_rows_ok(xv) and xv.is_contiguous() and dim in (-1, xv.dim() - 1)
                    and not (half_to_float and xv.dtype == torch.float32)):
                log = node.target == aten._log_softmax.default
                node.target = torch.ops.b200.log_softmax.default if log else torch.ops.b200.softmax.default
                node.meta["b200_kernel"] = new_kernel_name("log_softmax" if log else "softmax")
    gm.graph.lint()
    gm.recompile()
    return gm
