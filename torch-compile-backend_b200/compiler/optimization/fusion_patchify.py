"""Patch-embedding lowering (an extension: the reference has none).

A convolution whose kernel equals its stride, with no padding, dilation or
groups (ViT's patch embedding: 16x16 kernel, stride 16) is a matrix product
over non-overlapping patches.  The reference backend leaves aten.convolution
to ATen, where cuDNN runs it as an implicit-GEMM convolution with layout
conversions around it.  This pass rewrites the node as ATen ops the rest of
the backend already handles:

    x [B, C, H, W] -> view [B, C, Hp, k, Wp, k] -> permute -> contiguous
      -> view [B*Hp*Wp, C*k*k]                          (im2col, one copy)
    addmm(bias, patches, w.view(OC, C*k*k).t())         (a tensor-core GEMM)
    -> view [B, Hp, Wp, OC] -> permute -> contiguous -> [B, OC, Hp, Wp]

The result has the convolution's NCHW layout, so every node after it keeps
the shapes and strides it was traced with.  When the convolution's only use
is the patch-embedding idiom `flatten(2).transpose(1, 2)` (a view to
[B, OC, Hp*Wp], then a transpose to [B, Hp*Wp, OC]), the GEMM's row-major
[B*Hp*Wp, OC] output already is that token-major tensor: the transpose's
users get a view of it, and neither the NCHW copy nor the strided read of a
transposed view downstream (ViT's class-token concatenation) remains.  The
GEMM is then a candidate for the epilogue pass like any other addmm.
"""
from __future__ import annotations

import torch
import torch.fx as fx

from . import config
from .fusion_pointwise import _tensor_meta

aten = torch.ops.aten


def _match(conv: fx.Node):
    if conv.op != "call_function" or conv.target != aten.convolution.default or conv.kwargs:
        return None
    x, w, b, stride, padding, dilation, transposed, output_padding, groups = conv.args
    xv, wv, ov = _tensor_meta(x), _tensor_meta(w), _tensor_meta(conv)
    if xv is None or wv is None or ov is None or xv.dim() != 4 or wv.dim() != 4:
        return None
    oc, c, kh, kw = (int(s) for s in wv.shape)
    bsz, cx, h, wd = (int(s) for s in xv.shape)
    ok = (
        not transposed and groups == 1 and list(stride) == [kh, kw] and list(padding) == [0, 0]
        and list(dilation) == [1, 1] and cx == c and h % kh == 0 and wd % kw == 0
        and xv.is_contiguous() and wv.is_contiguous() and ov.is_contiguous()
        and xv.dtype == wv.dtype and xv.dtype in (torch.bfloat16, torch.float16)
        and config.on_target_device(xv) and config.on_target_device(wv)
        and (b is None or (_tensor_meta(b) is not None and _tensor_meta(b).dtype == xv.dtype))
    )
    if not ok:
        return None
    return x, w, b, (bsz, c, h // kh, kh, wd // kw, kw, oc)


def _token_major_use(conv: fx.Node, bsz: int, oc: int, hw: int):
    """(view, transpose) when the convolution's only use is
    view([B, OC, Hp*Wp]) whose only use is transpose(1, 2) (or the equal
    permute), i.e. `conv(x).flatten(2).transpose(1, 2)`; else None."""
    if len(conv.users) != 1:
        return None
    v = next(iter(conv.users))
    vv = _tensor_meta(v)
    if (v.op != "call_function" or v.target not in (aten.view.default, aten._unsafe_view.default)
            or len(v.users) != 1 or vv is None or tuple(vv.shape) != (bsz, oc, hw)):
        return None
    t = next(iter(v.users))
    if t.op != "call_function":
        return None
    if t.target == aten.transpose.int and len(t.args) == 3 and sorted(int(d) % 3 for d in t.args[1:]) == [1, 2]:
        return v, t
    if t.target == aten.permute.default and [int(d) % 3 for d in t.args[1]] == [0, 2, 1]:
        return v, t
    return None


def _emit(gm: fx.GraphModule, target, args, kwargs=None) -> fx.Node:
    """Insert a call and give it the fake value it computes (meta['val'])."""
    n = gm.graph.call_function(target, tuple(args), kwargs or {})

    def val(a):
        if isinstance(a, fx.Node):
            return a.meta["val"]
        if isinstance(a, (list, tuple)):
            return type(a)(val(x) for x in a)
        return a

    vals = [val(a) for a in args]
    flat = [v for x in vals for v in (x if isinstance(x, (list, tuple)) else [x])]
    fake = next(v for v in flat if isinstance(v, torch.Tensor))
    mode = getattr(fake, "fake_mode", None)
    if mode is not None:
        with mode:
            n.meta["val"] = target(*vals, **(kwargs or {}))
    else:  # real example values (tests without fake tracing)
        n.meta["val"] = target(*vals, **(kwargs or {}))
    return n


def fuse_patchify(gm: fx.GraphModule) -> fx.GraphModule:
    for conv in list(gm.graph.nodes):
        m = _match(conv)
        if m is None:
            continue
        x, w, b, (bsz, c, hp, kh, wp, kw, oc) = m
        tok = _token_major_use(conv, bsz, oc, hp * wp)
        with gm.graph.inserting_before(conv):
            xv = _emit(gm, aten.view.default, [x, [bsz, c, hp, kh, wp, kw]])
            xp = _emit(gm, aten.permute.default, [xv, [0, 2, 4, 1, 3, 5]])
            xc = _emit(gm, aten.clone.default, [xp], {"memory_format": torch.contiguous_format})
            a = _emit(gm, aten.view.default, [xc, [bsz * hp * wp, c * kh * kw]])
            w2 = _emit(gm, aten.view.default, [w, [oc, c * kh * kw]])
            wt = _emit(gm, aten.t.default, [w2])
            y = _emit(gm, aten.addmm.default, [b, a, wt]) if b is not None else _emit(gm, aten.mm.default, [a, wt])
            if tok is None:
                y4 = _emit(gm, aten.view.default, [y, [bsz, hp, wp, oc]])
                yp = _emit(gm, aten.permute.default, [y4, [0, 3, 1, 2]])
                out = _emit(gm, aten.clone.default, [yp], {"memory_format": torch.contiguous_format})
            else:
                out = _emit(gm, aten.view.default, [y, [bsz, hp * wp, oc]])
        if tok is None:
            out.meta = {**conv.meta, "val": out.meta["val"]}
            conv.replace_all_uses_with(out)
            gm.graph.erase_node(conv)
        else:
            v, t = tok
            out.meta = {**t.meta, "val": out.meta["val"]}
            t.replace_all_uses_with(out)
            for n in (t, v, conv):
                gm.graph.erase_node(n)
    gm.graph.lint()
    gm.recompile()
    return gm
