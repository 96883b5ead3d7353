"""Attention pass (an extension): replaces ATen's scaled-dot-product
attention node with ``torch.ops.b200.attention``, the library's tcgen05
attention kernel (csrc/attention.cu).

The reference leaves attention to ATen: its pointwise op table
(compiler/optimization/fusion_pointwise.py:12-30) has no attention entry, so
``aten._scaled_dot_product_{flash,cudnn,efficient}_attention`` stay in the
graph and run cuDNN or PyTorch's flash kernels.  This pass takes such a node
when the kernel covers it:

* inference only: of the node's outputs, only the attention output itself is
  read (training graphs also read the log-sum-exp for the backward pass);
* no dropout, no attention mask or bias; causal or not;
* q [B, H, S, 64], k and v [B, H / G, S_kv, 64] (grouped-query attention
  when G > 1), all bf16 or all f16, unit stride along the head dim and
  16-byte aligned rows;
* the output keeps the replaced node's layout.
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

SDPA_OPS = tuple(
    op for op in (
        getattr(aten, "_scaled_dot_product_flash_attention", None),
        getattr(aten, "_scaled_dot_product_cudnn_attention", None),
        getattr(aten, "_scaled_dot_product_efficient_attention", None),
        getattr(aten, "_scaled_dot_product_flash_attention_for_cpu", None),
    ) if op is not None
)
SDPA_OVERLOADS = tuple(op.default for op in SDPA_OPS)
HEAD_DIM = 64
DTYPES = (torch.bfloat16, torch.float16)


def _bound_args(node: fx.Node) -> dict:
    """The node's arguments by schema name, defaults filled in."""
    schema = node.target._schema
    out = {}
    for i, arg in enumerate(schema.arguments):
        if i < len(node.args):
            out[arg.name] = node.args[i]
        elif arg.name in node.kwargs:
            out[arg.name] = node.kwargs[arg.name]
        elif arg.has_default_value():
            out[arg.name] = arg.default_value
        else:
            out[arg.name] = None
    return out


def _layout_ok(v: torch.Tensor) -> bool:
    return (
        v is not None
        and v.dim() == 4
        and v.dtype in DTYPES
        and config.on_target_device(v)
        and all(isinstance(s, int) for s in v.shape)
        and v.shape[-1] == HEAD_DIM
        and v.stride(-1) == 1
        and all(v.stride(d) % 8 == 0 for d in range(3))
        and v.storage_offset() % 8 == 0
    )


def attention_replacement(node: fx.Node):
    """(q, k, v, causal, scale, out_stride, output-0 getitem nodes) when the
    kernel covers this SDPA node, else None."""
    if node.op != "call_function" or node.target not in SDPA_OVERLOADS:
        return None
    a = _bound_args(node)
    if a.get("dropout_p") not in (None, 0.0, 0):
        return None
    if a.get("attn_bias") is not None or a.get("attn_mask") is not None:
        return None
    if a.get("return_debug_mask"):
        return None
    q, k, v = a["query"], a["key"], a["value"]
    if not all(isinstance(t, fx.Node) for t in (q, k, v)):
        return None
    users = list(node.users)
    if not users or not all(u.op == "call_function" and u.target is operator.getitem and u.args[1] == 0
                            for u in users):
        return None
    qv, kv, vv = (_tensor_meta(t) for t in (q, k, v))
    if not all(_layout_ok(t) for t in (qv, kv, vv)):
        return None
    if not (qv.dtype == kv.dtype == vv.dtype and kv.shape == vv.shape):
        return None
    if qv.shape[0] != kv.shape[0] or qv.shape[1] % kv.shape[1] != 0:
        return None
    out = _tensor_meta(users[0])
    if out is None or tuple(out.shape) != tuple(qv.shape) or out.stride(-1) != 1 or \
            any(out.stride(d) % 8 for d in range(3)):
        return None
    scale = a.get("scale")
    scale = float(scale) if scale is not None else -1.0
    return q, k, v, bool(a.get("is_causal") or False), scale, [int(s) for s in out.stride()], users


def fuse_attention(gm: fx.GraphModule) -> fx.GraphModule:
    for node in list(gm.graph.nodes):
        rep = attention_replacement(node)
        if rep is None:
            continue
        q, k, v, causal, scale, stride, users = rep
        with gm.graph.inserting_before(node):
            new_node = gm.graph.call_function(torch.ops.b200.attention.default, (q, k, v, causal, scale, stride))
        new_node.meta = dict(users[0].meta)
        new_node.meta["b200_kernel"] = new_kernel_name("attention")
        new_node.meta["b200_group"] = [str(node.target)]
        for u in users:
            u.replace_all_uses_with(new_node)
            gm.graph.erase_node(u)
        gm.graph.erase_node(node)
    gm.graph.lint()
    gm.recompile()
    return gm
