"""Oracle for the fused pointwise kernel -- test infrastructure only.

Restates the reference's generated elementwise kernel
(compiler/optimization/fusion_pointwise.py:132-169): every external input is
read at the output index through its own broadcast strides and converted to
fp32 (:162-165), the group's ops run in fp32 one after another with the
expressions of POINTWISE_OPS (:12-30), Python scalars are fp32 constants
(:123), and the single store rounds to the output dtype (:168).
"""
from __future__ import annotations

import numpy as np

from .bf16 import round_to

F32 = np.float32


def _sigmoid(a):
    # tl.sigmoid: 1 / (1 + exp(-x))
    with np.errstate(over="ignore"):
        return (F32(1.0) / (F32(1.0) + np.exp(-a))).astype(F32)


def _tanh(a):
    # fusion_pointwise.py:26 -- tanh is computed as 2*sigmoid(2x) - 1.
    return (F32(2.0) * _sigmoid(F32(2.0) * a) - F32(1.0)).astype(F32)


def _erf(a):
    try:
        from scipy.special import erf
    except ImportError:  # pragma: no cover
        from math import erf as _e

        erf = np.vectorize(lambda t: _e(float(t)), otypes=[np.float64])
    return np.asarray(erf(np.asarray(a, dtype=np.float64))).astype(F32)


def _fmax(a, b):
    # tl.maximum / tl.minimum default: the non-NaN operand wins (IEEE maxNum).
    return np.fmax(a, b).astype(F32)


def _fmin(a, b):
    return np.fmin(a, b).astype(F32)


# aten op name (as in str(node.target) without the 'aten.' prefix) -> fp32 function.
OPS = {
    "add.Tensor": lambda a, b: (a + b).astype(F32),
    "sub.Tensor": lambda a, b: (a - b).astype(F32),
    "mul.Tensor": lambda a, b: (a * b).astype(F32),
    "div.Tensor": lambda a, b: (a / b).astype(F32),
    "neg.default": lambda a: (-a).astype(F32),
    "abs.default": lambda a: np.abs(a).astype(F32),
    "relu.default": lambda a: _fmax(a, F32(0.0)),
    "exp.default": lambda a: np.exp(a).astype(F32),
    "log.default": lambda a: np.log(a).astype(F32),
    "sqrt.default": lambda a: np.sqrt(a).astype(F32),
    "rsqrt.default": lambda a: (F32(1.0) / np.sqrt(a)).astype(F32),
    "erf.default": _erf,
    "sigmoid.default": _sigmoid,
    "tanh.default": _tanh,
    "maximum.default": _fmax,
    "minimum.default": _fmin,
    "_to_copy.default": lambda a, *dtype: a,  # identity in-kernel; the store rounds
}


def eval_group(spec, inputs, out_shape, out_dtype: str, acc=None, bias=None):
    """Evaluate a fused group.

    spec: [(op_name, args)] in topological order; args are ('in', i),
          ('node', j) or a float (a trailing dtype string on _to_copy).
    inputs: arrays broadcastable to out_shape (any float/int dtype).
    acc: for a GEMM epilogue, the fp32 accumulator standing for ('acc',);
         bias (optional) is added to it first (fusion_epilogue.py:142-143).
    Returns the result rounded to out_dtype (as fp32, or fp64 for fp64).
    """
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        xs = [np.broadcast_to(np.asarray(x).astype(F32), out_shape) for x in inputs]
        if acc is not None:
            acc = np.asarray(acc, dtype=F32)
            if bias is not None:
                acc = (acc + np.broadcast_to(np.asarray(bias).astype(F32), out_shape)).astype(F32)
        vals = []
        for op, args in spec:
            fn = OPS[op]
            ops = []
            for a in args:
                if isinstance(a, (tuple, list)) and a[0] == "in":
                    ops.append(xs[a[1]])
                elif isinstance(a, (tuple, list)) and a[0] == "node":
                    ops.append(vals[a[1]])
                elif isinstance(a, (tuple, list)) and a[0] == "acc":
                    ops.append(acc)
                elif isinstance(a, str):
                    continue  # cast target dtype
                else:
                    ops.append(F32(a))
            vals.append(np.asarray(fn(*ops), dtype=F32))
        return round_to(np.broadcast_to(vals[-1], out_shape), out_dtype)


def matrix_add(a, b, out_dtype: str = "float32"):
    """hand_written/matrix_add_kernel.py:6-20: flat elementwise a + b."""
    return round_to(np.asarray(a, dtype=F32) + np.asarray(b, dtype=F32), out_dtype)
