"""Oracle for GEMM + epilogue -- test infrastructure only.

Restates the reference's generated GEMM kernel
(compiler/optimization/fusion_epilogue.py:72-151): fp32 accumulation of
A[M,K] @ B[K,N] (:120-128), addmm bias added first (:142-143), the epilogue
group evaluated in fp32 on the accumulator (:134-146), one rounding store to
the output dtype (:147-149).  Also the standalone demos in hand_written/.
"""
from __future__ import annotations

import numpy as np

from .bf16 import round_to
from .pointwise import eval_group


def gemm_epilogue(a, b, spec, extras, out_dtype: str, bias=None):
    """out = round(group(acc [+ bias], extras)), acc = fp32(a) @ fp32(b).

    ``spec`` refers to the accumulator as ('acc',) and to extras as ('in', i).
    An empty spec stores the accumulator (plus bias) directly.
    """
    acc = np.asarray(a, dtype=np.float32) @ np.asarray(b, dtype=np.float32)
    if not spec:
        if bias is not None:
            acc = acc + np.asarray(bias, dtype=np.float32)
        return round_to(acc, out_dtype)
    return eval_group(spec, extras, acc.shape, out_dtype, acc=acc, bias=bias)


def hand_gemm(a, b):
    """hand_written/gemm_kernel.py:6-71: fp32 accumulate, fp16 result."""
    return round_to(np.asarray(a, dtype=np.float32) @ np.asarray(b, dtype=np.float32), "float16")


def hand_gemm_swizzled(a, b):
    """hand_written/gemm_swizzled_kernel.py:5-89: same product, grouped tile
    order (which does not change the values); fp32 accumulator stored into an
    fp16 tensor."""
    return hand_gemm(a, b)
