"""Oracle for the row-reduction kernels -- test infrastructure only.

No reference counterpart: the reference leaves pow/mean/native_layer_norm/
_softmax to ATen.  These restate the eager semantics of the decomposed ATen
graphs the row-reduction pass replaces, including the rounding points of the
casts between ops (the kernel's ROUND_* flags).
"""
from __future__ import annotations

import numpy as np

from .bf16 import round_to

F32 = np.float32
ROUND_NORMED, ROUND_AFFINE, ROUND_SILU = 1, 2, 4


def _rows(x):
    x = np.asarray(x, dtype=F32)
    return x.reshape(-1, x.shape[-1]), x.shape


def rms_norm(x, weight, eps, flags, x_dtype: str, out_dtype: str):
    """n = x * rsqrt(mean(x^2) + eps) [round to x dtype] ; y = weight * n."""
    r, shape = _rows(x)
    ms = (r * r).mean(axis=-1, keepdims=True, dtype=np.float64).astype(F32)
    n = (r * (F32(1.0) / np.sqrt(ms + F32(eps)))).astype(F32)
    if flags & ROUND_NORMED:
        n = round_to(n, x_dtype)
    y = n if weight is None else (np.asarray(weight, dtype=F32) * n).astype(F32)
    return round_to(y, out_dtype).reshape(shape)


def rms_norm_swiglu(x, weight, eps, flags, x_dtype: str, out_dtype: str):
    """y = rms_norm(x) (rounded to out dtype with ROUND_AFFINE); g, u = halves;
    out = silu(g) [round] * u."""
    y = rms_norm(x, weight, eps, flags, x_dtype, "float32")
    if flags & ROUND_AFFINE:
        y = round_to(y, out_dtype)
    half = y.shape[-1] // 2
    g, u = y[..., :half], y[..., half:]
    s = (g * (F32(1.0) / (F32(1.0) + np.exp(-g)))).astype(F32)
    if flags & ROUND_SILU:
        s = round_to(s, out_dtype)
    return round_to(s * u, out_dtype)


def layer_norm(x, weight, bias, eps, out_dtype: str):
    """aten.native_layer_norm over the last dim (biased variance, fp32 stats)."""
    r, shape = _rows(x)
    mean = r.mean(axis=-1, keepdims=True, dtype=np.float64).astype(F32)
    var = ((r - mean) ** 2).mean(axis=-1, keepdims=True, dtype=np.float64).astype(F32)
    rstd = (F32(1.0) / np.sqrt(var + F32(eps))).astype(F32)
    y = (r - mean) * rstd
    if weight is not None:
        y = y * np.asarray(weight, dtype=F32)
    if bias is not None:
        y = y + np.asarray(bias, dtype=F32)
    stat_shape = shape[:-1] + (1,)
    return round_to(y, out_dtype).reshape(shape), mean.reshape(stat_shape), rstd.reshape(stat_shape)


def softmax(x, out_dtype: str):
    r, shape = _rows(x)
    m = r.max(axis=-1, keepdims=True)
    e = np.exp(r - m).astype(F32)
    return round_to(e / e.sum(axis=-1, keepdims=True, dtype=np.float64).astype(F32), out_dtype).reshape(shape)


def log_softmax(x, out_dtype: str):
    r, shape = _rows(x)
    m = r.max(axis=-1, keepdims=True)
    s = np.exp(r - m).sum(axis=-1, keepdims=True, dtype=np.float64).astype(F32)
    return round_to(r - m - np.log(s), out_dtype).reshape(shape)
