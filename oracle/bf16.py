"""Rounding helpers for the oracle (numpy has no bfloat16).  Test infrastructure only."""
from __future__ import annotations

import numpy as np


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bfloat16 (ties to even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = x[nan]
    return out


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to `dtype` ('float32', 'float16', 'bfloat16', 'float64')
    and return them as fp32 (fp64 stays fp64)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bfloat16":
        return round_bf16(x)
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "float64":
        return x.astype(np.float64)
    return x
