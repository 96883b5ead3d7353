"""Rotary position embedding, rotate-half form -- TEST INFRASTRUCTURE ONLY.

No reference counterpart (the reference backend leaves rotate_half's aten.cat
in ATen); this restates eager PyTorch's decomposed graph for a 16-bit x:
    r = cat(-x[..., D/2:], x[..., :D/2])
    out = round(round(x * cos) + round(r * sin))
(each ATen op computes in fp32 and rounds its result to the tensor dtype).
Pinned against torch on CPU in tests/test_oracle_golden.py.
"""
from __future__ import annotations

import numpy as np

from .bf16 import round_to


def rope(x, cos, sin, dtype: str) -> np.ndarray:
    """x, cos, sin: fp32 arrays holding dtype values (cos / sin broadcast to x)."""
    x = np.asarray(x, dtype=np.float32)
    half = x.shape[-1] // 2
    r = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    a = round_to(x * np.asarray(cos, np.float32), dtype)
    b = round_to(r * np.asarray(sin, np.float32), dtype)
    return round_to(a + b, dtype)
