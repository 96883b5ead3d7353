"""Small seeded models whose compiled graphs exercise every fusion rule.

Shared by tests/golden/make_golden.py (which records what the reference
backend does with them) and the tests (which check this backend against those
records).  Shapes are small so the reference's kernels finish in seconds
under Triton's CPU interpreter.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class MLPBlock(nn.Module):
    """The reference benchmark's MLP block structure (bench/mlp.py:6-18):
    erf-GELU after fc1, then x + tanh(fc2) * scale."""

    def __init__(self, dim=32, hidden=64):
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden)
        self.fc2 = nn.Linear(hidden, dim)
        self.scale = nn.Parameter(torch.full((dim,), 0.5))

    def forward(self, x):
        h = F.gelu(self.fc1(x))
        y = self.fc2(h)
        return x + torch.tanh(y) * self.scale


class TanhGeluMLP(nn.Module):
    """The structure of the reference's CPU MLP benchmark (bench/mlp.py):
    Linear -> tanh-GELU -> Linear -> +x."""

    def __init__(self, dim=32, hidden=64):
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden)
        self.fc2 = nn.Linear(hidden, dim)

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(x), approximate="tanh")) + x


class SiluMLP(nn.Module):
    def __init__(self, dim=32, hidden=64):
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden)
        self.fc2 = nn.Linear(hidden, dim, bias=False)

    def forward(self, x):
        return self.fc2(F.silu(self.fc1(x)))


class Zoo(nn.Module):
    """Every POINTWISE_OPS entry, broadcasting ([N], [M,1]) and a transposed input."""

    def forward(self, x, y, col, row):
        a = torch.sigmoid(x) * y - torch.abs(x) / (1.0 + torch.exp(-y))
        b = torch.maximum(a, row) + torch.minimum(x.t().t(), col) - torch.neg(y)
        c = torch.sqrt(torch.abs(b) + 1.0) * torch.rsqrt(torch.abs(a) + 2.0) + torch.log(torch.abs(x) + 1.5)
        d = torch.relu(c - 1.0) + torch.tanh(b) * 0.25 + torch.erf(a * 0.5)
        e = (d + x.t().contiguous().t()) * 2.0 - 3.0 / (torch.abs(y) + 1.0)
        return e


class CastChain(nn.Module):
    """fp16 chains with _to_copy: an fp32 upcast inside a group, a closing
    downcast, and a downcast with a fusible user (which must split the group)."""

    def forward(self, x, y):
        t = x.to(torch.float32) * 2.0 + 1.0
        u = torch.sigmoid(t).to(torch.float16)
        v = (u + y) * 0.5
        return v.to(torch.float32).exp() - 1.0


def make_case(name: str):
    """Returns (module, inputs) with seed-0 weights and inputs."""
    g = torch.Generator().manual_seed(0)
    torch.manual_seed(0)
    if name == "mlp_block_fp32":
        return MLPBlock(), (torch.randn(16, 32, generator=g),)
    if name == "mlp_tanh_fp32":
        return TanhGeluMLP(), (torch.randn(16, 32, generator=g),)
    if name == "mlp_silu_fp32":
        return SiluMLP(), (torch.randn(16, 32, generator=g),)
    if name == "mlp_block_fp16":
        return MLPBlock().half(), (torch.randn(16, 32, generator=g).half(),)
    if name == "mlp_tanh_fp16":
        return TanhGeluMLP().half(), (torch.randn(16, 32, generator=g).half(),)
    if name == "zoo_fp32":
        x = torch.randn(24, 40, generator=g)
        y = torch.randn(24, 40, generator=g)
        col = torch.randn(24, 1, generator=g)
        row = torch.randn(40, generator=g)
        return Zoo(), (x, y, col, row)
    if name == "casts_fp16":
        return CastChain(), (torch.randn(24, 40, generator=g).half(), torch.randn(24, 40, generator=g).half())
    raise KeyError(name)


CASES = ["mlp_block_fp32", "mlp_tanh_fp32", "mlp_silu_fp32", "mlp_block_fp16", "mlp_tanh_fp16", "zoo_fp32",
         "casts_fp16"]
