"""Seeded inputs of the benchmark configurations, shared by the full-size
parity tests and the reference-backend runner (tests/ref_triton_runner.py),
so both processes build bit-identical tensors on the GPU.  Imports neither
this repository's backend nor the reference's."""
from __future__ import annotations

import torch

import bench_models as bm

SWEEP = [(512, 512, 512), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 4096, 14336)]
ACTS = ["none", "gelu", "silu"]


def sample_rows(M: int, n: int = 192) -> torch.Tensor:
    """n rows spread over [0, M), the first and last included (every 128-row
    tile band of the large GEMMs is hit)."""
    return torch.unique(torch.linspace(0, M - 1, min(n, M)).round().long())


def sweep_point(i: int, device: str = "cuda"):
    """Block and inputs of sweep point i (shape-major, act-minor), as the
    benchmark builds them: X, R ~ N(0, 0.02), W ~ N(0, 0.02), b ~ N(0, 0.01)."""
    (M, N, K), act = SWEEP[i // 3], ACTS[i % 3]
    g = torch.Generator(device=device).manual_seed(1000 + i)
    x = (0.02 * torch.randn(M, K, device=device, generator=g)).to(torch.bfloat16)
    r = (0.02 * torch.randn(M, N, device=device, generator=g)).to(torch.bfloat16)
    blk = bm.GemmEpilogueBlock(K, N, act)
    bm.init_sweep_block(blk, torch.Generator().manual_seed(i))
    return blk.to(device, torch.bfloat16).eval(), x, r


class TanhMLP(torch.nn.Module):
    """The benchmark's MLP: Linear(1024 -> 4096) + bias, tanh-GELU,
    Linear(4096 -> 1024) + bias, + x."""

    def __init__(self):
        super().__init__()
        self.fc1 = torch.nn.Linear(1024, 4096)
        self.fc2 = torch.nn.Linear(4096, 1024)

    def forward(self, x):
        return self.fc2(torch.nn.functional.gelu(self.fc1(x), approximate="tanh")) + x


def mlp(device: str = "cuda"):
    """The MLP config with nn.Linear's default init from seed 0 and
    x[64, 1024] ~ N(0, 1), fp32."""
    torch.manual_seed(0)
    m = TanhMLP().to(device).eval()
    g = torch.Generator(device=device).manual_seed(0)
    x = torch.randn(64, 1024, device=device, generator=g)
    return m, x
