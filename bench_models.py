"""Model definitions for the benchmark configurations (random init, no
checkpoints, no timm): ViT-B/16, a Llama-style decoder and the fused-GEMM
sweep block.  Used by bench.py and tests/test_gpu_models.py.

The reference benches the same families through timm's vit_base_patch16_224
(bench/bench_vit.py:9) and transformers' LlamaForCausalLM
(bench/bench_llama.py:7-21); these are self-contained equivalents of the
configurations the benchmark quotes.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class GemmEpilogueBlock(nn.Module):
    """Y = act(X W^T + b) + R -- one point of the fused GEMM sweep."""

    def __init__(self, k: int, n: int, act: str):
        super().__init__()
        self.lin = nn.Linear(k, n)
        self.act = act

    def forward(self, x, r):
        y = self.lin(x)
        if self.act == "gelu":
            y = F.gelu(y)
        elif self.act == "silu":
            y = F.silu(y)
        return y + r


def init_sweep_block(block: GemmEpilogueBlock, gen: torch.Generator) -> None:
    with torch.no_grad():
        block.lin.weight.normal_(0.0, 0.02, generator=gen)
        block.lin.bias.normal_(0.0, 0.01, generator=gen)


# --------------------------------------------------------------------- MLP
class MLP(nn.Module):
    """The benchmark's MLP configuration: x[64,1024] fp32 ->
    Linear(1024->4096) -> GELU(tanh) -> Linear(4096->1024) -> + x, with
    nn.Linear's default init.  The reference's bench/mlp.py:6-19 block has
    the same GEMM shapes with an erf GELU and an x + tanh(y) * scale tail."""

    def __init__(self, dim=1024, hidden=4096):
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden)
        self.fc2 = nn.Linear(hidden, dim)

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(x), approximate="tanh")) + x


def mlp_flops(rows=64, dim=1024, hidden=4096) -> float:
    return 2.0 * rows * dim * hidden * 2


# --------------------------------------------------------------------- ViT
class ViTBlock(nn.Module):
    def __init__(self, dim: int, heads: int, mlp: int):
        super().__init__()
        self.heads = heads
        self.norm1 = nn.LayerNorm(dim, eps=1e-6)
        self.qkv = nn.Linear(dim, 3 * dim)
        self.proj = nn.Linear(dim, dim)
        self.norm2 = nn.LayerNorm(dim, eps=1e-6)
        self.fc1 = nn.Linear(dim, mlp)
        self.fc2 = nn.Linear(mlp, dim)

    def forward(self, x):
        B, T, C = x.shape
        h = self.heads
        qkv = self.qkv(self.norm1(x)).view(B, T, 3, h, C // h).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2])
        x = x + self.proj(a.transpose(1, 2).reshape(B, T, C))
        return x + self.fc2(F.gelu(self.fc1(self.norm2(x))))


class ViT(nn.Module):
    """ViT-B/16: 224x224 images, patch 16 (196 tokens + CLS), pre-LN,
    learned positional embedding, 1000-class head."""

    def __init__(self, img=224, patch=16, dim=768, depth=12, heads=12, mlp=3072, classes=1000):
        super().__init__()
        self.patch = nn.Conv2d(3, dim, patch, patch)
        n = (img // patch) ** 2
        self.cls = nn.Parameter(torch.zeros(1, 1, dim))
        self.pos = nn.Parameter(0.02 * torch.randn(1, n + 1, dim))
        self.blocks = nn.ModuleList(ViTBlock(dim, heads, mlp) for _ in range(depth))
        self.norm = nn.LayerNorm(dim, eps=1e-6)
        self.head = nn.Linear(dim, classes)

    def forward(self, img):
        x = self.patch(img).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls.expand(x.shape[0], -1, -1), x], dim=1) + self.pos
        for blk in self.blocks:
            x = blk(x)
        return self.head(self.norm(x)[:, 0])


def vit_flops_per_image(img=224, patch=16, dim=768, depth=12, mlp=3072, classes=1000) -> float:
    t = (img // patch) ** 2 + 1
    lin = 2 * t * (dim * 3 * dim + dim * dim + 2 * dim * mlp)
    attn = 2 * 2 * t * t * dim
    embed = 2 * (t - 1) * 3 * patch * patch * dim
    return depth * (lin + attn) + embed + 2 * dim * classes


# ------------------------------------------------------------------- Llama
class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, h):
        dt = h.dtype
        x = h.to(torch.float32)
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * x.to(dt)


def _rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


class LlamaLayer(nn.Module):
    def __init__(self, dim, heads, kv_heads, ffn, eps):
        super().__init__()
        self.h, self.kv, self.hd = heads, kv_heads, dim // heads
        self.in_norm = RMSNorm(dim, eps)
        self.q = nn.Linear(dim, heads * self.hd, bias=False)
        self.k = nn.Linear(dim, kv_heads * self.hd, bias=False)
        self.v = nn.Linear(dim, kv_heads * self.hd, bias=False)
        self.o = nn.Linear(heads * self.hd, dim, bias=False)
        self.post_norm = RMSNorm(dim, eps)
        self.gate = nn.Linear(dim, ffn, bias=False)
        self.up = nn.Linear(dim, ffn, bias=False)
        self.down = nn.Linear(ffn, dim, bias=False)

    def forward(self, x, cos, sin):
        B, S, D = x.shape
        h = self.in_norm(x)
        q = self.q(h).view(B, S, self.h, self.hd).transpose(1, 2)
        k = self.k(h).view(B, S, self.kv, self.hd).transpose(1, 2)
        v = self.v(h).view(B, S, self.kv, self.hd).transpose(1, 2)
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        x = x + self.o(a.transpose(1, 2).reshape(B, S, D))
        h = self.post_norm(x)
        return x + self.down(F.silu(self.gate(h)) * self.up(h))


class Llama(nn.Module):
    """Llama-style decoder: RMSNorm, RoPE, GQA attention, SwiGLU FFN."""

    def __init__(self, vocab=128256, dim=2048, layers=16, heads=32, kv_heads=8, ffn=8192, eps=1e-5,
                 theta=500000.0, max_seq=2048):
        super().__init__()
        self.embed = nn.Embedding(vocab, dim)
        self.layers = nn.ModuleList(LlamaLayer(dim, heads, kv_heads, ffn, eps) for _ in range(layers))
        self.norm = RMSNorm(dim, eps)
        self.lm_head = nn.Linear(dim, vocab, bias=False)
        self.hd, self.theta, self.max_seq = dim // heads, theta, max_seq
        self.register_buffer("cos", torch.empty(max_seq, self.hd, dtype=torch.float32), persistent=False)
        self.register_buffer("sin", torch.empty(max_seq, self.hd, dtype=torch.float32), persistent=False)
        self.reset_rope()

    def reset_rope(self) -> None:
        """(Re)computes the rotary tables (also after materialising a model
        built on the meta device)."""
        hd, dev = self.hd, self.cos.device
        inv = 1.0 / (self.theta ** (torch.arange(0, hd, 2, dtype=torch.float32, device=dev) / hd))
        f = torch.outer(torch.arange(self.max_seq, dtype=torch.float32, device=dev), inv)
        emb = torch.cat([f, f], dim=-1)
        with torch.no_grad():
            self.cos.copy_(emb.cos())
            self.sin.copy_(emb.sin())

    def forward(self, ids):
        S = ids.shape[1]
        x = self.embed(ids)
        cos, sin = self.cos[:S].to(x.dtype), self.sin[:S].to(x.dtype)
        for layer in self.layers:
            x = layer(x, cos, sin)
        return self.lm_head(self.norm(x))


def init_normal_(model: nn.Module, std: float, gen: torch.Generator) -> None:
    """N(0, std) for every weight matrix/embedding; norms keep 1."""
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() >= 2:
                p.normal_(0.0, std, generator=gen)


def llama_flops_per_token(seq=2048, vocab=128256, dim=2048, layers=16, heads=32, kv_heads=8, ffn=8192) -> float:
    hd = dim // heads
    lin = 2 * (dim * heads * hd + 2 * dim * kv_heads * hd + heads * hd * dim + 3 * dim * ffn)
    attn = 2 * 2 * seq * dim / 2  # causal: half the score/value work
    return layers * (lin + attn) + 2 * dim * vocab


def _check():
    assert math.isclose(vit_flops_per_image() / 1e9, 35.1, rel_tol=0.05)
