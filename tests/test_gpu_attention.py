"""GPU parity of the tcgen05 attention kernel (b200k_attention), called
through the C ABI and through torch.ops.b200.attention, against an fp32
reference of softmax(scale q k^T [causal]) v.

Tolerance: the kernel rounds the probabilities to the 16-bit input type
before the second product, as flash attention does; outputs (weighted means
of v ~ N(0, 1)) are compared at 1.5e-2 absolute + 1e-2 relative to fp32, and
to PyTorch's own 16-bit SDPA at the same bound.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from compiler import runtime
from compiler.runtime import cabi

pytestmark = pytest.mark.gpu
DEV = "cuda"
runtime.load()


def _ref(q, k, v, causal, scale=None):
    G = q.shape[1] // k.shape[1]
    kf = k.float().repeat_interleave(G, dim=1)
    vf = v.float().repeat_interleave(G, dim=1)
    s = (q.float() @ kf.transpose(-1, -2)) * (scale if scale else 1.0 / math.sqrt(q.shape[-1]))
    if causal:
        L, S = q.shape[2], k.shape[2]
        mask = torch.ones(L, S, dtype=torch.bool, device=q.device).tril()
        s = s.masked_fill(~mask, float("-inf"))
    return torch.softmax(s, -1) @ vf


def _make(B, H, Hkv, L, S, dtype, layout, g):
    def one(h, n):
        if layout == "bshd":  # [B, S, H, D] in memory, viewed as [B, H, S, D]
            return torch.randn(B, n, h, 64, device=DEV, generator=g).to(dtype).transpose(1, 2)
        return torch.randn(B, h, n, 64, device=DEV, generator=g).to(dtype)

    return one(H, L), one(Hkv, S), one(Hkv, S)


CASES = [
    (2, 4, 4, 197, 197, False),    # ViT-B/16 length, ragged blocks
    (1, 8, 2, 256, 256, True),     # grouped-query, causal
    (2, 4, 1, 1000, 1000, True),   # one kv head, ragged causal
    (1, 2, 2, 64, 64, False),      # a single partial tile
    (1, 2, 2, 64, 300, False),     # more keys than queries
    (1, 2, 1, 100, 300, True),     # causal with L != S (top-left mask, as torch SDPA)
    (1, 4, 2, 2048, 2048, True),   # the Llama prefill's length
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}x{c[1]}/{c[2]}x{c[3]}x{c[4]}{'-causal' if c[5] else ''}"
                                             for c in CASES])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("layout", ["bhsd", "bshd"])
def test_attention_matches_fp32(case, dtype, layout):
    B, H, Hkv, L, S, causal = case
    g = torch.Generator(device=DEV).manual_seed(B * 1000 + L + S)
    q, k, v = _make(B, H, Hkv, L, S, dtype, layout, g)
    out = torch.full((B, H, L, 64), float("nan"), device=DEV, dtype=dtype)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    cabi.attention(q, k, v, out, causal=causal, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    want = _ref(q, k, v, causal)
    torch.testing.assert_close(out.float(), want, atol=1.5e-2, rtol=1e-2)
    theirs = F.scaled_dot_product_attention(q, k, v, is_causal=causal, enable_gqa=H != Hkv)
    torch.testing.assert_close(out.float(), theirs.float(), atol=1.5e-2, rtol=1e-2)


def test_attention_scale_and_torch_op_layout():
    g = torch.Generator(device=DEV).manual_seed(3)
    q, k, v = _make(2, 4, 2, 333, 333, torch.bfloat16, "bshd", g)
    # output in [B, S, H, D] memory order, as ATen's flash kernels produce it
    stride = list(torch.empty(2, 333, 4, 64).transpose(1, 2).stride())
    out = torch.ops.b200.attention(q, k, v, True, 0.2, stride)
    assert list(out.stride()) == stride
    torch.testing.assert_close(out.float(), _ref(q, k, v, True, 0.2), atol=1.5e-2, rtol=1e-2)
    runtime.check_status()


def test_attention_stalled_wait_times_out_and_context_survives():
    """The test hook withholds the first score block's ready signal: the
    softmax's wait runs out after 50 ms, the kernel reports B200K_ERR_TIMEOUT,
    drains and frees its tensor memory, and the next call is correct."""
    g = torch.Generator(device=DEV).manual_seed(5)
    q, k, v = _make(1, 4, 4, 512, 512, torch.bfloat16, "bhsd", g)
    out = torch.empty_like(q)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    cabi.attention(q, k, v, out, causal=True, status=status, timeout_ns=50_000_000,
                   test_flags=cabi.ATTN_TEST_WITHHOLD_SCORES)
    torch.cuda.synchronize()
    assert status.item() == 6
    status.zero_()
    cabi.attention(q, k, v, out, causal=True, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    torch.testing.assert_close(out.float(), _ref(q, k, v, True), atol=1.5e-2, rtol=1e-2)
