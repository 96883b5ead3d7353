"""Pins the oracle: it must reproduce every kernel output the reference's own
Triton kernels produced on the recorded inputs (tests/golden/make_golden.py)."""
import numpy as np
import pytest

import oracle

TOL = {"float32": (1e-5, 1e-6), "float16": (2e-3, 1e-3), "float64": (1e-5, 1e-6)}


def _kernel_ids():
    import json
    import os

    with open(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.json")) as f:
        meta = json.load(f)
    return [i for i, k in enumerate(meta["kernels"]) if k["calls"]]


@pytest.mark.parametrize("k", _kernel_ids())
def test_oracle_matches_reference_kernel(golden, k):
    meta, arrays = golden
    ent = meta["kernels"][k]
    ins = [arrays[f"k{k}_in{i}"] for i in range(ent["n_inputs"])]
    shape = tuple(ent["out_shape"])
    if ent["kind"] == "pointwise":
        got = oracle.eval_group(ent["spec"], ins, shape, ent["out_dtype"])
    else:
        bias = ins[0] if ent["bias_first"] else None
        got = oracle.gemm_epilogue(arrays[f"k{k}_a"], arrays[f"k{k}_b"], ent["spec"], ins, ent["out_dtype"], bias=bias)
    ref = arrays[f"k{k}_out"]
    rtol, atol = TOL[ent["out_dtype"]]
    if ent["kind"] == "gemm_epilogue":
        # fp32 accumulation order differs from the interpreter's tl.dot; one
        # fp16 ulp of slack on the rounded output.
        rtol, atol = max(rtol, 1e-3), max(atol, 1e-3)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=atol)


def test_golden_covers_every_pointwise_op(golden):
    meta, _ = golden
    seen = {op for k in meta["kernels"] if k["calls"] for op, _ in k["spec"]}
    for name in oracle.OPS:
        assert name in seen, f"no golden vector exercises {name}"


def test_hand_written_oracles():
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 4)).astype(np.float32)
    b = rng.standard_normal((3, 4)).astype(np.float32)
    np.testing.assert_array_equal(oracle.matrix_add(a, b), a + b)
    a16 = rng.standard_normal((64, 32)).astype(np.float16)
    b16 = rng.standard_normal((32, 48)).astype(np.float16)
    ref = (a16.astype(np.float32) @ b16.astype(np.float32)).astype(np.float16).astype(np.float32)
    np.testing.assert_array_equal(oracle.hand_gemm(a16, b16), ref)
    np.testing.assert_array_equal(oracle.hand_gemm_swizzled(a16, b16), ref)


def test_bf16_rounding_matches_torch():
    import torch

    x = torch.randn(10000, dtype=torch.float32) * 100
    x[:4] = torch.tensor([float("inf"), float("-inf"), 0.0, -0.0])
    ref = x.to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(oracle.round_bf16(x.numpy()), ref)


def test_rowreduce_oracles_match_torch_cpu():
    import torch
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(0)
    x = torch.randn(8, 64, generator=g).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(64, generator=g)).to(torch.bfloat16)
    x32 = x.float()
    n = (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    y = w * n
    got = oracle.rms_norm(x.float().numpy(), w.float().numpy(), 1e-6, 1, "bfloat16", "bfloat16")
    np.testing.assert_allclose(got, y.float().numpy(), rtol=1e-2, atol=1e-2)
    gq, up = y.split(32, -1)
    sw = F.silu(gq.float()).to(torch.bfloat16) * up
    got = oracle.rms_norm_swiglu(x.float().numpy(), w.float().numpy(), 1e-6, 7, "bfloat16", "bfloat16")
    np.testing.assert_allclose(got, sw.float().numpy(), rtol=1e-2, atol=1e-2)
    lw, lb = torch.randn(64, generator=g), torch.randn(64, generator=g)
    xl = torch.randn(5, 3, 64, generator=g)
    out, mean, rstd = torch.ops.aten.native_layer_norm(xl, [64], lw, lb, 1e-5)
    o2, m2, r2 = oracle.layer_norm(xl.numpy(), lw.numpy(), lb.numpy(), 1e-5, "float32")
    np.testing.assert_allclose(o2, out.numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(m2, mean.numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(r2, rstd.numpy(), rtol=1e-5, atol=1e-6)
    xs = torch.randn(7, 100, generator=g) * 2
    np.testing.assert_allclose(oracle.softmax(xs.numpy(), "float32"), torch.softmax(xs, -1).numpy(), rtol=1e-5,
                               atol=1e-7)
    np.testing.assert_allclose(oracle.log_softmax(xs.numpy(), "float32"), torch.log_softmax(xs, -1).numpy(),
                               rtol=1e-5, atol=1e-5)


def test_rope_oracle_matches_torch_cpu_bit_for_bit():
    import torch

    g = torch.Generator().manual_seed(0)
    for dt, name in ((torch.bfloat16, "bfloat16"), (torch.float16, "float16")):
        x = torch.randn(2, 4, 16, 64, generator=g).to(dt)
        c = torch.randn(16, 64, generator=g).to(dt)
        s = torch.randn(16, 64, generator=g).to(dt)
        x1, x2 = x.chunk(2, dim=-1)
        ref = x * c + torch.cat((-x2, x1), dim=-1) * s
        got = oracle.rope(x.float().numpy(), c.float().numpy(), s.float().numpy(), name)
        np.testing.assert_array_equal(got, ref.float().numpy())
