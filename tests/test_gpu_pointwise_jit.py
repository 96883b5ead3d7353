"""Generated pointwise kernels on the GPU (csrc/pointwise_jit.cu).

b200k_pointwise compiles a straight-line kernel per program for launches that
merge to rank <= 2 over bf16/f16/f32 operands; these tests check that such
launches really take that path (the process's counters move, nothing fails
to compile), that its results agree with the oracle and with the interpreter
kernels (B200K_POINTWISE_JIT=0) on the same inputs, and that unit counts that
are not multiples of a thread block's units are covered exactly.
"""
import os

import numpy as np
import pytest
import torch

import oracle
import spec_graph
from compiler import runtime
from compiler.optimization.program import compile_group
from compiler.runtime import cabi

pytestmark = pytest.mark.gpu
DEV = "cuda"

SPECS = {
    "add_half": ([["add.Tensor", [["in", 0], ["in", 1]]], ["mul.Tensor", [["node", 0], 0.5]]], 2),
    "silu_residual_scale": ([["sigmoid.default", [["in", 0]]], ["mul.Tensor", [["in", 0], ["node", 0]]],
                             ["add.Tensor", [["node", 1], ["in", 1]]], ["mul.Tensor", [["node", 2], ["in", 2]]]], 3),
    "zoo": ([["sigmoid.default", [["in", 0]]], ["mul.Tensor", [["node", 0], ["in", 1]]],
             ["abs.default", [["in", 0]]], ["exp.default", [["in", 1]]], ["add.Tensor", [["node", 3], 1.0]],
             ["div.Tensor", [["node", 2], ["node", 4]]], ["sub.Tensor", [["node", 1], ["node", 5]]],
             ["maximum.default", [["node", 6], ["in", 2]]], ["minimum.default", [["node", 7], ["in", 3]]],
             ["tanh.default", [["node", 8]]], ["erf.default", [["node", 9]]], ["neg.default", [["node", 10]]],
             ["relu.default", [["node", 11]]], ["add.Tensor", [["node", 12], 1.5]], ["sqrt.default", [["node", 13]]],
             ["rsqrt.default", [["node", 14]]], ["log.default", [["node", 15]]], ["sub.Tensor", [["node", 16], 2.0]]],
            4),
}


@pytest.fixture(scope="module", autouse=True)
def _lib():
    runtime.load()
    cabi.library()


def _run(ins, spec, n_in, out_dtype, jit: bool):
    nodes, ops = spec_graph.build(spec, n_in)
    prog = compile_group(nodes, ops)
    shape = torch.broadcast_shapes(*[t.shape for t in ins])
    out = torch.empty(shape, device=DEV, dtype=out_dtype)
    old = os.environ.get("B200K_POINTWISE_JIT")
    os.environ["B200K_POINTWISE_JIT"] = "1" if jit else "0"
    try:
        cabi.pointwise(ins, prog.code, prog.imm, out)
        torch.cuda.synchronize()
    finally:
        if old is None:
            del os.environ["B200K_POINTWISE_JIT"]
        else:
            os.environ["B200K_POINTWISE_JIT"] = old
    return out


def _inputs(name, shape, dtypes, kinds, g):
    """kinds[i]: 'full' ([*shape]), 'row' ([shape[-1]], innermost stride 1 on a
    stride-0 outer dim) or 'col' ([shape[0], 1], innermost stride 0)."""
    ins = []
    for dt, kind in zip(dtypes, kinds):
        s = shape if kind == "full" else (shape[-1:] if kind == "row" else (shape[0], 1))
        t = torch.randn(s, device=DEV, generator=g)
        if name == "zoo":
            t = t * 2.0
        ins.append(t.to(dt))
    return ins


CASES = [
    ("add_half", (4096, 1024), [torch.bfloat16] * 2, ["full", "full"], torch.bfloat16),
    ("add_half", (4096, 1024), [torch.float16, torch.float32], ["full", "row"], torch.float32),
    ("add_half", (33, 8 * 127), [torch.float32] * 2, ["full", "col"], torch.float16),
    ("silu_residual_scale", (2048, 768), [torch.bfloat16] * 3, ["full", "full", "row"], torch.bfloat16),
    ("silu_residual_scale", (197, 3072), [torch.bfloat16, torch.float32, torch.bfloat16], ["full", "full", "col"],
     torch.bfloat16),
    ("zoo", (1000, 40), [torch.float32, torch.bfloat16, torch.float16, torch.float32], ["full", "full", "row", "col"],
     torch.float32),
    ("zoo", (64, 8 * 129), [torch.float32] * 4, ["full"] * 4, torch.float32),
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_generated_kernel_matches_oracle_and_interpreter(case):
    name, shape, dtypes, kinds, out_dtype = CASES[case]
    spec, n_in = SPECS[name]
    g = torch.Generator(device=DEV).manual_seed(case)
    ins = _inputs(name, shape, dtypes, kinds, g)
    before = cabi.pointwise_jit_stats()
    got = _run(ins, spec, n_in, out_dtype, jit=True)
    after = cabi.pointwise_jit_stats()
    assert after["failed"] == before["failed"], "a generated kernel failed to compile or load"
    assert after["launches"] == before["launches"] + 1, "the launch did not take the generated kernel"
    ref = _run(ins, spec, n_in, out_dtype, jit=False)
    assert cabi.pointwise_jit_stats()["launches"] == after["launches"]
    od = str(out_dtype).split(".")[-1]
    want = oracle.eval_group(spec, [t.float().cpu().numpy() for t in ins], tuple(shape), od)
    # fp32 within 1e-5 relative; 16-bit outputs within their rounding.
    rtol, atol = (1e-5, 1e-6) if out_dtype == torch.float32 else (1e-2, 1e-2)
    np.testing.assert_allclose(got.float().cpu().numpy(), want.astype(np.float32), rtol=rtol, atol=atol)
    # The interpreter computes the same ops: equal up to one rounding of the
    # output (its tanh may fuse 2*s-1 into one FMA).
    g32, r32 = got.float(), ref.float()
    if out_dtype == torch.float32:
        torch.testing.assert_close(g32, r32, rtol=1e-6, atol=1e-6)
    else:
        ulp = 2.0 ** -7 if out_dtype == torch.bfloat16 else 2.0 ** -10
        assert ((g32 - r32).abs() <= ulp * r32.abs().clamp_min(1e-3)).all()


@pytest.mark.parametrize("units", [1, 255, 256 * 4 - 1, 256 * 4 + 1, 148 * 2 * 256 * 4 + 37])
def test_generated_kernel_covers_every_unit(units):
    """1-D launches whose unit count is not a multiple of one loop step: every
    element is written once (the output starts as NaN) and equals x + y."""
    n = units * 8
    g = torch.Generator(device=DEV).manual_seed(units)
    x = torch.randn(n, device=DEV, generator=g).to(torch.bfloat16)
    y = torch.randn(n, device=DEV, generator=g).to(torch.bfloat16)
    spec = [["add.Tensor", [["in", 0], ["in", 1]]]]
    nodes, ops = spec_graph.build(spec, 2)
    prog = compile_group(nodes, ops)
    out = torch.full((n + 8,), float("nan"), device=DEV, dtype=torch.bfloat16)
    before = cabi.pointwise_jit_stats()["launches"]
    cabi.pointwise([x, y], prog.code, prog.imm, out[:n])
    torch.cuda.synchronize()
    assert cabi.pointwise_jit_stats()["launches"] == before + 1
    assert torch.equal(out[:n], (x.float() + y.float()).to(torch.bfloat16))
    assert torch.isnan(out[n:].float()).all()  # nothing past the end


def test_out_of_scope_launches_take_the_interpreter():
    """f64 output and 5 inputs are outside the generated kernels' scope."""
    g = torch.Generator(device=DEV).manual_seed(7)
    xs = [torch.randn(64, 64, device=DEV, generator=g) for _ in range(5)]
    spec = [["add.Tensor", [["in", 0], ["in", 1]]], ["add.Tensor", [["node", 0], ["in", 2]]],
            ["add.Tensor", [["node", 1], ["in", 3]]], ["add.Tensor", [["node", 2], ["in", 4]]]]
    before = cabi.pointwise_jit_stats()["launches"]
    got = _run(xs, spec, 5, torch.float32, jit=True)
    got64 = _run(xs[:2], spec[:1], 2, torch.float64, jit=True)
    assert cabi.pointwise_jit_stats()["launches"] == before
    torch.testing.assert_close(got, xs[0] + xs[1] + xs[2] + xs[3] + xs[4], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(got64, (xs[0] + xs[1]).double(), rtol=1e-7, atol=1e-7)
