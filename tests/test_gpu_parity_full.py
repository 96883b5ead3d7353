"""Parity at the benchmark's full configurations.

* every point of the fused GEMM sweep, through torch.compile(custom_backend),
  against an fp32 eager reference of the same block on sampled rows, with an
  element-wise bound;
* the same points and the fp32 MLP against the reference backend's own
  Triton kernels on the same GPU (run from baseline/_ref in a subprocess on
  bit-identical seeded inputs);
* ViT-B/16 at batch 64, 12 layers, and the 16-layer Llama-style prefill at
  2 x 2048 against fp32 eager PyTorch with the same (bf16-rounded) weights.

Tolerances, written here as the task states them: a bf16 GEMM + epilogue is
within 2e-2 relative to an fp32 eager reference.  Element-wise that is
|got - want| <= 2e-2 * (|act(xW^T + b)| + |R|): the error of a sum is bounded
by the magnitudes of its terms, not by the (possibly cancelled) sum.
"""
import os
import subprocess
import sys
import tempfile

import pytest
import torch

import bench_models as bm
import sweep_inputs as si
from compiler import runtime
from compiler.backend import custom_backend

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref", "compiler")


def _fp32_terms(blk, x, r, rows):
    """fp32 eager act(x W^T + b) and R on `rows` (no TF32)."""
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        lin = blk.lin
        y = x[rows].float() @ lin.weight.float().t() + lin.bias.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    if blk.act == "gelu":
        y = torch.nn.functional.gelu(y)
    elif blk.act == "silu":
        y = torch.nn.functional.silu(y)
    return y, r[rows].float()


def _compiled_sweep_outputs():
    outs = {}
    torch._dynamo.config.recompile_limit = max(torch._dynamo.config.recompile_limit, 64)
    with torch.no_grad():
        for i in range(3 * len(si.SWEEP)):
            blk, x, r = si.sweep_point(i)
            torch._dynamo.reset()
            y = torch.compile(blk, backend=custom_backend)(x, r)
            rows = si.sample_rows(x.shape[0]).to(x.device)
            act, res = _fp32_terms(blk, x, r, rows)
            outs[i] = (y[rows].float(), act, res)
            del blk, x, r, y
    runtime.check_status()
    return outs


@pytest.fixture(scope="module")
def sweep_outputs():
    return _compiled_sweep_outputs()


@pytest.mark.parametrize("i", range(12), ids=[f"{s[0]}x{s[1]}x{s[2]}-{a}" for s in si.SWEEP for a in si.ACTS])
def test_sweep_point_vs_fp32_eager(sweep_outputs, i):
    got, act, res = sweep_outputs[i]
    want = act + res
    bound = 2e-2 * (act.abs() + res.abs()) + 1e-6
    bad = (got - want).abs() > bound
    assert not bad.any(), f"{int(bad.sum())} of {bad.numel()} elements outside the bound"
    # and the usual relative norm
    assert ((got - want).norm() / want.norm()).item() < 1e-2


def _run_reference(case: str) -> dict:
    if not os.path.isdir(REF):
        pytest.skip("reference backend not installed in baseline/_ref")
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "ref.pt")
        r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "ref_triton_runner.py"), case, out],
                           capture_output=True, text=True, timeout=1500)
        assert r.returncode == 0, r.stderr[-3000:]
        return torch.load(out)


def test_sweep_matches_reference_triton_backend(sweep_outputs):
    """Each sweep point against the reference backend's Triton kernels on the
    same inputs (both bf16; the bound above, with the reference's output as
    the value compared)."""
    ref = _run_reference("sweep")
    for i in range(12):
        got, act, res = sweep_outputs[i]
        theirs = ref[i].to(got.device).float()
        bound = 2e-2 * (act.abs() + res.abs()) + 1e-6
        bad = (got - theirs).abs() > bound
        assert not bad.any(), f"point {i}: {int(bad.sum())} elements differ beyond the bound"


def test_mlp_fp32_matches_reference_triton_backend_and_eager():
    """The benchmark's fp32 MLP on the GPU: this backend, the reference
    backend and eager fp32 (no TF32) agree to fp32 accumulation-order
    differences."""
    m, x = si.mlp()
    torch._dynamo.reset()
    with torch.no_grad():
        want = m(x)
        got = torch.compile(m, backend=custom_backend)(x)
    ref = _run_reference("mlp")["mlp"].to(got.device)
    scale = want.abs().max().item()
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5 * scale)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4 * scale)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def _fp32_twin(model_bf16, make):
    m32 = make()
    m32.load_state_dict({k: v.float() for k, v in model_bf16.state_dict().items()}, strict=False)
    return m32.to("cuda").float().eval()


def test_vit_b16_full_config_vs_fp32_eager():
    """ViT-B/16, batch 64, 12 layers (the benchmark config)."""
    torch.manual_seed(0)
    model = bm.ViT().to("cuda", torch.bfloat16).eval()
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(64, 3, 224, 224, device="cuda", generator=g).to(torch.bfloat16)
    m32 = _fp32_twin(model, bm.ViT)
    torch._dynamo.reset()
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.no_grad():
            want = m32(x.float())
            eager = model(x)
            f = torch.compile(model, backend=custom_backend)
            got = [f(x) for _ in range(3)]  # op by op, recorded, replayed
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    runtime.check_status()
    e_ours, e_eager = _rel(got[-1], want), _rel(eager, want)
    print(f"ViT-B/16 b64: rel err vs fp32 ours {e_ours:.4f} eager-bf16 {e_eager:.4f}")
    assert e_ours < 2e-2
    assert torch.equal(got[0], got[2])  # the replayed graph computes what the op-by-op run did


def test_llama_full_depth_vs_fp32_eager():
    """The 16-layer Llama-style prefill (dim 2048, GQA 32/8, SwiGLU 8192,
    vocab 128256) at batch 2 x 2048."""
    model = bm.Llama()
    bm.init_normal_(model, 0.02, torch.Generator().manual_seed(0))
    model = model.to("cuda", torch.bfloat16).eval()
    g = torch.Generator(device="cuda").manual_seed(0)
    ids = torch.randint(0, 128256, (2, 2048), device="cuda", generator=g)
    m32 = _fp32_twin(model, bm.Llama)
    torch._dynamo.reset()
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.no_grad():
            want = m32(ids)
            eager = model(ids)
            got = torch.compile(model, backend=custom_backend)(ids)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    runtime.check_status()
    e_ours, e_eager = _rel(got, want), _rel(eager, want)
    print(f"Llama 16L 2x2048: rel err vs fp32 ours {e_ours:.4f} eager-bf16 {e_eager:.4f}")
    # Sixteen bf16 layers drift from fp32 by more than one GEMM's 2e-2 bar:
    # eager PyTorch bf16 itself lands at 2.8e-2 on this config.  The bar for
    # the whole model is therefore "no farther from fp32 than eager bf16"
    # (5 % slack), with 3e-2 as the absolute limit.
    assert e_ours < 3e-2
    assert e_ours <= 1.05 * e_eager
