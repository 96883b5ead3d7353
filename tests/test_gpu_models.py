"""End-to-end GPU parity: models compiled with custom_backend (the drop-in
API) against the reference backend's recorded outputs and eager PyTorch."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import bench_models as bm
from cases import CASES, make_case
from compiler import runtime
from compiler.backend import backend, custom_backend
from helpers import b200_targets, capturing_backend

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("extensions", [False, True])
def test_golden_models_match_reference_backend(golden, case, extensions):
    """Reference grouping (extensions off: the same kernels as the reference)
    and the extended grouping both reproduce the reference backend's output."""
    from compiler.optimization import config

    meta, arrays = golden
    model, inputs = make_case(case)
    model = model.to(DEV)
    inputs = [t.to(DEV) for t in inputs]
    old = config.EXTENSIONS
    config.EXTENSIONS = extensions
    try:
        torch._dynamo.reset()
        be, graphs = capturing_backend()
        with torch.no_grad():
            out = torch.compile(model, backend=be)(*inputs)
    finally:
        config.EXTENSIONS = old
    targets = b200_targets(graphs)
    n_ref = len(meta["models"][case]["groups"])
    if not extensions:
        assert len(targets) == n_ref
    ref = arrays[f"{case}_ref_out"]
    tol = (1e-5, 1e-5) if out.dtype == torch.float32 else (1e-2, 1e-2)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=tol[0], atol=tol[1])


def test_backend_alias_and_boxed_compiler():
    assert backend is custom_backend
    from compiler.backend import compiler
    assert callable(compiler)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.fixture
def attention_pass():
    """The attention pass is opt-in; these tests run it."""
    from compiler.optimization import config

    old = config.ENABLE_ATTENTION
    config.ENABLE_ATTENTION = True
    yield
    config.ENABLE_ATTENTION = old


def test_vit_block_stack_bf16(attention_pass):
    torch.manual_seed(0)
    model = bm.ViT(depth=2).to(DEV, torch.bfloat16).eval()
    x = torch.randn(2, 3, 224, 224, device=DEV, dtype=torch.bfloat16)
    torch._dynamo.reset()
    be, graphs = capturing_backend()
    with torch.no_grad():
        want = model(x)
        got = torch.compile(model, backend=be)(x)
    t = [str(s) for s in b200_targets(graphs)]
    # proj+res, fc1+gelu, fc2+res per block; qkv (bias only, no pointwise tail) stays cuBLAS
    assert t.count("b200.gemm_epilogue.default") == 3 * 2
    assert "b200.layer_norm.default" in t
    assert t.count("b200.attention.default") == 2  # one per block (the tcgen05 attention kernel)
    runtime.check_status()
    ops = [n.target for g in graphs for n in g.graph.nodes if n.op == "call_function"]
    assert torch.ops.aten.convolution.default not in ops  # patch embedding lowered to a GEMM
    assert _rel(got, want) < 2e-2


def test_llama_small_bf16(attention_pass):
    torch.manual_seed(0)
    model = bm.Llama(vocab=1024, dim=256, layers=2, heads=4, kv_heads=2, ffn=512, max_seq=128)
    bm.init_normal_(model, 0.02, torch.Generator().manual_seed(0))
    model = model.to(DEV, torch.bfloat16).eval()
    ids = torch.randint(0, 1024, (2, 128), device=DEV)
    torch._dynamo.reset()
    be, graphs = capturing_backend()
    with torch.no_grad():
        want = model(ids)
        got = torch.compile(model, backend=be)(ids)
    t = [str(s) for s in b200_targets(graphs)]
    assert "b200.rms_norm.default" in t
    assert t.count("b200.gemm_rope.default") == 2 * 2  # q and k projections with their rotations, per layer
    assert "b200.rope.default" not in t
    assert t.count("b200.attention.default") == 2  # causal grouped-query attention per layer
    # per layer: o + residual, gate (silu * up), down + residual, all on the compiled path
    epi = [n for g in graphs for n in g.graph.nodes if n.op == "call_function"
           and n.target == torch.ops.b200.gemm_epilogue.default]
    assert len(epi) == 3 * 2 and all(list(n.args[7]) for n in epi)
    runtime.check_status()
    assert _rel(got, want) < 2e-2


def test_training_step_grads_match_eager():
    """Forward and backward graphs both go through the passes (bw_compiler)."""
    torch.manual_seed(0)
    model, (x,) = make_case("mlp_block_fp32")
    model = model.to(DEV, torch.bfloat16)
    ref = make_case("mlp_block_fp32")[0].to(DEV, torch.bfloat16)
    ref.load_state_dict(model.state_dict())
    x = x.to(DEV, torch.bfloat16)
    torch._dynamo.reset()
    out = torch.compile(model, backend=custom_backend)(x)
    out.float().sum().backward()
    ref(x).float().sum().backward()
    assert _rel(out, ref(x)) < 2e-2
    assert _rel(model.fc1.weight.grad, ref.fc1.weight.grad) < 3e-2
    assert _rel(model.fc2.bias.grad, ref.fc2.bias.grad) < 3e-2


def _training_grads(model, inputs, n_graphs=2):
    """One forward + backward of `model` compiled with the backend (forward
    and backward graphs through the passes) and of an fp32 copy run eagerly;
    returns (graphs, [(name, grad, fp32 grad)], (input grad, fp32 input grad))."""
    import copy

    ref = copy.deepcopy(model).float()
    x = inputs[0].detach().clone().requires_grad_(True)
    xr = inputs[0].detach().float().clone().requires_grad_(True)
    torch._dynamo.reset()
    be, graphs = capturing_backend()
    out = torch.compile(model, backend=be)(x, *inputs[1:])
    want = ref(xr, *[t.float() for t in inputs[1:]])
    wgt = torch.randn(out.shape, device=DEV, generator=torch.Generator(device=DEV).manual_seed(7))
    (out.float() * wgt).sum().backward()
    (want * wgt).sum().backward()
    runtime.check_status()
    assert len(graphs) == n_graphs  # the backward graph went through the compiler too
    assert _rel(out, want) < 2e-2
    pairs = [(n, p.grad, dict(ref.named_parameters())[n].grad) for n, p in model.named_parameters()]
    return graphs, pairs, (x.grad, xr.grad)


def test_vit_block_training_step_matches_fp32_eager():
    """A ViT-B/16-style block (bf16, training): every parameter and input
    gradient against the same block in fp32, eager; the backward graph's
    gradient accumulations run as fused kernels."""
    torch.manual_seed(0)
    model = bm.ViTBlock(256, 4, 1024).to(DEV, torch.bfloat16)
    x = torch.randn(4, 65, 256, device=DEV, dtype=torch.bfloat16)
    graphs, pairs, (gx, gx_ref) = _training_grads(model, (x,))
    assert len(pairs) == 12
    for name, got, want in pairs:
        assert _rel(got, want) < 3e-2, name
    assert _rel(gx, gx_ref) < 3e-2
    bw = [str(t) for t in b200_targets(graphs[1:])]
    assert "b200.pointwise.default" in bw


def test_llama_layer_training_step_matches_fp32_eager():
    """A Llama-style decoder layer (bf16, training, GQA, RoPE): every
    parameter and input gradient against fp32 eager; the backward graph's
    input-gradient GEMMs that feed gradient sums run with that sum as their
    epilogue."""
    torch.manual_seed(0)
    model = bm.LlamaLayer(256, 4, 2, 512, 1e-5)
    bm.init_normal_(model, 0.02, torch.Generator().manual_seed(0))
    model = model.to(DEV, torch.bfloat16)
    tables = bm.Llama(vocab=16, dim=256, layers=0, heads=4, kv_heads=2, ffn=512, max_seq=128)
    cos, sin = (t.to(DEV, torch.bfloat16) for t in (tables.cos, tables.sin))
    x = torch.randn(2, 128, 256, device=DEV, dtype=torch.bfloat16)
    graphs, pairs, (gx, gx_ref) = _training_grads(model, (x, cos, sin))
    assert len(pairs) == 9
    for name, got, want in pairs:
        assert _rel(got, want) < 3e-2, name
    assert _rel(gx, gx_ref) < 3e-2
    bw = [str(t) for t in b200_targets(graphs[1:])]
    assert bw.count("b200.gemm_epilogue.default") >= 2


def test_hand_written_api():
    from hand_written.gemm_kernel import gemm
    from hand_written.gemm_swizzled_kernel import gemm as gemm_sw
    from hand_written.matrix_add_kernel import matrix_add

    for n in [128, 512, 2048]:
        a = torch.randn(n, n, device=DEV, dtype=torch.float16)
        b = torch.randn(n, n, device=DEV, dtype=torch.float16)
        ref = (a.float() @ b.float())
        for fn in (gemm, gemm_sw):
            c = fn(a, b)
            assert c.dtype == torch.float16 and c.shape == (n, n)
            torch.testing.assert_close(c.float(), ref, rtol=1e-2, atol=1e-1 * (n / 128) ** 0.5)
    torch.manual_seed(0)
    a = torch.randn(3, 4, device=DEV)
    b = torch.randn(3, 4, device=DEV)
    torch.testing.assert_close(matrix_add(a, b), a + b)
    with pytest.raises(ValueError):
        matrix_add(a.cpu(), b.cpu())
    with pytest.raises(ValueError):
        matrix_add(a, b[:2])
    with pytest.raises(ValueError):
        matrix_add(a, b.half())
    with pytest.raises(ValueError):
        matrix_add(a.int(), b.int())


def test_gemm_timeout_surfaces_through_compiled_graph():
    """A fused GEMM whose device-side wait runs out (the test hook withholds
    its first tile's accumulator-ready signal for one launch) is reported by
    the compiled graph's next call as a RuntimeError; the error is reported
    once and later calls compute the right result again."""
    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.fc = torch.nn.Linear(512, 512)

        def forward(self, x):
            return F.gelu(self.fc(x)) + x

    torch.manual_seed(0)
    m = Block().to(DEV, torch.bfloat16).eval()
    x = torch.randn(256, 512, device=DEV, dtype=torch.bfloat16)
    torch._dynamo.reset()
    runtime.check_status()
    f = torch.compile(m, backend=custom_backend)
    with torch.no_grad():
        want = f(x).clone()
        torch.ops.b200.gemm_test_stall_next(50_000_000)
        f(x)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="timed out"):
            f(x)
        got = f(x)
        runtime.check_status()
    assert torch.equal(got, want)


def test_check_status_raises_after_a_stalled_gemm():
    a = torch.randn(256, 512, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(512, 512, device=DEV, dtype=torch.bfloat16)
    runtime.check_status()
    from compiler.optimization.program import OP

    torch.ops.b200.gemm_test_stall_next(50_000_000)
    torch.ops.b200.gemm_epilogue(a, w.t(), [], [OP["MOV"] * 10], [0.0], [256, 512], torch.bfloat16,
                                 [1, -1, 0, -1, -1, -1])
    with pytest.raises(RuntimeError, match="status 6"):
        runtime.check_status()
    runtime.check_status()  # cleared


def test_fp32_mlp_fuses_on_tf32_when_allowed():
    """With torch's allow_tf32 on, the fp32 MLP's two GEMMs take the
    library's TF32 kernels (bias + tanh-GELU, bias + residual) and match
    eager cuBLAS TF32; with it off they stay cuBLAS fp32, as in the
    reference (compiler/optimization/fusion_epilogue.py:82-86)."""
    import sweep_inputs as si

    m, x = si.mlp()
    old = torch.backends.cuda.matmul.allow_tf32
    try:
        for allow in (True, False):
            torch.backends.cuda.matmul.allow_tf32 = allow
            torch._dynamo.reset()
            be, graphs = capturing_backend()
            with torch.no_grad():
                want = m(x)
                got = torch.compile(m, backend=be)(x)
            t = [str(s) for s in b200_targets(graphs)]
            assert t.count("b200.gemm_epilogue.default") == (2 if allow else 0)
            assert _rel(got, want) < (5e-3 if allow else 1e-5)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    runtime.check_status()
