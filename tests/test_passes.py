"""CPU tests of the FX passes: grouping parity with the reference, program
lowering (checked through the machine emulator against the reference's own
kernel outputs), and the documented extensions."""
import random

import numpy as np
import pytest
import torch
import torch.fx as fx
import torch.nn as nn
import torch.nn.functional as F

import machine_emulator
import oracle
import spec_graph
from cases import CASES, make_case
from compiler.optimization.program import MAX_SLOTS, ProgramError, compile_group
from helpers import fused_graphs, kernels_of

aten = torch.ops.aten


@pytest.mark.parametrize("case", CASES)
def test_grouping_matches_reference(golden, case):
    """With the extensions off, the passes make the reference's decisions:
    same kernels, same kind, same member ops, same order."""
    meta, _ = golden
    model, inputs = make_case(case)
    graphs = fused_graphs(model, inputs, extensions=False)
    ours = [(k, ops) for gm in graphs for k, ops, _ in kernels_of(gm)]
    ref = [(k, ops) for k, ops in meta["models"][case]["groups"]]
    assert ours == ref


@pytest.mark.parametrize("case", CASES)
def test_operand_order_matches_reference(golden, case):
    """Each fused node takes the reference closure's argument order:
    (*external_inputs) for pointwise, (mat1, mat2, bias?, *externals) for GEMM."""
    meta, _ = golden
    model, inputs = make_case(case)
    graphs = fused_graphs(model, inputs, extensions=False)
    ref = [k for k in meta["kernels"] if k["case"] == case and k["calls"]]
    ours = [n for gm in graphs for _, _, n in kernels_of(gm)]
    assert len(ours) == len(ref)
    for n, k in zip(ours, ref):
        operands = n.args[0] if k["kind"] == "pointwise" else n.args[2]
        assert len(operands) == k["n_inputs"]


def _lower(ent):
    if ent["kind"] == "pointwise":
        nodes, ops = spec_graph.build(ent["spec"], ent["n_inputs"])
        return compile_group(nodes, ops)
    nodes, ops = spec_graph.build(ent["spec"], ent["n_inputs"], with_acc=True)
    pro = [("ADD", ops[1])] if ent["bias_first"] else None
    return compile_group(nodes, ops, prologue=pro, prologue_target=ops[0])


def _golden_ids():
    import json
    import os

    with open(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.json")) as f:
        return [i for i, k in enumerate(json.load(f)["kernels"]) if k["calls"]]


@pytest.mark.parametrize("k", _golden_ids())
def test_lowered_program_reproduces_reference_kernel(golden, k):
    meta, arrays = golden
    ent = meta["kernels"][k]
    prog = _lower(ent)
    ins = [arrays[f"k{k}_in{i}"] for i in range(ent["n_inputs"])]
    shape = tuple(ent["out_shape"])
    if ent["kind"] == "gemm_epilogue":
        ins = [arrays[f"k{k}_a"] @ arrays[f"k{k}_b"]] + ins
    slots = [np.broadcast_to(x.astype(np.float32), shape) for x in ins]
    got = oracle.round_to(machine_emulator.run(prog.code, prog.imm, slots), ent["out_dtype"])
    rtol, atol = (1e-5, 1e-6) if ent["out_dtype"] == "float32" else (2e-3, 1e-3)
    if ent["kind"] == "gemm_epilogue":
        rtol, atol = max(rtol, 1e-3), max(atol, 1e-3)
    np.testing.assert_allclose(got, arrays[f"k{k}_out"], rtol=rtol, atol=atol)


UNARY = ["neg.default", "abs.default", "relu.default", "exp.default", "sigmoid.default", "tanh.default",
         "erf.default"]
BINARY = ["add.Tensor", "sub.Tensor", "mul.Tensor", "div.Tensor", "maximum.default", "minimum.default"]


def _random_spec(rng: random.Random, n_in: int, n_ops: int):
    spec = []
    for j in range(n_ops):
        def pick():
            r = rng.random()
            if r < 0.2:
                return round(rng.uniform(-2, 2), 3)
            if r < 0.55 or j == 0:
                return ["in", rng.randrange(n_in)]
            return ["node", rng.randrange(j)]

        if rng.random() < 0.35:
            a = pick()
            if not isinstance(a, list):
                a = ["in", 0]
            spec.append([rng.choice(UNARY), [a]])
        else:
            a, b = pick(), pick()
            if not isinstance(a, list) and not isinstance(b, list):
                a = ["in", rng.randrange(n_in)]
            spec.append([rng.choice(BINARY), [a, b]])
    return spec


@pytest.mark.parametrize("seed", range(60))
def test_lowering_random_dags(seed):
    """Random expression DAGs (shared subexpressions, operands reused,
    scalar on either side): lowering + emulation == direct evaluation."""
    rng = random.Random(seed)
    n_in = rng.randint(1, 5)
    spec = _random_spec(rng, n_in, rng.randint(2, 14))
    nodes, ops = spec_graph.build(spec, n_in)
    try:
        prog = compile_group(nodes, ops)
    except ProgramError:
        pytest.skip("needs more than the machine's slots")
    npr = np.random.default_rng(seed)
    ins = [npr.standard_normal((5, 7)).astype(np.float32) for _ in range(n_in)]
    want = oracle.eval_group(spec, ins, (5, 7), "float32")
    got = machine_emulator.run(prog.code, prog.imm, ins)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6, equal_nan=True)


def test_program_rejects_too_many_live_values():
    g = fx.Graph()
    ins = [g.placeholder(f"x{i}") for i in range(MAX_SLOTS)]
    # sum of pairwise products keeps every input live until the end
    nodes = []
    acc = None
    for i in range(MAX_SLOTS):
        p = g.call_function(aten.mul.Tensor, (ins[i], ins[(i + 1) % MAX_SLOTS]))
        nodes.append(p)
        if acc is not None:
            acc = g.call_function(aten.add.Tensor, (acc, p))
            nodes.append(acc)
        else:
            acc = p
    extra = g.call_function(aten.mul.Tensor, (nodes[0], nodes[2]))
    nodes.append(extra)
    with pytest.raises(ProgramError):
        compile_group(nodes + [g.call_function(aten.add.Tensor, (acc, extra))], ins)


# ------------------------------------------------------------- extensions
class RMSSwiGLU(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.weight = nn.Parameter(1 + 0.02 * torch.randn(d))

    def forward(self, h):
        dt = h.dtype
        x = h.to(torch.float32)
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
        y = self.weight * x.to(dt)
        g, u = y.split(y.shape[-1] // 2, dim=-1)
        return F.silu(g) * u


class RMSOnly(RMSSwiGLU):
    def forward(self, h):
        dt = h.dtype
        x = h.to(torch.float32)
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-5)
        return self.weight * x.to(dt)


def _targets(gm):
    return [n.target for n in gm.graph.nodes if n.op == "call_function"]


def test_rmsnorm_swiglu_becomes_one_kernel():
    (gm,) = fused_graphs(RMSSwiGLU(64).to(torch.bfloat16), (torch.randn(4, 64).to(torch.bfloat16),))
    t = _targets(gm)
    assert t == [torch.ops.b200.rms_norm_swiglu.default]
    n = next(n for n in gm.graph.nodes if n.op == "call_function")
    assert n.args[2] == pytest.approx(1e-6) and n.args[3] == 7 and n.args[4] == torch.bfloat16


def test_rmsnorm_alone_and_fp32():
    (gm,) = fused_graphs(RMSOnly(64).to(torch.bfloat16), (torch.randn(2, 3, 64).to(torch.bfloat16),))
    assert _targets(gm) == [torch.ops.b200.rms_norm.default]
    n = next(n for n in gm.graph.nodes if n.op == "call_function")
    assert n.args[3] == 1  # round the normalised value to bf16 before the weight
    (gm,) = fused_graphs(RMSOnly(64), (torch.randn(2, 64),))
    n = next(n for n in gm.graph.nodes if n.op == "call_function")
    assert n.target == torch.ops.b200.rms_norm.default and n.args[3] == 0


def test_rmsnorm_not_fused_when_intermediate_escapes():
    class Leak(nn.Module):
        def forward(self, h):
            x = h.to(torch.float32)
            v = x.pow(2).mean(-1, keepdim=True)
            return x * torch.rsqrt(v + 1e-6), v

    (gm,) = fused_graphs(Leak(), (torch.randn(4, 64).to(torch.bfloat16),))
    assert aten.mean.dim in _targets(gm)


def test_layernorm_softmax_and_3d_linear_lookthrough():
    class Blk(nn.Module):
        def __init__(self):
            super().__init__()
            self.ln = nn.LayerNorm(64)
            self.fc = nn.Linear(64, 128)
            self.fc2 = nn.Linear(128, 64)

        def forward(self, x):
            return self.fc2(F.gelu(self.fc(self.ln(x)))) + x, torch.softmax(x, -1)

    x = torch.randn(2, 5, 64).to(torch.bfloat16)
    (gm,) = fused_graphs(Blk().to(torch.bfloat16), (x,))
    t = _targets(gm)
    assert torch.ops.b200.layer_norm.default in t
    assert torch.ops.b200.softmax.default in t
    assert t.count(torch.ops.b200.gemm_epilogue.default) == 2
    assert aten.addmm.default not in t
    # Without the extensions the reference's rules apply: no 3-d anchor, no row kernels.
    (gm,) = fused_graphs(Blk().to(torch.bfloat16), (x,), extensions=False)
    t = _targets(gm)
    assert torch.ops.b200.gemm_epilogue.default not in t and aten.native_layer_norm.default in t


def test_fp32_gemm_left_to_aten():
    """fp32 matmuls (no TF32) stay cuBLAS; their pointwise tail is fused."""
    model, inputs = make_case("mlp_tanh_fp32")
    (gm,) = fused_graphs(model, inputs)
    t = _targets(gm)
    assert aten.addmm.default in t and torch.ops.b200.pointwise.default in t


def _epi_nodes(model, inputs):
    from helpers import fused_graphs as fg
    (gm,) = fg(model, inputs)
    return [n for n in gm.graph.nodes if n.op == "call_function" and n.target == torch.ops.b200.gemm_epilogue.default]


@pytest.mark.parametrize("act,code", [("none", 0), ("gelu", 1), ("silu", 3)])
def test_sweep_epilogues_take_the_compiled_path(act, code):
    import bench_models as bm
    m = bm.GemmEpilogueBlock(64, 128, act).to(torch.bfloat16)
    (n,) = _epi_nodes(m, (torch.randn(32, 64).to(torch.bfloat16), torch.randn(32, 128).to(torch.bfloat16)))
    rnd = -1 if act == "none" else 2  # bf16 rounding after the activation
    assert list(n.args[7]) == [1, 0, code, rnd, -1, 1]


def test_canonical_form_variants():
    """MLPBlock fc2 (x + tanh(y)*scale), tanh-GELU, and a non-canonical chain."""
    model, inputs = make_case("mlp_block_fp16")
    forms = [list(n.args[7]) for n in _epi_nodes(model, inputs)]
    assert [1, 0, 6, -1, 1, 2] in forms        # bias, tanh, *scale, +x
    assert [1, 0, 1, -1, -1, -1] in forms       # bias, gelu(erf)
    model, inputs = make_case("mlp_tanh_fp16")
    forms = [list(n.args[7]) for n in _epi_nodes(model, inputs)]
    assert [1, 0, 2, -1, -1, -1] in forms and [1, 0, 0, -1, -1, 1] in forms

    class Odd(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc = nn.Linear(64, 64)

        def forward(self, x):
            return torch.exp(self.fc(x)) * x - 1.0

    (n,) = _epi_nodes(Odd().half(), (torch.randn(16, 64).half(),))
    assert list(n.args[7]) == []  # interpreted


def test_residual_without_bias_takes_the_residual_role():
    """x + o(a) with a bias-free Linear: the full [M, N] operand is the
    residual (streamed by the compiled path), never the bias, which only a
    row vector can be."""
    class Res(nn.Module):
        def __init__(self):
            super().__init__()
            self.o = nn.Linear(64, 64, bias=False)

        def forward(self, x, a):
            return x + self.o(a)

    x = torch.randn(2, 8, 64).to(torch.bfloat16)
    forms = [list(n.args[7]) for n in _epi_nodes(Res().to(torch.bfloat16), (x, x.clone()))]
    assert forms == [[1, -1, 0, -1, -1, 0]]


def test_llama_gate_up_epilogue_is_canonical():
    """silu(gate(h)) * up(h): the gate GEMM's epilogue multiplies by the up GEMM output."""
    class SwiGLU(nn.Module):
        def __init__(self):
            super().__init__()
            self.g = nn.Linear(64, 128, bias=False)
            self.u = nn.Linear(64, 128, bias=False)

        def forward(self, h):
            return F.silu(self.g(h)) * self.u(h)

    forms = [list(n.args[7]) for n in _epi_nodes(SwiGLU().to(torch.bfloat16), (torch.randn(2, 8, 64).to(torch.bfloat16),))]
    assert [1, -1, 3, 2, 0, -1] in forms


def test_pointwise_keeps_permuted_layout():
    """An elementwise chain on a transposed view keeps ATen's output layout."""
    class Rope(nn.Module):
        def forward(self, q, c, s):
            q = q.transpose(1, 2)
            return q * c + torch.neg(q) * s

    q = torch.randn(2, 8, 4, 16)
    c = torch.randn(8, 16)
    (gm,) = fused_graphs(Rope(), (q, c, c))
    n = next(n for n in gm.graph.nodes if n.op == "call_function" and n.target == torch.ops.b200.pointwise.default)
    assert list(n.args[5]) == list(n.meta["val"].stride()) and not n.meta["val"].is_contiguous()


class _RopeLlama(nn.Module):
    """Llama's rotate_half (chunk -> split) on a transposed q."""

    def forward(self, q, c, s):
        q = q.transpose(1, 2)
        x1, x2 = q.chunk(2, dim=-1)
        return q * c + torch.cat((-x2, x1), dim=-1) * s


class _RopeHF(nn.Module):
    """The slice form of rotate_half, cos / sin broadcast from [B, 1, S, D]."""

    def forward(self, q, c, s):
        x1 = q[..., : q.shape[-1] // 2]
        x2 = q[..., q.shape[-1] // 2:]
        return (q * c) + (torch.cat((-x2, x1), dim=-1) * s)


def _rope_nodes(gm):
    return [n for n in gm.graph.nodes if n.op == "call_function" and n.target == torch.ops.b200.rope.default]


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_rope_pass_replaces_rotate_half_group(dt):
    q = torch.randn(2, 16, 4, 64).to(dt)
    c = torch.randn(16, 64).to(dt)
    (gm,) = fused_graphs(_RopeLlama(), (q, c, c.clone()))
    (n,) = _rope_nodes(gm)
    ops = {str(m.target) for m in gm.graph.nodes if m.op == "call_function"}
    assert not any(k in o for o in ops for k in ("cat", "neg", "split", "mul", "add"))
    eager = _RopeLlama()(q, c, c)
    assert list(n.args[3]) == list(eager.stride())  # the decomposed graph's layout
    q2 = torch.randn(2, 4, 16, 64).to(dt)
    c2 = torch.randn(2, 1, 16, 64).to(dt)
    (gm,) = fused_graphs(_RopeHF(), (q2, c2, c2.clone()))
    assert len(_rope_nodes(gm)) == 1


def test_rope_pass_leaves_other_chains():
    q = torch.randn(2, 16, 4, 64)
    c = torch.randn(16, 64)
    (gm,) = fused_graphs(_RopeLlama(), (q, c, c.clone()))  # fp32: no fused kernel for it
    assert not _rope_nodes(gm)

    class Swapped(nn.Module):  # cat(x1, -x2) is not rotate_half
        def forward(self, q, c, s):
            q = q.transpose(1, 2)
            x1, x2 = q.chunk(2, dim=-1)
            return q * c + torch.cat((x1, -x2), dim=-1) * s

    qb, cb = q.to(torch.bfloat16), c.to(torch.bfloat16)
    (gm,) = fused_graphs(Swapped(), (qb, cb, cb.clone()))
    assert not _rope_nodes(gm)
    (gm,) = fused_graphs(_RopeLlama(), (qb, cb, cb.clone()), extensions=False)
    assert not _rope_nodes(gm)


def test_llama_layer_fuses_both_rotations():
    import bench_models as bm

    layer = bm.LlamaLayer(128, 4, 2, 256, 1e-5).to(torch.bfloat16)
    m = bm.Llama(vocab=32, dim=128, layers=1, heads=4, kv_heads=2, ffn=256, max_seq=16)
    x = torch.randn(1, 16, 128).to(torch.bfloat16)
    cos, sin = m.cos[:16].to(torch.bfloat16), m.sin[:16].to(torch.bfloat16)
    graphs = fused_graphs(layer, (x, cos, sin))
    # 32-wide heads: the rotations stay kernels of their own
    assert sum(len(_rope_nodes(g)) for g in graphs) == 2


def test_rotated_projection_with_broadcast_tables():
    """cos / sin given as [1, 1, S, 64] tables (the Hugging Face layout) are
    viewed as [S, 64] for the rotary GEMM."""
    import bench_models as bm

    class HFStyle(nn.Module):
        def __init__(self):
            super().__init__()
            self.q = nn.Linear(256, 256, bias=False)

        def forward(self, x, cos, sin):
            B, S, _ = x.shape
            q = self.q(x).view(B, S, 4, 64).transpose(1, 2)
            return q * cos + bm._rotate_half(q) * sin

    m = bm.Llama(vocab=32, dim=256, layers=0, heads=4, kv_heads=2, ffn=256, max_seq=16)
    cos, sin = (t[:16].to(torch.bfloat16)[None, None] for t in (m.cos, m.sin))
    (gm,) = fused_graphs(HFStyle().to(torch.bfloat16), (torch.randn(2, 16, 256).to(torch.bfloat16), cos, sin))
    (node,) = [n for n in gm.graph.nodes if n.op == "call_function" and n.target == torch.ops.b200.gemm_rope.default]
    for t in node.args[2:4]:
        assert tuple(t.meta["val"].shape) == (16, 64)
    assert node.args[4] == 16 and tuple(node.meta["val"].shape) == (2, 16, 256)


def test_rotated_projection_pass_rules():
    """The q / k projection folds into gemm_rope only for a plain mm viewed
    as 64-wide heads; a projection read by anything else, an fp32 one, or
    extensions off keep the separate rotation (or no rotation kernel)."""
    import bench_models as bm

    def graph_of(layer, dt=torch.bfloat16, extensions=True):
        m = bm.Llama(vocab=32, dim=256, layers=0, heads=4, kv_heads=2, ffn=256, max_seq=16)
        x = torch.randn(2, 16, 256).to(dt)
        cos, sin = m.cos[:16].to(dt), m.sin[:16].to(dt)
        (gm,) = fused_graphs(layer.to(dt), (x, cos, sin), extensions=extensions)
        return [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]

    class LeakQ(bm.LlamaLayer):
        def forward(self, x, cos, sin):
            B, S, _ = x.shape
            q = self.q(self.in_norm(x)).view(B, S, self.h, self.hd).transpose(1, 2)
            return q * cos + bm._rotate_half(q) * sin, q  # the unrotated heads escape

    t = graph_of(bm.LlamaLayer(256, 4, 2, 256, 1e-5))
    assert t.count("b200.gemm_rope.default") == 2 and "b200.rope.default" not in t
    t = graph_of(LeakQ(256, 4, 2, 256, 1e-5))
    assert "b200.gemm_rope.default" not in t and t.count("b200.rope.default") == 1
    t = graph_of(bm.LlamaLayer(256, 4, 2, 256, 1e-5), extensions=False)
    assert "b200.gemm_rope.default" not in t and "b200.rope.default" not in t
    t = graph_of(bm.LlamaLayer(256, 4, 2, 256, 1e-5), dt=torch.float32)
    assert "b200.gemm_rope.default" not in t


class _Patch(nn.Module):
    def __init__(self, bias=True):
        super().__init__()
        self.proj = nn.Conv2d(3, 32, 16, 16, bias=bias)

    def forward(self, img):
        return self.proj(img).flatten(2).transpose(1, 2)


@pytest.mark.parametrize("bias", [True, False])
def test_patchify_lowers_patch_conv_to_gemm(bias):
    """A kernel == stride convolution becomes im2col + (add)mm with the
    convolution's NCHW result layout; the rewritten graph computes the same
    values as the convolution (run here on CPU in fp32 arithmetic)."""
    torch.manual_seed(0)
    model = _Patch(bias).to(torch.bfloat16)
    img = torch.randn(2, 3, 64, 64).to(torch.bfloat16)
    (gm,) = fused_graphs(model, (img,))
    targets = [n.target for n in gm.graph.nodes if n.op == "call_function"]
    assert torch.ops.aten.convolution.default not in targets
    assert (torch.ops.aten.addmm.default if bias else torch.ops.aten.mm.default) in targets
    # numerics of the lowering itself: conv2d == im2col @ w^T (+ b), fp32 on CPU
    x, w = img.float(), model.proj.weight.float()
    p = x.view(2, 3, 4, 16, 4, 16).permute(0, 2, 4, 1, 3, 5).reshape(32, 768)
    y = p @ w.view(32, 768).t() + (model.proj.bias.float() if bias else 0)
    ref = torch.nn.functional.conv2d(x, w, model.proj.bias.float() if bias else None, stride=16)
    torch.testing.assert_close(y.view(2, 4, 4, 32).permute(0, 3, 1, 2), ref, rtol=1e-4, atol=1e-4)
    # flatten(2).transpose(1, 2): the GEMM's [B*HW, OC] rows are the tokens, so
    # the transpose and the NCHW copy are gone and the result is a view
    assert torch.ops.aten.transpose.int not in targets
    clones = [n for n in gm.graph.nodes if n.target == torch.ops.aten.clone.default]
    assert len(clones) == 1 and tuple(clones[0].meta["val"].shape) == (2, 4, 4, 3, 16, 16)  # im2col only
    out = [n for n in gm.graph.nodes if n.op == "output"][0].args[0][0]
    val = out.meta["val"]
    assert tuple(val.shape) == (2, 16, 32) and val.is_contiguous()


def test_patchify_keeps_the_nchw_layout_for_other_uses():
    """A patch convolution whose result is used as an image (here: a
    pointwise op on the NCHW tensor) gets the permute-back copy, so every
    later node sees the layout it was traced with."""

    class PatchAct(nn.Module):
        def __init__(self):
            super().__init__()
            self.proj = nn.Conv2d(3, 32, 16, 16)

        def forward(self, img):
            return torch.relu(self.proj(img))

    (gm,) = fused_graphs(PatchAct().to(torch.bfloat16), (torch.randn(2, 3, 64, 64).to(torch.bfloat16),))
    targets = [n.target for n in gm.graph.nodes if n.op == "call_function"]
    assert torch.ops.aten.convolution.default not in targets
    clones = [n for n in gm.graph.nodes if n.target == torch.ops.aten.clone.default]
    assert [tuple(n.meta["val"].shape) for n in clones] == [(2, 4, 4, 3, 16, 16), (2, 32, 4, 4)]
    assert clones[1].meta["val"].is_contiguous()


def test_broadcast_cat_inputs_are_made_contiguous():
    """ViT's class-token concatenation: the expanded (zero-stride) input of
    the cat gets a contiguous copy, the token input is left alone, and the
    values are the same."""

    class ClsCat(nn.Module):
        def __init__(self):
            super().__init__()
            self.cls = nn.Parameter(torch.randn(1, 1, 32))

        def forward(self, x):
            return torch.cat([self.cls.expand(x.shape[0], -1, -1), x], dim=1) * 2

    model = ClsCat().to(torch.bfloat16)
    x = torch.randn(4, 6, 32).to(torch.bfloat16)
    (gm,) = fused_graphs(model, (x,))
    cat = [n for n in gm.graph.nodes if n.target == torch.ops.aten.cat.default][0]
    first, second = cat.args[0]
    assert first.target == torch.ops.aten.clone.default and first.args[0].target == torch.ops.aten.expand.default
    assert first.meta["val"].is_contiguous() and tuple(first.meta["val"].shape) == (4, 1, 32)
    assert second.target != torch.ops.aten.clone.default


def test_patchify_leaves_overlapping_convolutions():
    class Conv(nn.Module):
        def __init__(self):
            super().__init__()
            self.c = nn.Conv2d(3, 8, 3, 1, padding=1)

        def forward(self, x):
            return self.c(x)

    (gm,) = fused_graphs(Conv().to(torch.bfloat16), (torch.randn(1, 3, 16, 16).to(torch.bfloat16),))
    assert torch.ops.aten.convolution.default in [n.target for n in gm.graph.nodes if n.op == "call_function"]


def test_epilogue_profitability_rule():
    """The measured cost model: fused wherever the benchmark and model
    shapes put a pointwise tail on a GEMM; cuBLAS plus a separate kernel for
    a deep GEMM whose tail is too small to pay for the library's gap."""
    from compiler.optimization.fusion_epilogue import fusion_pays

    bf = 2
    # the sweep's points (bias + act + bf16 residual)
    for M, N, K in [(512, 512, 512), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 4096, 14336)]:
        assert fusion_pays(M, N, K, bf, bf, M * N * bf + N * bf)
    # ViT fc1 (bias + GELU), fc2 / proj (bias + residual); Llama gate (x up), down (+ residual)
    assert fusion_pays(12608, 3072, 768, bf, bf, 3072 * bf)
    assert fusion_pays(12608, 768, 3072, bf, bf, 12608 * 768 * bf + 768 * bf)
    assert fusion_pays(16384, 8192, 2048, bf, bf, 16384 * 8192 * bf)
    assert fusion_pays(16384, 2048, 8192, bf, bf, 16384 * 2048 * bf)
    # a deep GEMM with an activation alone: the tail (one 33 MB round trip)
    # is smaller than the library's 6 % gap on 550 GFLOP
    assert not fusion_pays(4096, 4096, 16384, bf, bf, 0)


def test_attention_pass_rewrites_sdpa_nodes():
    """ViT's and the Llama block's scaled-dot-product attention become
    b200.attention nodes (causal flag, default scale, the replaced node's
    output layout); head_dim other than 64 stays in ATen."""
    import bench_models as bm
    from compiler.optimization import config

    old = config.ENABLE_ATTENTION
    config.ENABLE_ATTENTION = True
    try:
        _attention_pass_checks(bm)
    finally:
        config.ENABLE_ATTENTION = old


def _attention_pass_checks(bm):
    torch.manual_seed(0)
    vit = bm.ViT(depth=1).to(torch.bfloat16).eval()
    (g,) = fused_graphs(vit, [torch.randn(2, 3, 224, 224).to(torch.bfloat16)])
    att = [n for n in g.graph.nodes if n.op == "call_function" and n.target == torch.ops.b200.attention.default]
    assert len(att) == 1 and att[0].args[3] is False and att[0].args[4] == -1.0
    assert list(att[0].meta["val"].stride()) == list(att[0].args[5])

    llama = bm.Llama(vocab=256, dim=256, layers=2, heads=4, kv_heads=2, ffn=256, max_seq=64).to(torch.bfloat16).eval()
    (g,) = fused_graphs(llama, [torch.randint(0, 256, (2, 64))])
    att = [n for n in g.graph.nodes if n.op == "call_function" and n.target == torch.ops.b200.attention.default]
    assert len(att) == 2 and all(n.args[3] is True for n in att)
    q, k = (n.meta["val"] for n in att[0].args[:2])
    assert q.shape[1] == 4 and k.shape[1] == 2  # grouped-query heads passed through

    small = bm.Llama(vocab=256, dim=128, layers=1, heads=4, kv_heads=2, ffn=256, max_seq=64).to(torch.bfloat16).eval()
    (g,) = fused_graphs(small, [torch.randint(0, 256, (2, 64))])
    assert not any(n.target == torch.ops.b200.attention.default for n in g.graph.nodes if n.op == "call_function")


def test_fp32_epilogue_fusion_follows_allow_tf32():
    """fp32 GEMMs are fused (TF32 kernels) only while torch allows TF32,
    the reference's rule for its fp32 dots; otherwise they stay ATen."""
    model, inputs = make_case("mlp_block_fp32")
    old = torch.backends.cuda.matmul.allow_tf32
    try:
        counts = {}
        for allow in (True, False):
            torch.backends.cuda.matmul.allow_tf32 = allow
            (g,) = fused_graphs(model, inputs)
            counts[allow] = sum(1 for n in g.graph.nodes if n.op == "call_function"
                                and n.target == torch.ops.b200.gemm_epilogue.default)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    assert counts[True] >= 1 and counts[False] == 0


def test_transposed_a_matmul_with_pointwise_tail_is_fused():
    """mm(t(g), x) -- the weight-gradient product of a backward graph -- with
    a pointwise consumer reaches the library (A read M-major), as the
    reference's anchor takes any 2-d mm with a pointwise tail
    (compiler/optimization/fusion_epilogue.py:45-69); an fp32 one without
    TF32 stays ATen."""

    class WGrad(nn.Module):
        def forward(self, g, x, c):
            return (g.t() @ x) * 0.5 + c

    g, x = torch.randn(96, 32).to(torch.bfloat16), torch.randn(96, 48).to(torch.bfloat16)
    c = torch.randn(32, 48).to(torch.bfloat16)
    nodes = _epi_nodes(WGrad(), (g, x, c))
    assert len(nodes) == 1
    a = nodes[0].args[0].meta["val"]
    assert a.shape == (32, 96) and a.stride() == (1, 32)
    (gm,) = fused_graphs(WGrad(), (g.float(), x.float(), c.float()))
    assert torch.ops.b200.gemm_epilogue.default not in _targets(gm)
