"""GPU parity of the sm_100a kernels, called through the C ABI (ctypes), against
the oracle and the reference kernels' recorded outputs.

Tolerances: fp32 pointwise 1e-5 relative (+1e-6 absolute); fp16/bf16 results
one rounding of the output dtype; GEMM + epilogue 2e-2 relative to an fp32
reference (scaled by the output's magnitude), as the task's parity bar states.
"""
import json
import os

import numpy as np
import pytest
import torch

import oracle
import spec_graph
from compiler import runtime
from compiler.optimization.program import OP, canonical_form, compile_group
from compiler.runtime import cabi

pytestmark = pytest.mark.gpu
DEV = "cuda"

with open(os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.json")) as _f:
    _META = json.load(_f)
GOLDEN_IDS = [i for i, k in enumerate(_META["kernels"]) if k["calls"]]

GELU_ERF = [["mul.Tensor", [["acc"], 0.5]], ["mul.Tensor", [["acc"], 0.7071067811865476]], ["erf.default", [["node", 1]]],
            ["add.Tensor", [["node", 2], 1.0]], ["mul.Tensor", [["node", 0], ["node", 3]]]]
SILU = [["sigmoid.default", [["acc"]]], ["mul.Tensor", [["acc"], ["node", 0]]]]
GELU_TANH = [["mul.Tensor", [["acc"], ["acc"]]], ["mul.Tensor", [["node", 0], ["acc"]]],
             ["mul.Tensor", [["node", 1], 0.044715]], ["add.Tensor", [["acc"], ["node", 2]]],
             ["mul.Tensor", [["node", 3], 0.7978845608028654]], ["mul.Tensor", [["acc"], 0.5]],
             ["tanh.default", [["node", 4]]], ["add.Tensor", [["node", 6], 1.0]],
             ["mul.Tensor", [["node", 5], ["node", 7]]]]
ACTS = {"none": [], "gelu": GELU_ERF, "silu": SILU, "gelu_tanh": GELU_TANH}


def _tdt(name):
    return getattr(torch, name)


def _assert_close(got: torch.Tensor, want: np.ndarray, rtol: float, atol: float):
    np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=rtol, atol=atol)


def _gemm_tol(want: np.ndarray) -> tuple[float, float]:
    return 2e-2, 2e-2 * float(np.abs(want).max() + 1e-6)


def epilogue_program(act: str, residual: bool, bias: bool = True):
    """Program for out = act(acc [+ bias]) [+ residual] with extras (bias, residual)."""
    spec = [list(s) for s in ACTS[act]]
    n_in = (1 if bias else 0) + (1 if residual else 0)
    if residual:
        last = ["node", len(spec) - 1] if spec else ["acc"]
        spec = spec + [["add.Tensor", [last, ["in", n_in - 1]]]]
    if not spec:
        spec = [["add.Tensor", [["acc"], 0.0]]] if not bias else []
    nodes, ops = spec_graph.build(spec, n_in, with_acc=True) if spec else (None, None)
    if spec:
        pro = [("ADD", ops[1])] if bias else None
        prog = compile_group(nodes, ops, prologue=pro, prologue_target=ops[0], rounding_casts=True)
        return prog.code, prog.imm, spec, canonical_form(prog, 1 + n_in)
    # bias only: acc + bias
    return [OP["MOV"] * 10, OP["ADD"] * 10 + 1], [0.0, 0.0], [], [1, 0, 0, -1, -1, -1]


@pytest.fixture(scope="module", autouse=True)
def _lib():
    runtime.load()
    cabi.library()


@pytest.mark.parametrize("k", [i for i in GOLDEN_IDS if _META["kernels"][i]["kind"] == "pointwise"])
def test_golden_pointwise_kernel(golden, k):
    meta, arrays = golden
    ent = meta["kernels"][k]
    nodes, ops = spec_graph.build(ent["spec"], ent["n_inputs"])
    prog = compile_group(nodes, ops)
    ins = [torch.from_numpy(arrays[f"k{k}_in{i}"]).to(DEV, _tdt(ent["in_dtypes"][i])) for i in range(ent["n_inputs"])]
    out = torch.empty(ent["out_shape"], device=DEV, dtype=_tdt(ent["out_dtype"]))
    cabi.pointwise(ins, prog.code, prog.imm, out)
    torch.cuda.synchronize()
    rtol, atol = (1e-5, 1e-6) if ent["out_dtype"] == "float32" else (2e-3, 1e-3)
    _assert_close(out, arrays[f"k{k}_out"], rtol, atol)
    # the oracle agrees on the same inputs
    want = oracle.eval_group(ent["spec"], [arrays[f"k{k}_in{i}"] for i in range(ent["n_inputs"])],
                             tuple(ent["out_shape"]), ent["out_dtype"])
    _assert_close(out, want, rtol, atol)


@pytest.mark.parametrize("k", [i for i in GOLDEN_IDS if _META["kernels"][i]["kind"] == "gemm_epilogue"])
@pytest.mark.parametrize("b_layout", ["k_major", "n_major"])
def test_golden_gemm_epilogue_kernel(golden, k, b_layout):
    meta, arrays = golden
    ent = meta["kernels"][k]
    nodes, ops = spec_graph.build(ent["spec"], ent["n_inputs"], with_acc=True)
    pro = [("ADD", ops[1])] if ent["bias_first"] else None
    prog = compile_group(nodes, ops, prologue=pro, prologue_target=ops[0])
    dt = _tdt(ent["ab_dtype"])
    a = torch.from_numpy(arrays[f"k{k}_a"]).to(DEV, dt)
    bnp = arrays[f"k{k}_b"]
    b = torch.from_numpy(bnp.T.copy()).to(DEV, dt).t() if b_layout == "k_major" else torch.from_numpy(bnp).to(DEV, dt)
    extras = [torch.from_numpy(arrays[f"k{k}_in{i}"]).to(DEV, _tdt(ent["in_dtypes"][i])) for i in range(ent["n_inputs"])]
    out = torch.empty(ent["out_shape"], device=DEV, dtype=_tdt(ent["out_dtype"]))
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    cabi.gemm_epilogue(a, b, extras, prog.code, prog.imm, out, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    _assert_close(out, arrays[f"k{k}_out"], 2e-3, 2e-3)


SWEEP = [(512, 512, 512), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 4096, 14336)]


@pytest.mark.parametrize("shape", SWEEP)
@pytest.mark.parametrize("act", ["none", "gelu", "silu"])
@pytest.mark.parametrize("path", ["compiled", "interpreted"])
def test_gemm_sweep_configs(shape, act, path):
    """The fused GEMM sweep at its full sizes, Y = act(X W^T + b) + R in bf16,
    through the compiled epilogue path and the program interpreter; checked
    on 192 sampled rows against the fp32 oracle."""
    M, N, K = shape
    g = torch.Generator(device=DEV).manual_seed(0)
    x = (0.02 * torch.randn(M, K, device=DEV, generator=g)).to(torch.bfloat16)
    w = (0.02 * torch.randn(N, K, device=DEV, generator=g)).to(torch.bfloat16)
    b = (0.01 * torch.randn(N, device=DEV, generator=g)).to(torch.bfloat16)
    r = (0.02 * torch.randn(M, N, device=DEV, generator=g)).to(torch.bfloat16)
    code, imm, spec, form = epilogue_program(act, residual=True)
    assert form is not None
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, out, status=status, form=form if path == "compiled" else None)
    torch.cuda.synchronize()
    assert status.item() == 0
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(1))[:192].sort().values
    rows[0], rows[-1] = 0, M - 1
    xs = x[rows.to(DEV)].float().cpu().numpy()
    want = oracle.gemm_epilogue(xs, w.float().cpu().numpy().T, spec,
                                [b.float().cpu().numpy(), r[rows.to(DEV)].float().cpu().numpy()], "bfloat16",
                                bias=b.float().cpu().numpy())
    _assert_close(out[rows.to(DEV)], want, *_gemm_tol(want))


@pytest.mark.parametrize("M,N,K", [(1, 8, 8), (37, 72, 24), (128, 256, 64), (130, 260, 72), (300, 100, 136),
                                   (257, 1000, 768), (64, 4096, 1024)])
@pytest.mark.parametrize("config", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("ab", ["bfloat16", "float16"])
@pytest.mark.parametrize("path", ["compiled", "interpreted"])
def test_gemm_edge_shapes(M, N, K, config, ab, path):
    """Ragged M/N/K (partial tiles, K tail inside a 64-wide block, M < 128,
    N whose rows are not 16-byte multiples -> direct-store path), every tile
    config (an interpreted epilogue forced to 192-wide or CTA-pair tiles
    runs 256-wide ones), both operand dtypes,
    gelu-tanh + bias + residual."""
    dt = _tdt(ab)
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N)
    x = torch.randn(M, K, device=DEV, generator=g).to(dt)
    w = torch.randn(N, K, device=DEV, generator=g).to(dt)
    b = torch.randn(N, device=DEV, generator=g).to(dt)
    r = torch.randn(M, N, device=DEV, generator=g).to(dt)
    code, imm, spec, form = epilogue_program("gelu_tanh", residual=True)
    assert form is not None
    out = torch.empty(M, N, device=DEV, dtype=dt)
    cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, out, tile_config=config,
                       form=form if path == "compiled" else None)
    torch.cuda.synchronize()
    want = oracle.gemm_epilogue(x.float().cpu().numpy(), w.float().cpu().numpy().T, spec,
                                [b.float().cpu().numpy(), r.float().cpu().numpy()], ab, bias=b.float().cpu().numpy())
    _assert_close(out, want, *_gemm_tol(want))


@pytest.mark.parametrize("pair_cfg", [3, 4])
@pytest.mark.parametrize("act", ["none", "gelu", "silu"])
@pytest.mark.parametrize("shape", [(256, 256, 64), (4096, 4096, 4096), (2000, 3000, 1600), (300, 520, 2048),
                                   (12608, 768, 3072), (1000, 1300, 4160)])
def test_gemm_pair_tiles_equal_single_cta_tiles(pair_cfg, act, shape):
    """256 x 256 and 256 x 512 tiles on CTA pairs (configs 3 and 4, tcgen05
    cta_group::2) against 128 x 256 tiles on single CTAs (config 0): the same
    MMAs over the same K order and the same epilogue, so the outputs are
    equal bit for bit, full and ragged tiles alike (N = 1300: a 512-wide tile
    whose second half is partly and wholly past N); and the fp32 oracle
    agrees on sampled rows."""
    M, N, K = shape
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    x = (0.02 * torch.randn(M, K, device=DEV, generator=g)).to(torch.bfloat16)
    w = (0.02 * torch.randn(N, K, device=DEV, generator=g)).to(torch.bfloat16)
    b = (0.01 * torch.randn(N, device=DEV, generator=g)).to(torch.bfloat16)
    r = (0.02 * torch.randn(M, N, device=DEV, generator=g)).to(torch.bfloat16)
    code, imm, spec, form = epilogue_program(act, residual=True)
    outs = []
    for cfg in (pair_cfg, 0):
        out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, out, tile_config=cfg, status=status, form=form)
        torch.cuda.synchronize()
        assert status.item() == 0
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    rows = torch.arange(0, M, max(1, M // 64), device=DEV)
    want = oracle.gemm_epilogue(x[rows].float().cpu().numpy(), w.float().cpu().numpy().T, spec,
                                [b.float().cpu().numpy(), r[rows].float().cpu().numpy()], "bfloat16",
                                bias=b.float().cpu().numpy())
    _assert_close(outs[0][rows], want, *_gemm_tol(want))


def test_gemm_192_tiles_with_interpreted_epilogue_run_config_0():
    """Forcing the 192-wide config for an epilogue that is interpreted runs
    the 256-wide config instead, with the same result."""
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(200, 64, device=DEV, generator=g).to(torch.bfloat16)
    w = torch.randn(192, 64, device=DEV, generator=g).to(torch.bfloat16)
    b = torch.randn(192, device=DEV, generator=g).to(torch.bfloat16)
    code, imm, _, _ = epilogue_program("none", residual=False)
    outs = []
    for cfg in (2, 0):
        out = torch.empty(200, 192, device=DEV, dtype=torch.bfloat16)
        cabi.gemm_epilogue(x, w.t(), [b], code, imm, out, tile_config=cfg)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def role_program(act: str, role: str, round_to: str | None):
    """Program for out = [round(] act(acc + bias) [)] (+ m | * m) with extras
    (bias, m): the rounding cast, when given, sits where the decomposed graph
    of a 16-bit model has it, between the activation and the 16-bit op."""
    spec = [list(s) for s in ACTS[act]]
    last = ["node", len(spec) - 1] if spec else ["acc"]
    if round_to is not None:
        spec.append(["_to_copy.default", [last, round_to]])
        last = ["node", len(spec) - 1]
    spec.append(["add.Tensor" if role == "res" else "mul.Tensor", [last, ["in", 1]]])
    nodes, ops = spec_graph.build(spec, 2, with_acc=True)
    prog = compile_group(nodes, ops, prologue=[("ADD", ops[1])], prologue_target=ops[0], rounding_casts=True)
    return prog.code, prog.imm, spec, canonical_form(prog, 3)


@pytest.mark.parametrize("role", ["res", "scale"])
@pytest.mark.parametrize("act", ["none", "silu", "gelu"])
@pytest.mark.parametrize("dt", ["bfloat16", "float16"])
@pytest.mark.parametrize("rounded", [True, False])
@pytest.mark.parametrize("config", [0, 1, 2, 3, 4])
def test_gemm_row_operand_roles(role, act, dt, rounded, config):
    """A full 16-bit matrix as residual or scale, after an activation that is
    (rounded) or is not rounded to the output type first.  Rounded, the
    compiled path applies the op to packed 16-bit pairs; the result equals
    the interpreted program's bit for bit where both paths share the
    activation's implementation (none, silu) and the fp32 oracle within the
    GEMM tolerance everywhere.  Ragged M and N cover partial tiles."""
    M, N, K = 300, 520, 200
    t = _tdt(dt)
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randn(M, K, device=DEV, generator=g).to(t)
    w = (0.1 * torch.randn(N, K, device=DEV, generator=g)).to(t)
    b = torch.randn(N, device=DEV, generator=g).to(t)
    m = torch.randn(M, N, device=DEV, generator=g).to(t)
    code, imm, spec, form = role_program(act, role, dt if rounded else None)
    assert form is not None and form[3] == (B200K_DT[dt] if rounded else -1)
    assert form[5 if role == "res" else 4] == 1
    outs = {}
    for path in ("compiled", "interpreted"):
        out = torch.empty(M, N, device=DEV, dtype=t)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        cfg = 0 if (config >= 2 and path == "interpreted") else config  # 192-wide, pairs: compiled only
        cabi.gemm_epilogue(x, w.t(), [b, m], code, imm, out, tile_config=cfg, status=status,
                           form=form if path == "compiled" else None)
        torch.cuda.synchronize()
        assert status.item() == 0
        outs[path] = out
    if act != "gelu":
        assert torch.equal(outs["compiled"], outs["interpreted"])
    want = oracle.gemm_epilogue(x.float().cpu().numpy(), w.float().cpu().numpy().T, spec,
                                [b.float().cpu().numpy(), m.float().cpu().numpy()], dt, bias=b.float().cpu().numpy())
    _assert_close(outs["compiled"], want, *_gemm_tol(want))


B200K_DT = {"float32": 0, "float16": 1, "bfloat16": 2}


@pytest.mark.parametrize("out_dtype", ["float32", "float16"])
def test_gemm_extras_broadcast_and_strided(out_dtype):
    """Epilogue operands of every layout: [M,1] column, 0-d scalar, fp32 row
    vector, a transposed [M,N] view; N-major B; fp32 output."""
    M, N, K = 200, 320, 96
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(M, K, device=DEV, generator=g).half()
    bm = torch.randn(K, N, device=DEV, generator=g).half()  # N-major B
    col = torch.randn(M, 1, device=DEV, generator=g)
    scal = torch.tensor(1.5, device=DEV)
    rowv = torch.randn(N, device=DEV, generator=g)
    rt = torch.randn(N, M, device=DEV, generator=g).half().t()
    spec = [["mul.Tensor", [["acc"], ["in", 0]]], ["add.Tensor", [["node", 0], ["in", 1]]],
            ["maximum.default", [["node", 1], ["in", 2]]], ["sub.Tensor", [["node", 2], ["in", 3]]]]
    nodes, ops = spec_graph.build(spec, 4, with_acc=True)
    prog = compile_group(nodes, ops)
    out = torch.empty(M, N, device=DEV, dtype=_tdt(out_dtype))
    cabi.gemm_epilogue(x, bm, [col, scal, rowv, rt], prog.code, prog.imm, out)
    torch.cuda.synchronize()
    want = oracle.gemm_epilogue(x.float().cpu().numpy(), bm.float().cpu().numpy(), spec,
                                [t.float().cpu().numpy() for t in (col, scal, rowv, rt)], out_dtype)
    _assert_close(out, want, *_gemm_tol(want))


def test_gemm_repeated_calls_reuse_nothing_stale():
    """Two different problems back to back on one stream give independent results."""
    for M, N, K in [(256, 512, 128), (1024, 256, 64)]:
        x = torch.randn(M, K, device=DEV).to(torch.bfloat16)
        w = torch.randn(N, K, device=DEV).to(torch.bfloat16)
        out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
        cabi.gemm_epilogue(x, w.t(), [], [], [], out)
        torch.cuda.synchronize()
        want = x.float().cpu().numpy() @ w.float().cpu().numpy().T
        _assert_close(out, oracle.round_to(want, "bfloat16"), *_gemm_tol(want))


def test_gemm_rejects_bad_layout():
    """A with neither a unit K nor a unit M stride is refused with an error
    code, not computed wrongly; so is an fp32 M-major A (TF32 runs K-major
    operands only)."""
    x = torch.randn(64, 128, device=DEV).to(torch.bfloat16)[:, ::2]  # strides (128, 2)
    w = torch.randn(56, 64, device=DEV).to(torch.bfloat16)
    out = torch.empty(64, 56, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(cabi.CError) as e:
        cabi.gemm_epilogue(x, w.t(), [], [], [], out)
    assert e.value.code == 4
    xf = torch.randn(64, 64, device=DEV).t()  # fp32, strides (1, 64)
    outf = torch.empty(64, 56, device=DEV)
    with pytest.raises(cabi.CError) as e:
        cabi.gemm_epilogue(xf, torch.randn(56, 64, device=DEV).t(), [], [], [], outf)
    assert e.value.code == 4


@pytest.mark.parametrize("M,N,K", [(37, 72, 24), (128, 256, 64), (130, 260, 72), (300, 100, 136),
                                   (1000, 768, 264), (999, 768, 257), (2048, 1024, 4096)])
@pytest.mark.parametrize("b_layout", ["k_major", "n_major"])
@pytest.mark.parametrize("config", [0, 1, 3])
@pytest.mark.parametrize("ab", ["bfloat16", "float16"])
def test_gemm_m_major_a(M, N, K, b_layout, config, ab):
    """A stored M-major (unit M stride: the transposed gradient that a
    backward graph's weight-gradient mm reads), with K-major and N-major B,
    ragged shapes, gelu-tanh + bias + residual (interpreted), against the
    oracle; a forced CTA-pair config runs 128-row tiles."""
    dt = _tdt(ab)
    g = torch.Generator(device=DEV).manual_seed(M + 3 * N + K)
    m_pad = (M + 7) // 8 * 8  # the K stride (elements) keeps 16-byte rows
    x = torch.randn(K, m_pad, device=DEV, generator=g).to(dt)[:, :M].t()  # [M, K], strides (1, m_pad)
    assert x.stride() == (1, m_pad)
    w = torch.randn(N, K, device=DEV, generator=g).to(dt)
    # B [K, N] as t(W) (K-major) or row-major (N-major), rows padded to 16 bytes
    k_pad, n_pad = (K + 7) // 8 * 8, (N + 7) // 8 * 8
    if b_layout == "k_major":
        bmat = torch.zeros(N, k_pad, device=DEV, dtype=dt)[:, :K].copy_(w).t()
    else:
        bmat = torch.zeros(K, n_pad, device=DEV, dtype=dt)[:, :N].copy_(w.t())
    b = torch.randn(N, device=DEV, generator=g).to(dt)
    r = torch.randn(M, N, device=DEV, generator=g).to(dt)
    code, imm, spec, form = epilogue_program("gelu_tanh", residual=True)
    out = torch.empty(M, N, device=DEV, dtype=dt)
    cabi.gemm_epilogue(x, bmat, [b, r], code, imm, out, tile_config=config, form=form)
    torch.cuda.synchronize()
    want = oracle.gemm_epilogue(x.float().cpu().numpy(), w.float().cpu().numpy().T, spec,
                                [b.float().cpu().numpy(), r.float().cpu().numpy()], ab, bias=b.float().cpu().numpy())
    _assert_close(out, want, *_gemm_tol(want))
    if (K * x.element_size()) % 16:
        return  # a K-major copy of A would not have 16-byte rows
    # the same product from a K-major copy of A is bit-identical (same tiles, same MMA order)
    out2 = torch.empty_like(out)
    cabi.gemm_epilogue(x.contiguous(), bmat, [b, r], code, imm, out2, tile_config=config, form=None)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


# ------------------------------------------------------------- pointwise
def test_pointwise_broadcast_strided_and_dtypes():
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(33, 48, device=DEV, generator=g)
    xt = torch.randn(48, 33, device=DEV, generator=g).t()  # transposed view
    row = torch.randn(48, device=DEV, generator=g).half()
    col = torch.randn(33, 1, device=DEV, generator=g).to(torch.bfloat16)
    mask = torch.rand(33, 48, device=DEV, generator=g) > 0.5
    idx = torch.randint(-3, 3, (33, 48), device=DEV, generator=g, dtype=torch.int32)
    spec = [["mul.Tensor", [["in", 0], ["in", 1]]], ["add.Tensor", [["node", 0], ["in", 2]]],
            ["sub.Tensor", [["node", 1], ["in", 3]]], ["mul.Tensor", [["node", 2], ["in", 4]]],
            ["add.Tensor", [["node", 3], ["in", 5]]]]
    nodes, ops = spec_graph.build(spec, 6)
    prog = compile_group(nodes, ops)
    ins = [x, xt, row, col, mask, idx]
    for od in ("float32", "float64", "bfloat16"):
        out = torch.empty(33, 48, device=DEV, dtype=_tdt(od))
        cabi.pointwise(ins, prog.code, prog.imm, out)
        torch.cuda.synchronize()
        want = oracle.eval_group(spec, [t.float().cpu().numpy() for t in ins], (33, 48), od)
        tol = (1e-5, 1e-6) if od != "bfloat16" else (1e-2, 1e-2)
        _assert_close(out, want, *tol)


@pytest.mark.parametrize("shape", [(1,), (7,), (3, 5, 7), (2, 3, 4, 5, 6, 8), (16384, 8192)])
def test_pointwise_shapes(shape):
    x = torch.randn(shape, device=DEV).to(torch.bfloat16)
    y = torch.randn(shape[-1:], device=DEV).to(torch.bfloat16)
    spec = [["sigmoid.default", [["in", 0]]], ["mul.Tensor", [["in", 0], ["node", 0]]],
            ["mul.Tensor", [["node", 1], ["in", 1]]]]
    nodes, ops = spec_graph.build(spec, 2)
    prog = compile_group(nodes, ops)
    out = torch.empty(shape, device=DEV, dtype=torch.bfloat16)
    cabi.pointwise([x, y], prog.code, prog.imm, out)
    torch.cuda.synchronize()
    if x.numel() > 1 << 20:  # full size: property check on a row sample
        sel = slice(0, 64)
        want = oracle.eval_group(spec, [x[sel].float().cpu().numpy(), y.float().cpu().numpy()],
                                 tuple(x[sel].shape), "bfloat16")
        _assert_close(out[sel], want, 1e-2, 1e-2)
        assert torch.isfinite(out).all()
    else:
        want = oracle.eval_group(spec, [x.float().cpu().numpy(), y.float().cpu().numpy()], shape, "bfloat16")
        _assert_close(out, want, 1e-2, 1e-2)


def test_pointwise_empty_is_noop():
    x = torch.empty(0, 5, device=DEV)
    out = torch.empty(0, 5, device=DEV)
    cabi.pointwise([x], [OP["MOV"] * 10], [0.0], out)


# ------------------------------------------------------------- row kernels
@pytest.mark.parametrize("rows,cols", [(16384, 8192), (37, 64), (5, 4096), (3, 200), (8, 32768), (9, 2048),
                                       (6, 1536), (5, 3072), (4, 6144), (1000, 512), (3001, 1024), (2999, 2048)])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("flags", [7, 1])
def test_rms_norm_swiglu(rows, cols, dtype, flags):
    """16-bit rows whose half is a multiple of 8 run the specialised kernel
    (flags 7: every rounding of the 16-bit graph) -- with many rows whose
    half splits into 64, 128 or 256 x 2 vectors, the row-loop kernel that
    loads one row ahead (odd row counts end a loop mid-pair); the others, and
    flag sets it does not implement, the generic one."""
    dt = _tdt(dtype)
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(rows, cols, device=DEV, generator=g).to(dt)
    w = (1 + 0.02 * torch.randn(cols, device=DEV, generator=g)).to(dt)
    out = torch.empty(rows, cols // 2, device=DEV, dtype=dt)
    rstd = torch.empty(rows, device=DEV)
    cabi.rownorm(x, cabi.ROW_RMSNORM_SWIGLU, w, None, 1e-6, flags, out, rstd_out=rstd)
    torch.cuda.synchronize()
    for sel in (slice(0, min(rows, 256)), slice(max(rows - 64, 0), rows)):
        xs = x[sel].float().cpu().numpy()
        want = oracle.rms_norm_swiglu(xs, w.float().cpu().numpy(), 1e-6, flags, dtype, dtype)
        _assert_close(out[sel], want, 1e-2, 1e-2)
        want_rstd = 1.0 / np.sqrt((xs.astype(np.float64) ** 2).mean(-1) + 1e-6)
        _assert_close(rstd[sel], want_rstd, 1e-5, 0)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("cols", [2048, 768, 100, 1536, 3072])
def test_rms_norm(dtype, cols):
    dt = _tdt(dtype)
    x = torch.randn(67, cols, device=DEV).to(dt)
    w = (1 + 0.1 * torch.randn(cols, device=DEV)).to(dt)
    flags = 0 if dtype == "float32" else 1
    out = torch.empty_like(x)
    rstd = torch.empty(67, device=DEV)
    cabi.rownorm(x, cabi.ROW_RMSNORM, w, None, 1e-5, flags, out, rstd_out=rstd)
    torch.cuda.synchronize()
    want = oracle.rms_norm(x.float().cpu().numpy(), w.float().cpu().numpy(), 1e-5, flags, dtype, dtype)
    tol = (1e-5, 1e-5) if dtype == "float32" else (1e-2, 1e-2)
    _assert_close(out, want, *tol)


@pytest.mark.parametrize("rows,cols", [(64 * 197, 768), (64 * 197 + 1, 768), (10, 1024), (3, 50), (17, 520),
                                       (1, 768), (5, 16384), (7, 1536), (9, 3072)])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_layer_norm(rows, cols, dtype):
    """Full-size, odd and ragged row counts; the check covers the first and
    the last rows."""
    dt = _tdt(dtype)
    x = torch.randn(rows, cols, device=DEV).to(dt)
    w = torch.randn(cols, device=DEV).to(dt)
    b = torch.randn(cols, device=DEV).to(dt)
    out = torch.empty_like(x)
    mean = torch.empty(rows, device=DEV)
    rstd = torch.empty(rows, device=DEV)
    cabi.rownorm(x, cabi.ROW_LAYERNORM, w, b, 1e-6, 0, out, mean_out=mean, rstd_out=rstd)
    torch.cuda.synchronize()
    for sel in (slice(0, 500), slice(max(0, rows - 300), rows)):
        o, m, r = oracle.layer_norm(x[sel].float().cpu().numpy(), w.float().cpu().numpy(),
                                    b.float().cpu().numpy(), 1e-6, dtype)
        _assert_close(out[sel], o, 1e-2, 2e-2)
        _assert_close(mean[sel], m[:, 0], 1e-5, 1e-5)
        _assert_close(rstd[sel], r[:, 0], 1e-4, 1e-5)


@pytest.mark.parametrize("rows,cols", [(32768, 4096), (7, 1000), (3, 33), (2, 32768), (6, 8192), (5, 2048),
                                       (5, 768), (3, 1536), (4, 3072)])
@pytest.mark.parametrize("log", [False, True])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_softmax(rows, cols, log, dtype):
    g = torch.Generator(device=DEV).manual_seed(0)
    x = (2 * torch.randn(rows, cols, device=DEV, generator=g)).to(_tdt(dtype))
    x[0, : min(cols, 5)] = -float("inf")  # masked entries
    out = torch.empty_like(x)
    cabi.softmax(x, out, log=log)
    torch.cuda.synchronize()
    sel = slice(0, 128)
    fn = oracle.log_softmax if log else oracle.softmax
    want = fn(x[sel].float().cpu().numpy(), dtype)
    _assert_close(out[sel], want, 1e-2, 1e-2 if log else 1e-4)
    if not log:  # every row sums to one
        s = out.float().sum(-1)
        assert torch.allclose(s, torch.ones_like(s), atol=2e-2)


def test_gemm_rejects_form_that_contradicts_program():
    x = torch.randn(64, 64, device=DEV).to(torch.bfloat16)
    w = torch.randn(64, 64, device=DEV).to(torch.bfloat16)
    b = torch.randn(64, device=DEV).to(torch.bfloat16)
    code, imm, spec, form = epilogue_program("gelu", residual=False)
    out = torch.empty(64, 64, device=DEV, dtype=torch.bfloat16)
    bad = list(form)
    bad[2] = 3  # claims SiLU
    with pytest.raises(cabi.CError) as e:
        cabi.gemm_epilogue(x, w.t(), [b], code, imm, out, form=bad)
    assert e.value.code == 7


# ------------------------------------------------------------- rotary embedding
def _rope_eager(x, c, s):
    x1, x2 = x.chunk(2, dim=-1)
    return x * c + torch.cat((-x2, x1), dim=-1) * s


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("case", ["llama_q", "llama_k", "hf_bcast", "d128", "unaligned", "odd_half"])
def test_rope_matches_eager_bit_for_bit(dtype, case):
    """b200k_rope against eager PyTorch's decomposed rotate-half graph on the
    same inputs: products and sum round to the 16-bit type in both, so the
    results are equal bit for bit -- on the 8-wide path (transposed q / k
    views with a [S, D] table, [B, 1, S, D] tables, D = 128) and on the
    element-wise path (a view one element off 16-byte alignment, D / 2 not a
    multiple of 8)."""
    dt = _tdt(dtype)
    g = torch.Generator(device=DEV).manual_seed(7)
    B, S = 2, 256
    if case in ("llama_q", "llama_k"):
        H = 32 if case == "llama_q" else 8
        x = torch.randn(B, S, H, 64, device=DEV, generator=g).to(dt).transpose(1, 2)
        c, s = (torch.randn(S, 64, device=DEV, generator=g).to(dt) for _ in range(2))
    elif case == "hf_bcast":
        x = torch.randn(B, 4, S, 64, device=DEV, generator=g).to(dt)
        c, s = (torch.randn(B, 1, S, 64, device=DEV, generator=g).to(dt) for _ in range(2))
    elif case == "d128":
        x = torch.randn(B, 4, S, 128, device=DEV, generator=g).to(dt)
        c, s = (torch.randn(S, 128, device=DEV, generator=g).to(dt) for _ in range(2))
    elif case == "unaligned":
        base = torch.randn(B * 4 * S * 64 + 1, device=DEV, generator=g).to(dt)
        x = base[1:].view(B, 4, S, 64)
        c, s = (torch.randn(S, 64, device=DEV, generator=g).to(dt) for _ in range(2))
    else:
        x = torch.randn(B, 4, S, 20, device=DEV, generator=g).to(dt)
        c, s = (torch.randn(S, 20, device=DEV, generator=g).to(dt) for _ in range(2))
    want = _rope_eager(x, c, s)
    out = torch.empty_strided(want.shape, want.stride(), device=DEV, dtype=dt)
    cabi.rope(x, c, s, out)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    ref = oracle.rope(x.float().cpu().numpy(), c.float().cpu().numpy(), s.float().cpu().numpy(), dtype)
    np.testing.assert_array_equal(out.float().cpu().numpy(), ref)
    # and through the torch op with the decomposed graph's layout
    got = torch.ops.b200.rope(x, c, s, list(want.stride()))
    assert got.stride() == want.stride() and torch.equal(got, want)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("B,S,H,K", [(2, 128, 4, 256), (3, 300, 8, 512), (8, 256, 32, 2048), (1, 2048, 8, 2048),
                                     (8, 2048, 32, 2048)])
@pytest.mark.parametrize("config", [-1, 0, 1, 3])
def test_gemm_rope_equals_gemm_then_rope(dtype, B, S, H, K, config):
    """The rotary epilogue (b200k_gemm_rope) against the same GEMM stored
    plainly and rotated by b200k_rope: bit-identical (the same accumulators
    round to the same 16-bit q, and both rotations round each product and the
    sum as eager PyTorch does); against eager PyTorch on the fp32 product
    within one rounding; rows past a multiple of the period, partial tiles
    (S = 300) and a padded table stride."""
    dt = _tdt(dtype)
    g = torch.Generator(device=DEV).manual_seed(B * 1000 + S + H)
    N = H * 64
    x = (0.5 * torch.randn(B * S, K, device=DEV, generator=g)).to(dt)
    w = (0.05 * torch.randn(N, K, device=DEV, generator=g)).to(dt)
    tab = torch.randn(2, S, 72, device=DEV, generator=g).to(dt)  # row stride 72 elements
    cos, sin = tab[0, :, :64], tab[1, :, :64]
    out = torch.empty(B * S, N, device=DEV, dtype=dt)
    cabi.gemm_rope(x, w.t(), cos, sin, out, tile_config=config)
    plain = torch.empty_like(out)
    base_cfg = {3: 0, -1: cabi.library().b200k_gemm_pick_config(B * S, N, K)}.get(config, config)
    base_cfg = {2: 0, 3: 0, 4: 0}.get(base_cfg, base_cfg)  # the same accumulators on one-CTA tiles
    cabi.gemm_epilogue(x, w.t(), [], [], [], plain, tile_config=base_cfg)
    q = plain.view(B, S, H, 64).transpose(1, 2)
    want = torch.empty_strided(q.shape, q.stride(), device=DEV, dtype=dt)
    cabi.rope(q, cos, sin, want)
    torch.cuda.synchronize()
    got = out.view(B, S, H, 64).transpose(1, 2)
    assert torch.equal(got, want)
    ref = _rope_eager((x.float() @ w.float().t()).to(dt).view(B, S, H, 64).transpose(1, 2), cos, sin)
    np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(),
                               rtol=2e-2, atol=2e-2 * float(ref.float().abs().max()))
    # the torch op, as the compiled graph calls it
    op = torch.ops.b200.gemm_rope(x, w.t(), cos, sin, S, [B, S, N])
    assert op.shape == (B, S, N)
    if config == -1:  # the op picks the tile config as the C entry does by default
        assert torch.equal(op.view(B * S, N), out)


# ------------------------------------------------------------- failure detection
@pytest.mark.parametrize("config", [0, 3, 4])
def test_gemm_stalled_wait_times_out_and_context_survives(config):
    """A wait that nothing completes (the test hook withholds the first
    tile's accumulator-ready signal) runs out after the 50 ms limit: the
    kernel reports B200K_ERR_TIMEOUT in the status word, drains, frees TMEM
    and returns -- on the one-CTA kernel and on the CTA-pair kernel -- and the
    same context then computes a correct GEMM."""
    M, N, K = 1024, 1024, 2048
    g = torch.Generator(device=DEV).manual_seed(9)
    x = (0.02 * torch.randn(M, K, device=DEV, generator=g)).to(torch.bfloat16)
    w = (0.02 * torch.randn(N, K, device=DEV, generator=g)).to(torch.bfloat16)
    b = (0.01 * torch.randn(N, device=DEV, generator=g)).to(torch.bfloat16)
    r = (0.02 * torch.randn(M, N, device=DEV, generator=g)).to(torch.bfloat16)
    code, imm, spec, form = epilogue_program("gelu", residual=True)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, out, tile_config=config, status=status,
                       timeout_ns=50_000_000, form=form, test_flags=cabi.GEMM_TEST_WITHHOLD_READY)
    torch.cuda.synchronize()
    assert status.item() == 6  # B200K_ERR_TIMEOUT
    status.zero_()
    cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, out, tile_config=config, status=status, form=form)
    torch.cuda.synchronize()
    assert status.item() == 0
    want = oracle.gemm_epilogue(x[:64].float().cpu().numpy(), w.float().cpu().numpy().T, spec,
                                [b.float().cpu().numpy(), r[:64].float().cpu().numpy()], "bfloat16",
                                bias=b.float().cpu().numpy())
    _assert_close(out[:64], want, *_gemm_tol(want))


# ------------------------------------------------------------- TF32
@pytest.mark.parametrize("M,N,K", [(1000, 520, 300), (512, 1024, 2048), (4096, 4096, 1024)])
@pytest.mark.parametrize("case", ["gelu", "silu_residual", "bias_to_bf16"])
@pytest.mark.parametrize("config", [-1, 1])
def test_gemm_tf32(M, N, K, case, config):
    """fp32 operands on the TF32 tensor cores (what the backend emits when
    torch allows TF32): the compiled form (bias + activation, fp32 out), the
    interpreter (fp32 residual; a cast to bf16) and the 128-wide tile, against
    the fp32 oracle.  TF32 rounds each operand to 10 significand bits, so the
    bound is 5e-3 relative to the output's magnitude."""
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    x = torch.randn(M, K, device=DEV, generator=g)
    w = torch.randn(N, K, device=DEV, generator=g) / K ** 0.5
    b = 0.1 * torch.randn(N, device=DEV, generator=g)
    r = torch.randn(M, N, device=DEV, generator=g)
    act, res, out_dt = {"gelu": ("gelu", False, "float32"), "silu_residual": ("silu", True, "float32"),
                        "bias_to_bf16": ("none", False, "bfloat16")}[case]
    code, imm, spec, form = epilogue_program(act, residual=res)
    out = torch.empty(M, N, device=DEV, dtype=_tdt(out_dt))
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    extras = [b, r] if res else [b]
    cabi.gemm_epilogue(x, w.t(), extras, code, imm, out, tile_config=config, status=status, form=form)
    torch.cuda.synchronize()
    assert status.item() == 0
    rows = slice(0, 96)
    want = oracle.gemm_epilogue(x[rows].cpu().numpy(), w.cpu().numpy().T, spec,
                                [b.cpu().numpy()] + ([r[rows].cpu().numpy()] if res else []), out_dt,
                                bias=b.cpu().numpy())
    tol = 5e-3 * float(np.abs(want).max() + 1e-6)
    _assert_close(out[rows], want, 5e-3 if out_dt == "float32" else 1e-2, tol)
