"""CUDA-graph replay of compiled inference graphs (compiler/graph_replay.py):
the decision logic on CPU, and op-by-op equality of replayed results on the
GPU."""
import pytest
import torch
import torch.fx as fx
import torch.nn as nn

from compiler import graph_replay
from compiler.optimization import config

DEV = "cuda"


def _chain(n_ops: int) -> fx.GraphModule:
    """x -> (view, relu) repeated: n_ops launching nodes and n_ops views."""
    g = fx.Graph()
    x = g.placeholder("x")
    for _ in range(n_ops):
        v = g.call_function(torch.ops.aten.view.default, (x, [-1]))
        x = g.call_function(torch.ops.aten.relu.default, (v,))
    g.output((x,))
    return fx.GraphModule(nn.Module(), g)


def test_launching_nodes_skip_views():
    assert graph_replay.launching_nodes(_chain(5)) == 5


def test_wrap_replays_only_graphs_with_enough_launches():
    fn = lambda args: args  # noqa: E731
    assert graph_replay.wrap(_chain(config.GRAPH_MIN_LAUNCHES - 1), fn) is fn
    r = graph_replay.wrap(_chain(config.GRAPH_MIN_LAUNCHES), fn)
    assert isinstance(r, graph_replay.GraphReplay) and r._boxed_call


def test_wrap_leaves_graphs_with_large_outputs_op_by_op():
    fn = lambda args: args  # noqa: E731
    gm = _chain(config.GRAPH_MIN_LAUNCHES)
    out = [n for n in gm.graph.nodes if n.op == "output"][0].args[0][0]
    out.meta["val"] = torch.empty(config.GRAPH_MAX_OUTPUT_MB * 2**20 // 2 + 1, dtype=torch.bfloat16, device="meta")
    assert graph_replay.output_bytes(gm) > config.GRAPH_MAX_OUTPUT_MB * 2**20
    assert graph_replay.wrap(gm, fn) is fn
    out.meta["val"] = torch.empty(64, 1000, dtype=torch.bfloat16, device="meta")
    assert isinstance(graph_replay.wrap(gm, fn), graph_replay.GraphReplay)


def test_cpu_inputs_run_op_by_op():
    calls = []

    def fn(args):
        calls.append(1)
        return [args[0] + 1]

    r = graph_replay.GraphReplay(fn)
    for _ in range(3):
        (y,) = r([torch.ones(3)])
        assert torch.equal(y, torch.full((3,), 2.0))
    assert len(calls) == 3 and r.graph is None and r.replays == 0


class _Blocks(nn.Module):
    """Pre-norm MLP blocks with residuals: well over 16 launches per call."""

    def __init__(self, dim=256, depth=6):
        super().__init__()
        self.norms = nn.ModuleList(nn.LayerNorm(dim) for _ in range(depth))
        self.up = nn.ModuleList(nn.Linear(dim, 4 * dim) for _ in range(depth))
        self.down = nn.ModuleList(nn.Linear(4 * dim, dim) for _ in range(depth))

    def forward(self, x):
        for n, u, d in zip(self.norms, self.up, self.down):
            x = x + d(torch.nn.functional.gelu(u(n(x))))
        return x


@pytest.mark.gpu
def test_replayed_graph_matches_op_by_op_and_outputs_survive_later_calls():
    """Five calls with fresh inputs: the first runs op by op, the second
    records, the rest replay.  Every result equals the op-by-op compiled
    function's on the same input bit for bit, and a result taken earlier is
    not overwritten by later calls (outputs are cloned out of the graph)."""
    from compiler.backend import custom_backend

    torch.manual_seed(0)
    model = _Blocks().to(DEV, torch.bfloat16).eval()
    xs = [torch.randn(512, 256, device=DEV, dtype=torch.bfloat16) for _ in range(5)]
    torch._dynamo.reset()
    before = graph_replay.REPLAYS
    with torch.no_grad():
        f = torch.compile(model, backend=custom_backend)
        outs = [f(x) for x in xs]
        kept = [o.clone() for o in outs]
        f(torch.randn(512, 256, device=DEV, dtype=torch.bfloat16))
    torch.cuda.synchronize()
    assert graph_replay.REPLAYS - before >= 4  # calls 2-5 and the extra call
    for o, k in zip(outs, kept):
        assert torch.equal(o, k)
    old = config.CUDA_GRAPHS
    try:
        config.CUDA_GRAPHS = False
        torch._dynamo.reset()
        with torch.no_grad():
            g = torch.compile(model, backend=custom_backend)
            want = [g(x) for x in xs]
    finally:
        config.CUDA_GRAPHS = old
        torch._dynamo.reset()
    for o, w in zip(outs, want):
        assert torch.equal(o, w)


@pytest.mark.gpu
def test_replay_reads_parameters_in_place():
    """A parameter changed in place between calls is seen by the replay (the
    graph reads parameters from their own storage)."""
    from compiler.backend import custom_backend

    torch.manual_seed(1)
    model = _Blocks(depth=4).to(DEV, torch.bfloat16).eval()
    x = torch.randn(256, 256, device=DEV, dtype=torch.bfloat16)
    torch._dynamo.reset()
    with torch.no_grad():
        f = torch.compile(model, backend=custom_backend)
        for _ in range(3):
            f(x)
        model.down[0].bias.add_(1.0)
        got = f(x)
        want = model(x)
    torch._dynamo.reset()
    torch.testing.assert_close(got.float(), want.float(), rtol=5e-2, atol=5e-2)


def _chain_with_head(n_ops: int, big: bool) -> fx.GraphModule:
    """x -> relu repeated n_ops times -> mm(view(x), t(w)) -> view: the head's
    output is marked larger than the clone limit when `big`."""
    g = fx.Graph()
    x = g.placeholder("x")
    w = g.placeholder("w")
    for _ in range(n_ops):
        x = g.call_function(torch.ops.aten.relu.default, (x,))
    v = g.call_function(torch.ops.aten.view.default, (x, [-1, 8]))
    wt = g.call_function(torch.ops.aten.t.default, (w,))
    mm = g.call_function(torch.ops.aten.mm.default, (v, wt))
    out = g.call_function(torch.ops.aten.view.default, (mm, [2, -1, 16]))
    small = g.call_function(torch.ops.aten.neg.default, (x,))
    n = config.GRAPH_MAX_OUTPUT_MB * 2**20 // 2 + 1 if big else 16
    out.meta["val"] = torch.empty(n, dtype=torch.bfloat16, device="meta")
    small.meta["val"] = torch.empty(16, dtype=torch.bfloat16, device="meta")
    g.output((out, small))
    return fx.GraphModule(nn.Module(), g)


def test_large_outputs_split_into_replayed_body_and_eager_tail():
    """The head (mm with its views) forms the tail; the relus stay in the
    replayed body; the tail's inputs are the body's last relu (handed over
    without a clone) and the weight argument."""
    gm = _chain_with_head(config.GRAPH_MIN_LAUNCHES, big=True)
    r = graph_replay.wrap(gm, lambda args: args)
    assert isinstance(r, graph_replay.TailReplay) and r._boxed_call
    tail_targets = [n.target for n in r.tail_gm.graph.nodes if n.op == "call_function"]
    assert sorted(map(str, tail_targets)) == sorted(["aten.view.default", "aten.t.default", "aten.mm.default",
                                                     "aten.view.default"])
    assert r.tail_args == [("body", 1), ("arg", 1)]
    assert r.plan == [("tail", 0), ("body", 0)]
    assert r.body.no_clone == frozenset({1})
    # On CPU tensors the body runs op by op; the results equal the graph's.
    x, w = torch.randn(4, 8), torch.randn(16, 8)
    got = r([x, w])
    want = gm(x, w)
    assert len(got) == 2 and all(torch.equal(a, b) for a, b in zip(got, want))


def test_small_outputs_replay_whole_and_unsplittable_graphs_run_op_by_op():
    gm = _chain_with_head(config.GRAPH_MIN_LAUNCHES, big=False)
    assert isinstance(graph_replay.wrap(gm, lambda a: a), graph_replay.GraphReplay)
    # too few launches left in the body once the head is split off
    gm = _chain_with_head(config.GRAPH_MIN_LAUNCHES - 2, big=True)
    fn = lambda a: a  # noqa: E731
    assert graph_replay.wrap(gm, fn) is fn
    # the head's input also feeds another output: the tail would be read by the body
    gm = _chain_with_head(config.GRAPH_MIN_LAUNCHES, big=True)
    mm = next(n for n in gm.graph.nodes if n.target == torch.ops.aten.mm.default)
    out = next(n for n in gm.graph.nodes if n.op == "output")
    with gm.graph.inserting_before(out):
        extra = gm.graph.call_function(torch.ops.aten.relu.default, (mm,))
    out.args = ((out.args[0][0], out.args[0][1], extra),)
    gm.recompile()
    assert graph_replay.wrap(gm, fn) is fn


class _BlocksWithHead(_Blocks):
    def __init__(self, dim=256, depth=6, vocab=4096):
        super().__init__(dim, depth)
        self.head = nn.Linear(dim, vocab, bias=False)

    def forward(self, x):
        return self.head(super().forward(x))


@pytest.mark.gpu
def test_split_replay_matches_op_by_op_and_outputs_survive_later_calls(monkeypatch):
    """A model whose output is above the clone limit (lowered to 1 MiB here):
    the body replays, the head runs op by op into fresh tensors, results equal
    the op-by-op compiled function's bit for bit and stay valid after later
    calls."""
    from compiler.backend import custom_backend

    monkeypatch.setattr(config, "GRAPH_MAX_OUTPUT_MB", 1)
    torch.manual_seed(2)
    model = _BlocksWithHead().to(DEV, torch.bfloat16).eval()
    xs = [torch.randn(512, 256, device=DEV, dtype=torch.bfloat16) for _ in range(4)]
    torch._dynamo.reset()
    before = graph_replay.REPLAYS
    with torch.no_grad():
        f = torch.compile(model, backend=custom_backend)
        outs = [f(x) for x in xs]
        kept = [o.clone() for o in outs]
        f(torch.randn(512, 256, device=DEV, dtype=torch.bfloat16))
    torch.cuda.synchronize()
    assert graph_replay.REPLAYS - before >= 3
    assert all(o.shape == (512, 4096) for o in outs)
    assert len({o.data_ptr() for o in outs}) == len(outs)  # fresh output tensors
    for o, k in zip(outs, kept):
        assert torch.equal(o, k)
    monkeypatch.setattr(config, "CUDA_GRAPHS", False)
    torch._dynamo.reset()
    with torch.no_grad():
        g = torch.compile(model, backend=custom_backend)
        want = [g(x) for x in xs]
    torch._dynamo.reset()
    for o, w in zip(outs, want):
        assert torch.equal(o, w)


def test_boxed_marker_survives_wrapping():
    """AOTAutograd reaches a backward graph's callable through a
    functools.wraps wrapper (torch._dynamo.disable); the list-argument marker
    has to survive it, or the backward call passes unpacked arguments."""
    from compiler.backend import StatusChecked

    for obj in (StatusChecked(lambda a: a, 0), graph_replay.GraphReplay(lambda a: a)):
        assert getattr(torch._dynamo.disable(obj), "_boxed_call", False)


class _BlocksWithBuffer(_Blocks):
    """_Blocks with a per-channel scale held as a module buffer."""

    def __init__(self, dim=256, depth=6):
        super().__init__(dim, depth)
        self.register_buffer("scale", torch.ones(dim))

    def forward(self, x):
        return super().forward(x) * self.scale


def test_static_input_indices_reach_the_inference_compiler():
    """Inside a dynamo compile the backend sees which graph inputs are the
    module's lifted parameters and buffers (AOTAutograd's static inputs)."""
    from torch._dynamo.backends.common import aot_autograd
    from torch._functorch.aot_autograd import make_boxed_func

    from compiler import backend as B

    seen = []

    def fw(gm, example_inputs):
        seen.append((B._static_inputs(), len(example_inputs)))
        return make_boxed_func(gm.forward)

    model = _BlocksWithBuffer(dim=16, depth=1).eval()
    torch._dynamo.reset()
    with torch.no_grad():
        torch.compile(model, backend=aot_autograd(fw_compiler=fw))(torch.randn(4, 16))
    torch._dynamo.reset()
    (static, n), = seen
    assert len(static) == n - 1  # every input but x: 6 parameters and the buffer
    assert B._static_inputs() == ()  # outside a compile


@pytest.mark.gpu
def test_replay_reads_buffers_in_place(monkeypatch):
    """A module buffer is read from its own storage by the replay (not copied
    into the graph per call): every input but x is recorded as read in
    place, and an in-place change between calls is seen."""
    from compiler.backend import custom_backend

    recorded = []
    orig = graph_replay.GraphReplay._record

    def record(self, args):
        orig(self, args)
        recorded.append((self, len(args)))

    monkeypatch.setattr(graph_replay.GraphReplay, "_record", record)
    torch.manual_seed(2)
    model = _BlocksWithBuffer().to(DEV, torch.bfloat16).eval()
    x = torch.randn(256, 256, device=DEV, dtype=torch.bfloat16)
    torch._dynamo.reset()
    before = graph_replay.REPLAYS
    with torch.no_grad():
        f = torch.compile(model, backend=custom_backend)
        for _ in range(3):
            f(x)
        model.scale.mul_(2.0)
        got = f(x)
        want = model(x)
    torch._dynamo.reset()
    assert graph_replay.REPLAYS - before >= 2
    (r, n), = recorded
    assert sum(r.persistent) == n - 1 and not r.persistent[[i for i in range(n) if i not in r.static][0]]
    torch.testing.assert_close(got.float(), want.float(), rtol=5e-2, atol=5e-2)
