"""CUDA-graph replay of compiled inference graphs (an extension: the
reference runs every compiled graph op by op from Python).

A compiled forward graph of a model issues one kernel launch per fused group
and per remaining ATen op: 195 launches for the Llama-style prefill, 90 for
ViT-B/16.  Run op by op, the host side of those calls leaves the GPU idle
between kernels (the Llama prefill: 31.4 ms of kernels in a 36.2 ms forward).
``GraphReplay`` records the graph's launches once into a CUDA graph and
replays it, so one host call issues all of them.

Semantics are those of the op-by-op function:
  * inputs: tensors that are the same storage at every call (parameters,
    module buffers) are read in place; every other tensor input is copied
    into the graph's own input buffer before each replay;
  * outputs: each replay's outputs are cloned out of the graph's buffers, so
    a result stays valid after later calls;
  * the first call runs op by op (it also warms up lazily initialised
    libraries); the second records the graph; any failure to record, and any
    call whose inputs no longer match the recording (another device, shape,
    dtype or stride, or a moved parameter), runs op by op instead.
The graph's intermediate buffers stay allocated (in a private memory pool)
for the life of the compiled function.  Only inference graphs with at least
``config.GRAPH_MIN_LAUNCHES`` launching nodes and CUDA inputs take this path;
training graphs, whose forward outputs are saved for the backward pass, do
not.  Outputs above ``config.GRAPH_MAX_OUTPUT_MB`` are not cloned out of a
graph: cloning them costs more than replay saves (measured on B200: ViT-B/16,
90 launches and a [64, 1000] output, 3.142 -> 2.998 ms per forward; the
Llama-style prefill, 195 launches of mostly long GEMMs and a 4.2 GB logits
output, 37.17 -> 38.36 ms with the logits cloned).  Such a graph is split
(``split_large_outputs``): the launching nodes that produce the large outputs,
with the views around them, form a tail that runs op by op into fresh
tensors, and the rest of the graph -- the body -- is replayed.  The body's
values that only the tail reads are handed over without a copy: the tail's
launches follow the replay on the same stream, before any later replay can
overwrite them.
"""
from __future__ import annotations

import torch
import torch.fx as fx

from compiler.optimization import config

aten = torch.ops.aten

# Replays issued by every GraphReplay of this process (a diagnostic count).
REPLAYS = 0

# Nodes that never launch a kernel (views, metadata, Python-level getitem).
_NO_LAUNCH = {
    aten.view.default, aten._unsafe_view.default, aten.reshape.default, aten.t.default, aten.transpose.int,
    aten.permute.default, aten.expand.default, aten.unsqueeze.default, aten.squeeze.dim, aten.squeeze.default,
    aten.slice.Tensor, aten.select.int, aten.split.Tensor, aten.split_with_sizes.default, aten.unbind.int,
    aten.alias.default, aten.detach.default, aten.as_strided.default, aten.sym_size.int, aten.sym_stride.int,
}


def launching_nodes(gm: fx.GraphModule) -> int:
    """Number of call_function nodes that launch work on the GPU."""
    n = 0
    for node in gm.graph.nodes:
        if node.op != "call_function" or node.target in _NO_LAUNCH:
            continue
        if getattr(node.target, "__name__", "") == "getitem":
            continue
        n += 1
    return n


def _is_persistent(t: torch.Tensor) -> bool:
    """A parameter or a leaf that requires grad: the same storage every call."""
    return isinstance(t, torch.nn.Parameter) or (t.requires_grad and t.is_leaf)


class GraphReplay:
    """Boxed callable: ``run(args)`` with ``args`` the graph's input list."""

    def __init__(self, fn, no_clone=(), static=()):
        # AOTAutograd's marker for the list-argument calling convention (an
        # instance attribute, so that functools.wraps wrappers copy it)
        self._boxed_call = True
        self.fn = fn  # boxed op-by-op function of the compiled graph
        self.no_clone = frozenset(no_clone)  # output indices returned as the graph's own buffers
        # input indices AOTAutograd marks static (the module's lifted parameters
        # and buffers): read in place like parameters, guarded by their address
        self.static = frozenset(static)
        self.calls = 0
        self.replays = 0
        self.graph = None
        self.disabled = False
        self.static_in = None
        self.persistent = None
        self.sig = None
        self.static_out = None
        self.ptrs = None

    @staticmethod
    def _signature(args):
        return [(a.device, a.dtype, tuple(a.shape), tuple(a.stride())) if isinstance(a, torch.Tensor) else a
                for a in args]

    def _eligible(self, args) -> bool:
        tensors = [a for a in args if isinstance(a, torch.Tensor)]
        if not tensors or not all(t.is_cuda for t in tensors):
            return False
        dev = tensors[0].device
        return all(t.device == dev for t in tensors) and all(
            isinstance(a, (torch.Tensor, int, float, bool, type(None))) for a in args)

    def _record(self, args):
        self.persistent = [isinstance(a, torch.Tensor) and (i in self.static or _is_persistent(a))
                           for i, a in enumerate(args)]
        self.static_in = [a if (not isinstance(a, torch.Tensor) or p) else a.clone()
                          for a, p in zip(args, self.persistent)]
        self.sig = self._signature(args)
        self.ptrs = [a.data_ptr() if p else None for a, p in zip(args, self.persistent)]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.fn(list(self.static_in))  # warm-up on the side stream, as graph capture requires
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            outs = self.fn(list(self.static_in))
        outs = list(outs) if isinstance(outs, (list, tuple)) else [outs]
        storages = {a.untyped_storage().data_ptr() for a in self.static_in if isinstance(a, torch.Tensor)}
        if any(isinstance(o, torch.Tensor) and o.untyped_storage().data_ptr() in storages for o in outs):
            raise RuntimeError("an output aliases an input")
        out_bytes = sum(o.numel() * o.element_size() for i, o in enumerate(outs)
                        if isinstance(o, torch.Tensor) and i not in self.no_clone)
        if out_bytes > config.GRAPH_MAX_OUTPUT_MB * 2**20:
            raise RuntimeError("outputs too large to clone per call")
        self.graph, self.static_out = graph, outs

    def _matches(self, args) -> bool:
        if self._signature(args) != self.sig:
            return False
        return all(p is None or a.data_ptr() == p for a, p in zip(args, self.ptrs))

    def __call__(self, args):
        self.calls += 1
        if self.disabled or not self._eligible(args):
            return self.fn(args)
        if self.graph is None:
            if self.calls == 1:
                return self.fn(args)  # op by op: warms up lazily initialised libraries
            try:
                self._record(args)
            except Exception:  # recording is an optimisation: fall back for good
                self.disabled = True
                self.graph = None
                return self.fn(args)
        if not self._matches(args):
            return self.fn(args)
        for a, s, p in zip(args, self.static_in, self.persistent):
            if isinstance(a, torch.Tensor) and not p and a.data_ptr() != s.data_ptr():
                s.copy_(a)
        self.graph.replay()
        self.replays += 1
        global REPLAYS
        REPLAYS += 1
        return [o.clone() if isinstance(o, torch.Tensor) and i not in self.no_clone else o
                for i, o in enumerate(self.static_out)]


def output_bytes(gm: fx.GraphModule) -> int:
    """Bytes of the graph's tensor outputs, from the traced metadata."""
    total = 0
    for node in gm.graph.nodes:
        if node.op != "output":
            continue
        outs = node.args[0] if isinstance(node.args[0], (list, tuple)) else [node.args[0]]
        for o in outs:
            v = o.meta.get("val") if isinstance(o, fx.Node) else None
            if isinstance(v, torch.Tensor):
                total += v.numel() * v.element_size()
    return total


def _node_bytes(n) -> int:
    v = n.meta.get("val") if isinstance(n, fx.Node) else None
    return v.numel() * v.element_size() if isinstance(v, torch.Tensor) else 0


def _launches(n: fx.Node) -> bool:
    return (n.op == "call_function" and n.target not in _NO_LAUNCH
            and getattr(n.target, "__name__", "") != "getitem")


class TailReplay:
    """Boxed callable of a split graph: the body replayed (GraphReplay), then
    the tail op by op on the body's values and the graph's inputs."""

    def __init__(self, body: GraphReplay, tail_gm: fx.GraphModule, n_body_outs: int, plan, tail_args):
        self._boxed_call = True  # as GraphReplay's
        self.body = body
        self.tail_gm = tail_gm
        self.n_body_outs = n_body_outs  # body outputs that are graph outputs
        self.plan = plan  # per graph output: ("body", i), ("tail", i) or ("const", value)
        self.tail_args = tail_args  # per tail input: ("body", i) or ("arg", i)

    def __call__(self, args):
        b = self.body(args)
        t_in = [b[i] if kind == "body" else args[i] for kind, i in self.tail_args]
        t = self.tail_gm(*t_in)
        out = []
        for kind, v in self.plan:
            out.append(b[v] if kind == "body" else t[v] if kind == "tail" else v)
        return out


def split_large_outputs(gm: fx.GraphModule, static=()):
    """A TailReplay of `gm` whose tail computes the outputs larger than
    ``config.GRAPH_MAX_OUTPUT_MB``, or None when the graph does not split
    cleanly (a large output that is an input, a tail value that the body also
    reads, or too few launches left in the body)."""
    limit = config.GRAPH_MAX_OUTPUT_MB * 2**20
    out_node = next(n for n in gm.graph.nodes if n.op == "output")
    outs = out_node.args[0]
    outs = list(outs) if isinstance(outs, (list, tuple)) else [outs]
    big = [o for o in outs if isinstance(o, fx.Node) and _node_bytes(o) > limit]
    if not big or any(o.op != "call_function" for o in big):
        return None
    # The tail: each large output's producer chain back to (and including) its
    # first launching node, plus every view feeding a tail node.
    tail, stack = set(), [(o, False) for o in big]
    while stack:
        n, past_launch = stack.pop()
        if n in tail or n.op != "call_function":
            continue
        if past_launch and _launches(n):
            continue  # a launching input of the producer stays in the body
        tail.add(n)
        for a in n.all_input_nodes:
            stack.append((a, past_launch or _launches(n)))
    for n in tail:
        if any(u not in tail and u is not out_node for u in n.users):
            return None
    if not any(_launches(n) for n in tail):
        return None
    order = [n for n in gm.graph.nodes if n in tail]
    ext = []
    for n in order:
        for a in n.all_input_nodes:
            if a not in tail and a not in ext:
                ext.append(a)

    # Body: every node outside the tail; outputs = the graph's other outputs,
    # then the tail's inputs that the body computes.
    body_g = fx.Graph()
    env = {}
    placeholders = []
    for n in gm.graph.nodes:
        if n.op == "output" or n in tail:
            continue
        env[n] = body_g.node_copy(n, lambda a: env[a])
        if n.op == "placeholder":
            placeholders.append(n)
    small = [o for o in outs if isinstance(o, fx.Node) and o not in tail]
    ext_body = [a for a in ext if a.op != "placeholder"]
    if any(o.op == "placeholder" for o in small):
        return None  # an input returned as an output: the replay would alias it
    body_g.output(tuple(env[o] for o in small) + tuple(env[a] for a in ext_body))
    body_gm = fx.GraphModule(gm, body_g)
    if launching_nodes(body_gm) < config.GRAPH_MIN_LAUNCHES:
        return None

    # Tail: placeholders for its inputs, then its nodes in graph order.
    tail_g = fx.Graph()
    tenv = {a: tail_g.placeholder(f"t_in{i}") for i, a in enumerate(ext)}
    for a, ph in tenv.items():
        ph.meta = dict(a.meta)
    for n in order:
        tenv[n] = tail_g.node_copy(n, lambda a: tenv[a])
    tail_outs = [o for o in outs if isinstance(o, fx.Node) and o in tail]
    tail_g.output(tuple(tenv[o] for o in tail_outs))
    tail_gm = fx.GraphModule(gm, tail_g)

    plan = []
    for o in outs:
        if isinstance(o, fx.Node) and o in tail:
            plan.append(("tail", tail_outs.index(o)))
        elif isinstance(o, fx.Node):
            plan.append(("body", small.index(o)))
        else:
            plan.append(("const", o))
    tail_args = [("arg", placeholders.index(a)) if a.op == "placeholder" else ("body", len(small) + ext_body.index(a))
                 for a in ext]
    no_clone = range(len(small), len(small) + len(ext_body))
    body = GraphReplay(lambda a: body_gm(*a), no_clone=no_clone, static=static)
    return TailReplay(body, tail_gm, len(small), plan, tail_args)


def wrap(gm: fx.GraphModule, boxed_fn, static=()):
    """The boxed function of an inference graph, replayed as a CUDA graph when
    it launches enough kernels to gain from it: whole when its outputs are
    small enough to clone per call, else split into a replayed body and a
    tail run op by op (``split_large_outputs``); otherwise `boxed_fn`.
    `static`: input indices read in place instead of copied per replay."""
    if not config.CUDA_GRAPHS or launching_nodes(gm) < config.GRAPH_MIN_LAUNCHES:
        return boxed_fn
    if output_bytes(gm) <= config.GRAPH_MAX_OUTPUT_MB * 2**20:
        return GraphReplay(boxed_fn, static=static)
    split = split_large_outputs(gm, static)
    return split if split is not None else boxed_fn
