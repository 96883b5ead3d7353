"""Lowering of a fused FX group to the kernel library's epilogue program.

The reference turns each group into Triton source, one SSA line per node
(compiler/optimization/fusion_pointwise.py:116-129, emit_pointwise_ops), and
JIT-compiles it.  Here a group becomes a short program for an accumulator
machine (include/b200k.h documents the instruction set), passed to the
kernel library as data.  The library either interprets it per element (the
GEMM epilogues outside the compiled canonical forms, and pointwise launches
outside the generated kernels' scope) or writes it out as straight-line CUDA
C and compiles that for sm_100a with NVRTC on first use
(csrc/pointwise_jit.cu), once per program and operand layout.

Machine model: one accumulator, ``MAX_SLOTS`` value slots.  Operands (the
group's external inputs, or for a GEMM epilogue the accumulator and the extra
tensors) arrive pre-loaded in slots 0..n-1.  Every binary op reads the
accumulator and a slot or an immediate; values still needed later are spilled
to a free slot before the accumulator is overwritten.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.fx as fx

aten = torch.ops.aten

# Mirror of the enums in include/b200k.h.
MAX_SLOTS = 8
MAX_INSTR = 64
MAX_INPUTS = 8
OPERAND_IMM = 8
OPERAND_NONE = 9

OP = {
    "NOP": 0, "MOV": 1, "STORE": 2, "ADD": 3, "SUB": 4, "RSUB": 5, "MUL": 6, "DIV": 7, "RDIV": 8,
    "MAX": 9, "MIN": 10, "NEG": 11, "ABS": 12, "RELU": 13, "EXP": 14, "LOG": 15, "SQRT": 16,
    "RSQRT": 17, "ERF": 18, "SIGMOID": 19, "TANH": 20, "ROUND_BF16": 21, "ROUND_F16": 22,
}
OP_NAME = {v: k for k, v in OP.items()}

# ATen op -> (machine op, swapped-operand machine op or None, is_unary).
# The set is exactly the reference's POINTWISE_OPS
# (compiler/optimization/fusion_pointwise.py:12-30); _to_copy is an identity
# inside a kernel (the final store rounds to the output dtype).
BINARY = {
    aten.add.Tensor: ("ADD", "ADD"),
    aten.sub.Tensor: ("SUB", "RSUB"),
    aten.mul.Tensor: ("MUL", "MUL"),
    aten.div.Tensor: ("DIV", "RDIV"),
    aten.maximum.default: ("MAX", "MAX"),
    aten.minimum.default: ("MIN", "MIN"),
}
UNARY = {
    aten.neg.default: "NEG",
    aten.abs.default: "ABS",
    aten.relu.default: "RELU",
    aten.exp.default: "EXP",
    aten.log.default: "LOG",
    aten.sqrt.default: "SQRT",
    aten.rsqrt.default: "RSQRT",
    aten.erf.default: "ERF",
    aten.sigmoid.default: "SIGMOID",
    aten.tanh.default: "TANH",
}
CAST = aten._to_copy.default


class ProgramError(ValueError):
    """The group does not fit the machine (too many live values or instructions)."""


@dataclass
class Program:
    code: list[int] = field(default_factory=list)
    imm: list[float] = field(default_factory=list)

    def emit(self, op: str, operand: int = OPERAND_NONE, imm: float = 0.0) -> None:
        if len(self.code) >= MAX_INSTR:
            raise ProgramError(f"program longer than {MAX_INSTR} instructions")
        self.code.append(OP[op] * 10 + operand)
        self.imm.append(float(imm))

    def __len__(self) -> int:
        return len(self.code)

    def listing(self) -> str:
        out = []
        for c, v in zip(self.code, self.imm):
            op, operand = OP_NAME[c // 10], c % 10
            arg = "" if operand == OPERAND_NONE else (f"#{v!r}" if operand == OPERAND_IMM else f"s{operand}")
            out.append(f"{op} {arg}".strip())
        return "; ".join(out)


def round_op_for(dtype: torch.dtype) -> str | None:
    if dtype == torch.bfloat16:
        return "ROUND_BF16"
    if dtype == torch.float16:
        return "ROUND_F16"
    return None


def _schedule(group: list[fx.Node]) -> list[fx.Node]:
    """Re-order a group for few live values: depth-first from the output,
    evaluating the operand with the larger subtree first (Sethi-Ullman
    order), so each value is produced right before it is consumed.  Every op
    is a pure elementwise function, so the order does not change any value."""
    members = set(group)
    size: dict[fx.Node, int] = {}

    def subtree(n: fx.Node) -> int:
        if n in size:
            return size[n]
        size[n] = 1 + sum(subtree(a) for a in n.args if isinstance(a, fx.Node) and a in members)
        return size[n]

    order: list[fx.Node] = []
    seen: set[fx.Node] = set()
    stack: list[tuple[fx.Node, bool]] = [(group[-1], False)]
    while stack:
        n, expanded = stack.pop()
        if n in seen:
            continue
        if expanded:
            seen.add(n)
            order.append(n)
            continue
        stack.append((n, True))
        kids = [a for a in n.args if isinstance(a, fx.Node) and a in members and a not in seen]
        # pushed last = visited first: the biggest subtree goes first
        for a in sorted(kids, key=subtree):
            stack.append((a, False))
    # Members that do not feed the output (impossible for the single-output
    # groups the passes build) are dropped: they cannot change the result.
    return order


def compile_group(
    group: list[fx.Node],
    operands: list[fx.Node],
    prologue: list[tuple[str, fx.Node | float]] | None = None,
    prologue_target: fx.Node | None = None,
    rounding_casts: bool = False,
) -> Program:
    """Lower ``group`` (topologically ordered, last node = output) to a program.

    ``operands[i]`` is pre-loaded in slot i.  ``prologue`` optionally rewrites
    the value of ``prologue_target`` (an operand) before the group runs, e.g.
    the addmm bias add ``acc = acc + bias`` (fusion_epilogue.py:142-143).
    With ``rounding_casts`` a cast to bf16/f16 inside the group emits a
    rounding op (used by fusions that cross sub-fp32 casts); otherwise casts
    are identities as in the reference.
    """
    prog = Program()
    group = _schedule(group)  # ends with the original output node

    # Casts alias their input unless they round.
    alias: dict[fx.Node, fx.Node] = {}

    def canon(n):
        while isinstance(n, fx.Node) and n in alias:
            n = alias[n]
        return n

    rounding: dict[fx.Node, str] = {}
    for node in group:
        if node.target == CAST:
            r = round_op_for(node.kwargs.get("dtype")) if rounding_casts and node is not group[-1] else None
            if r is None:
                alias[node] = node.args[0]
            else:
                rounding[node] = r

    # Last use (index into group) of every canonical value read by the group.
    last_use: dict[fx.Node, int] = {}
    for i, node in enumerate(group):
        if node in alias:
            continue
        for a in node.args:
            if isinstance(a, fx.Node):
                last_use[canon(a)] = i
    root = canon(group[-1])
    last_use[root] = len(group)  # the result is read by the final store

    slot_of: dict[fx.Node, int] = {}
    free = list(range(MAX_SLOTS))
    for i, op in enumerate(operands):
        if i >= MAX_SLOTS:
            raise ProgramError("more operands than slots")
        slot_of[op] = i
        free.remove(i)
    acc: fx.Node | None = None  # value currently in the accumulator

    def release(i: int) -> None:
        # Values whose last reader is node i (or that no node reads) give back their slot.
        for v in list(slot_of):
            if last_use.get(v, -1) <= i:
                free.append(slot_of.pop(v))
        free.sort()

    def spill_acc() -> None:
        nonlocal acc
        if acc is not None and acc not in slot_of and last_use.get(acc, -1) >= cur_index:
            if not free:
                raise ProgramError(f"more than {MAX_SLOTS} live values")
            s = free.pop(0)
            prog.emit("STORE", s)
            slot_of[acc] = s

    def load_acc(v: fx.Node) -> None:
        nonlocal acc
        if acc is v:
            return
        spill_acc()
        if v not in slot_of:
            raise ProgramError(f"value {v} is neither in the accumulator nor in a slot")
        prog.emit("MOV", slot_of[v])
        acc = v

    def operand_of(x) -> tuple[int, float]:
        if isinstance(x, fx.Node):
            v = canon(x)
            if v is acc and v not in slot_of:
                spill_acc()
            if v not in slot_of:
                raise ProgramError(f"value {v} not materialised")
            return slot_of[v], 0.0
        return OPERAND_IMM, float(x)

    cur_index = -1
    if prologue:
        target = prologue_target
        load_acc(target)
        for op, x in prologue:
            s, imm = operand_of(x)
            prog.emit(op, s, imm)
        # The operand's slot now holds a stale value: re-home the rewritten one.
        prog.emit("STORE", slot_of[target])

    for i, node in enumerate(group):
        cur_index = i
        if node in alias:
            continue
        if node in rounding:
            src = canon(node.args[0])
            load_acc(src)
            # `src` stays needed after this node only if it is in a slot.
            if last_use.get(src, -1) > i and src not in slot_of:
                spill_acc()
            prog.emit(rounding[node])
            acc = node
        elif node.target in UNARY:
            src = canon(node.args[0])
            if not isinstance(src, fx.Node):
                raise ProgramError("unary op on a scalar")
            load_acc(src)
            if last_use.get(src, -1) > i and src not in slot_of:
                spill_acc()
            prog.emit(UNARY[node.target])
            acc = node
        elif node.target in BINARY:
            op, swapped = BINARY[node.target]
            a, b = (canon(x) if isinstance(x, fx.Node) else x for x in node.args[:2])
            if isinstance(a, fx.Node) and acc is a:
                left, right, mop = a, b, op
            elif isinstance(b, fx.Node) and acc is b:
                left, right, mop = b, a, swapped
            elif isinstance(a, fx.Node):
                left, right, mop = a, b, op
            elif isinstance(b, fx.Node):
                left, right, mop = b, a, swapped
            else:
                raise ProgramError("binary op on two scalars")
            load_acc(left)
            # Keep `left` if a later node (or this node's right operand) reads it.
            if (last_use.get(left, -1) > i or right is left) and left not in slot_of:
                spill_acc()
            s, imm = operand_of(right)
            prog.emit(mop, s, imm)
            acc = node
        else:
            raise ProgramError(f"unsupported op {node.target}")
        release(i)

    if acc is not root:
        load_acc(root)
    return prog


def group_spec(group: list[fx.Node], operands: list[fx.Node]) -> list[tuple]:
    """A plain-data description of a group (op name, args as ('in', i) /
    ('node', j) / float), used to evaluate the same group in the oracle."""
    index = {n: j for j, n in enumerate(group)}
    opi = {n: i for i, n in enumerate(operands)}
    spec = []
    for node in group:
        args = []
        for a in node.args:
            if isinstance(a, fx.Node):
                args.append(("node", index[a]) if a in index else ("in", opi[a]))
            else:
                args.append(float(a))
        name = str(node.target).replace("aten.", "")
        if node.target == CAST:
            args.append(str(node.kwargs.get("dtype")).replace("torch.", ""))
        spec.append((name, tuple(args)))
    return spec


# ------------------------------------------------------------------ canonical form
# The GEMM kernel has a compiled path for programs of the form
#   v = acc [+ E_bias]; v = act(v); [v = round(v)]; [v *= E_scale]; [v += E_res]
# (include/b200k.h, B200kEpilogueForm).  canonical_form() recognises it by
# executing the program symbolically and comparing expression trees, with
# commutative operands in a fixed order.
ACT_CODES = {"NONE": 0, "GELU_ERF": 1, "GELU_TANH": 2, "SILU": 3, "RELU": 4, "SIGMOID": 5, "TANH": 6}
_DT_BF16, _DT_F16 = 2, 1


def _f32(v: float) -> float:
    import struct

    return struct.unpack("f", struct.pack("f", float(v)))[0]


def _mk(name: str, a, b):
    if name in ("add", "mul", "max", "min"):
        return (name,) + tuple(sorted((a, b), key=repr))
    return (name, a, b)


def _const(v):
    return ("c", _f32(v))


_ACT_TEMPLATES = {
    "NONE": lambda x: x,
    "GELU_ERF": lambda x: _mk("mul", _mk("mul", x, _const(0.5)),
                              _mk("add", ("erf", _mk("mul", x, _const(0.7071067811865476))), _const(1.0))),
    "GELU_TANH": lambda x: _mk("mul", _mk("mul", x, _const(0.5)), _mk("add", ("tanh", _mk(
        "mul", _mk("add", x, _mk("mul", _mk("mul", _mk("mul", x, x), x), _const(0.044715))),
        _const(0.7978845608028654))), _const(1.0))),
    "SILU": lambda x: _mk("mul", x, ("sigmoid", x)),
    "RELU": lambda x: ("relu", x),
    "SIGMOID": lambda x: ("sigmoid", x),
    "TANH": lambda x: ("tanh", x),
}

_SYM_BIN = {"ADD": "add", "SUB": "sub", "MUL": "mul", "DIV": "div", "MAX": "max", "MIN": "min"}


def symbolic(code: list[int], imm: list[float], n_operands: int):
    """Expression tree the program leaves in the accumulator."""
    slots = [("in", i) for i in range(n_operands)] + [("zero",)] * (MAX_SLOTS - n_operands)
    acc = slots[0]
    for c, v in zip(code, imm):
        op, o = divmod(int(c), 10)
        name = OP_NAME[op]
        x = slots[o] if o < MAX_SLOTS else (_const(v) if o == OPERAND_IMM else None)
        if name == "MOV":
            acc = x
        elif name == "STORE":
            slots[o] = acc
        elif name in _SYM_BIN:
            acc = _mk(_SYM_BIN[name], acc, x)
        elif name == "RSUB":
            acc = _mk("sub", x, acc)
        elif name == "RDIV":
            acc = _mk("div", x, acc)
        elif name != "NOP":
            acc = (name.lower(), acc)
    return acc


def canonical_form(prog: Program, n_operands: int, row_vector: list[bool] | None = None) -> list[int] | None:
    """[1, bias, act, round, scale, residual] (extras indices, -1 = absent) when
    the GEMM-epilogue program (slot 0 = accumulator) has the canonical form.

    ``row_vector[i]`` (operand i, slot 0 being the accumulator) says whether
    operand i broadcasts along rows (a [N] or [1, N] vector).  Only such an
    operand can be the bias: without an activation ``acc + x`` reads either
    way, and a full [M, N] matrix belongs in the residual role, whose kernel
    path streams it.  None = no restriction."""
    tree = symbolic(prog.code, prog.imm, n_operands)

    def peel(t, op):
        yield t, -1
        if t[0] == op:
            for inner, leaf in ((t[1], t[2]), (t[2], t[1])):
                if leaf[0] == "in" and 1 <= leaf[1] < n_operands:
                    yield inner, leaf[1]

    for t1, res in peel(tree, "add"):
        for t2, scale in peel(t1, "mul"):
            rounds = [(t2, -1)]
            if t2[0] == "round_bf16":
                rounds.append((t2[1], _DT_BF16))
            if t2[0] == "round_f16":
                rounds.append((t2[1], _DT_F16))
            for t3, rnd in rounds:
                for act, tmpl in _ACT_TEMPLATES.items():
                    for bias in [-1] + [i for i in range(1, n_operands) if row_vector is None or row_vector[i]]:
                        base = ("in", 0) if bias < 0 else _mk("add", ("in", 0), ("in", bias))
                        if tmpl(base) == t3:
                            return [1, bias - 1 if bias > 0 else -1, ACT_CODES[act], rnd,
                                    scale - 1 if scale > 0 else -1, res - 1 if res > 0 else -1]
    return None
