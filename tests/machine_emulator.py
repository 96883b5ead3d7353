"""numpy emulator of the kernels' accumulator machine (include/b200k.h).

Lets CPU tests check a lowered program (compiler/optimization/program.py)
against the oracle without a GPU: the emulator does exactly what
run_program() in csrc/common.cuh does, per element, in fp32.
"""
from __future__ import annotations

import numpy as np

from oracle.bf16 import round_bf16

F32 = np.float32
OPERAND_IMM, OPERAND_NONE, MAX_SLOTS = 8, 9, 8


def _sig(a):
    with np.errstate(over="ignore"):
        return (F32(1) / (F32(1) + np.exp(-a))).astype(F32)


def _erf(a):
    from scipy.special import erf

    return erf(a.astype(np.float64)).astype(F32)


BIN = {
    3: lambda a, x: a + x, 4: lambda a, x: a - x, 5: lambda a, x: x - a, 6: lambda a, x: a * x,
    7: lambda a, x: a / x, 8: lambda a, x: x / a, 9: np.fmax, 10: np.fmin,
}
UN = {
    11: lambda a: -a, 12: np.abs, 13: lambda a: np.fmax(a, F32(0)), 14: np.exp, 15: np.log, 16: np.sqrt,
    17: lambda a: F32(1) / np.sqrt(a), 18: _erf, 19: _sig, 20: lambda a: F32(2) * _sig(F32(2) * a) - F32(1),
    21: round_bf16, 22: lambda a: a.astype(np.float16).astype(F32),
}


def run(code, imm, slots_init: list[np.ndarray]) -> np.ndarray:
    """Run the program; slots_init[i] pre-loads slot i (already broadcast)."""
    shape = np.broadcast_shapes(*[s.shape for s in slots_init])
    r = [np.broadcast_to(s.astype(F32), shape).copy() for s in slots_init]
    r += [np.zeros(shape, F32) for _ in range(MAX_SLOTS - len(r))]
    acc = r[0].copy()
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        for c, v in zip(code, imm):
            op, operand = divmod(int(c), 10)
            x = None
            if operand < MAX_SLOTS:
                x = r[operand]
            elif operand == OPERAND_IMM:
                x = F32(v)
            if op == 0:
                continue
            if op == 1:
                acc = np.broadcast_to(x, shape).astype(F32).copy()
            elif op == 2:
                r[operand] = acc.copy()
            elif op in BIN:
                acc = np.asarray(BIN[op](acc, x), dtype=F32)
            elif op in UN:
                acc = np.asarray(UN[op](acc), dtype=F32)
            else:
                raise ValueError(f"bad opcode {c}")
    return acc
