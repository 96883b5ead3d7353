"""CPU checks of the pointwise kernel generator (csrc/pointwise_jit.cu): the
kernel it writes for every accumulator-machine instruction, every operand
dtype and broadcast kind, at merged rank 1 and 2, compiles for sm_100a with
NVRTC (no GPU needed), and launches outside its scope are refused."""
import pytest

from compiler import runtime
from compiler.optimization.program import OP
from compiler.runtime import cabi

IMM, NONE = 8, 9
BINARY = ["ADD", "SUB", "RSUB", "MUL", "DIV", "RDIV", "MAX", "MIN"]
UNARY = ["NEG", "ABS", "RELU", "EXP", "LOG", "SQRT", "RSQRT", "ERF", "SIGMOID", "TANH", "ROUND_BF16", "ROUND_F16"]


def every_instruction_program(n_in: int):
    """STORE to a temporary slot, each binary op on an input, an immediate and
    the temporary, every unary op, MOV from a slot and from an immediate."""
    tmp = n_in
    code, imm = [OP["STORE"] * 10 + tmp], [0.0]
    for name in BINARY:
        code += [OP[name] * 10 + (n_in - 1), OP[name] * 10 + IMM, OP[name] * 10 + tmp]
        imm += [0.0, 1.5, 0.0]
    for name in UNARY:
        code.append(OP[name] * 10 + NONE)
        imm.append(0.0)
    code += [OP["STORE"] * 10 + 0, OP["MOV"] * 10 + IMM, OP["ADD"] * 10 + 0, OP["NOP"] * 10 + NONE]
    imm += [0.0, -0.25, 0.0, 0.0]
    return code, imm


@pytest.fixture(scope="module", autouse=True)
def _lib():
    runtime.load()
    cabi.library()


@pytest.mark.parametrize("rank", [1, 2])
@pytest.mark.parametrize("dtypes,unit,out", [
    ([cabi.BF16, cabi.BF16], [1, 1], cabi.BF16),
    ([cabi.F32], [1], cabi.F32),
    ([cabi.F16, cabi.F32, cabi.BF16, cabi.F32], [1, 0, 1, 1], cabi.F16),
    ([cabi.F32, cabi.F32, cabi.BF16], [1, 1, 0], cabi.F32),
])
def test_generated_kernel_compiles(rank, dtypes, unit, out):
    code, imm = every_instruction_program(len(dtypes))
    rc, log = cabi.pointwise_jit_compile(rank, dtypes, unit, out, code, imm)
    assert rc == 0, log


def test_out_of_scope_requests_are_refused():
    code, imm = [OP["ADD"] * 10 + 1], [0.0]
    assert cabi.pointwise_jit_compile(3, [cabi.F32] * 2, [1, 1], cabi.F32, code, imm)[0] == 4  # rank 3
    assert cabi.pointwise_jit_compile(1, [cabi.F32] * 5, [1] * 5, cabi.F32, code, imm)[0] == 4  # 5 inputs
    assert cabi.pointwise_jit_compile(1, [cabi.F64, cabi.F32], [1, 1], cabi.F32, code, imm)[0] == 4
    assert cabi.pointwise_jit_compile(1, [cabi.F32] * 2, [1, 1], cabi.F64, code, imm)[0] == 4
    # an invalid instruction is a program error (B200K_ERR_PROGRAM), not a compile
    assert cabi.pointwise_jit_compile(1, [cabi.F32] * 2, [1, 1], cabi.F32, [99 * 10], [0.0])[0] not in (0, 4)


def test_counters_start_at_zero_without_a_gpu():
    s = cabi.pointwise_jit_stats()
    assert s == {"compiled": 0, "failed": 0, "launches": 0}
