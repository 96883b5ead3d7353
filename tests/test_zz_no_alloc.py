"""The allocation-free GEMM entry point, b200k_gemm_epilogue_noalloc.

For hosts that cannot call cudaMalloc (a capture-only runtime, a plugin
sandbox, a custom memory manager): the regular entry needs a caller-allocated
device status word, this one uses the library's own file-scope scratch.  The
test calls it through the C ABI twice in a row and checks each result
against the regular entry on the same inputs.  It lives in a file of its own
that pytest collects last, and passes alone in a fresh process as well as
after the other tests.
"""
import pytest
import torch

from compiler import runtime
from compiler.optimization.program import OP
from compiler.runtime import cabi

pytestmark = pytest.mark.gpu


def _program():
    # acc + bias, GELU (erf), + residual: the compiled-form path
    I = lambda op, operand=9, imm=0.0: (OP[op] * 10 + operand, imm)  # noqa: E731
    ins = [I("MOV", 0), I("ADD", 1), I("STORE", 0), I("MUL", 8, 0.7071067811865476), I("ERF"), I("ADD", 8, 1.0),
           I("STORE", 1), I("MOV", 0), I("MUL", 8, 0.5), I("MUL", 1), I("ADD", 2)]
    return [c for c, _ in ins], [v for _, v in ins], [1, 0, 1, -1, -1, 1]


@pytest.mark.parametrize("M,N,K", [(300, 520, 136), (1024, 768, 512)])
def test_noalloc_entry_matches_regular_entry_twice(M, N, K):
    runtime.load()
    cabi.library()
    dev = torch.device("cuda", 0)
    code, imm, form = _program()
    for call in range(2):
        g = torch.Generator(device=dev).manual_seed(17 + call)
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        w = torch.randn(N, K, device=dev, generator=g).to(torch.bfloat16)
        b = torch.randn(N, device=dev, generator=g).to(torch.bfloat16)
        r = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
        want = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        got = torch.full((M, N), float("nan"), device=dev, dtype=torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, want, status=status, form=form)
        cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, got, form=form, noalloc=True)
        torch.cuda.synchronize()
        assert status.item() == 0
        torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2)
