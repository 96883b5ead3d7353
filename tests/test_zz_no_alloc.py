"""The allocation-free GEMM entry point, b200k_gemm_epilogue_noalloc.

Some hosts cannot call cudaMalloc: a runtime that only records into CUDA
graphs, a plugin sandbox that hands out no device memory, an engine whose
own memory manager owns every byte.  They cannot supply the device status
word the regular entry takes, so this entry keeps that word in the
library's own file-scope scratch, and b200k_gemm_noalloc_status reads it
back.  The test calls both through the C ABI twice in a row and checks each
result bit for bit against the regular entry on the same inputs (the two
run the same kernel with the same tile choice), then makes one wait run out
and reads the timeout back through the reader.  It lives in a file of its
own that pytest collects last, and passes alone in a fresh process as well
as after the other tests.
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


def _inputs(M, N, K, seed):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    w = torch.randn(N, K, device=dev, generator=g).to(torch.bfloat16)
    b = torch.randn(N, device=dev, generator=g).to(torch.bfloat16)
    r = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
    return x, w, b, r


@pytest.mark.parametrize("M,N,K", [(300, 520, 136), (1024, 768, 512), (2048, 2048, 2048)])
def test_noalloc_entry_matches_regular_entry_twice(M, N, K):
    runtime.load()
    cabi.library()
    code, imm, form = _program()
    for call in range(2):
        x, w, b, r = _inputs(M, N, K, 17 + call)
        want = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
        got = torch.full((M, N), float("nan"), device=x.device, dtype=torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device=x.device)
        cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, want, status=status, form=form)
        cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, got, form=form, noalloc=True)
        assert cabi.gemm_noalloc_status() == 0
        torch.cuda.synchronize()
        assert status.item() == 0
        assert torch.equal(got, want)


def test_noalloc_entry_reports_a_stalled_wait():
    """The test hook withholds the first tile's accumulator-ready signal, so
    the epilogue's wait runs out after 50 ms; the timeout shows in the
    library's status word, the next call clears it, and the context stays
    usable."""
    runtime.load()
    code, imm, form = _program()
    M, N, K = 1024, 1024, 1024
    x, w, b, r = _inputs(M, N, K, 5)
    out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
    cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, out, form=form, noalloc=True, timeout_ns=50_000_000,
                       test_flags=cabi.GEMM_TEST_WITHHOLD_READY)
    assert cabi.gemm_noalloc_status() == 6  # B200K_ERR_TIMEOUT
    want = torch.empty_like(out)
    cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, want, status=torch.zeros(1, dtype=torch.int32, device=x.device),
                       form=form)
    cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, out, form=form, noalloc=True)
    assert cabi.gemm_noalloc_status() == 0
    assert torch.equal(out, want)
