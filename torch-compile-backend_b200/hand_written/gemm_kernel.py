"""`gemm(a, b)` with the API of the reference's hand_written/gemm_kernel.py:51-71:
C = A @ B accumulated in fp32, returned as fp16.  Runs the persistent tcgen05
GEMM of libb200k.so (torch.ops.b200.gemm_epilogue with an empty epilogue)
instead of the reference's 64x64x32 Triton tile kernel."""
import torch

from compiler import runtime

runtime.load()


def gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    assert a.shape[1] == b.shape[0], "incompatible tensor shapes"
    if a.dtype not in (torch.float16, torch.bfloat16) or b.dtype != a.dtype:
        raise ValueError("a and b must both be float16 or both bfloat16")
    if a.stride(1) != 1:
        a = a.contiguous()
    if b.stride(0) != 1 and b.stride(1) != 1:
        b = b.contiguous()
    M, N = a.shape[0], b.shape[1]
    return torch.ops.b200.gemm_epilogue(a, b, [], [], [], [M, N], torch.float16)
