"""Backend switches and the kernel library's limits.

Environment flags (read once at import, overridable as module attributes):
  B200_EXTENSIONS=0   reference-identical grouping only: no view look-through
                      for 3-d linears, no row-reduction or rotary-embedding
                      fusion, no patch-embedding lowering
  B200_EPILOGUE=0     skip the GEMM+epilogue pass
  B200_POINTWISE=0    skip the pointwise pass
  B200_ROWREDUCE=0    skip the row-reduction pass
  B200_ROPE=0         skip the rotary-embedding passes
  B200_GEMM_ROPE=0    keep a rotated q / k projection as cuBLAS + the rotation
                      kernel instead of one GEMM with the rotation epilogue
  B200_PATCHIFY=0     keep patch-embedding convolutions as convolutions
  B200_ATTENTION=1    replace ATen's scaled-dot-product attention nodes with
                      the library's attention kernel (off by default)
  B200_DUMP=1         print each compiled graph and the fused-kernel programs
  B200_FAST_EPILOGUE=0  always interpret GEMM epilogue programs
  B200_CUDA_GRAPHS=0  run compiled inference graphs op by op instead of
                      replaying them as CUDA graphs (compiler/graph_replay.py)
  B200_GRAPH_MIN_LAUNCHES=N  replay only graphs with at least N launching
                      nodes (default 16: one GEMM gains nothing from replay
                      but would pay the input and output copies)
  B200_GRAPH_MAX_OUTPUT_MB=N  replay only graphs whose outputs, cloned after
                      every replay, total at most N MiB (default 64)

The reference hard-codes its equivalents (AUTOTUNE_CONFIGS, BLOCK=1024,
DOT_DTYPES in compiler/optimization/fusion_epilogue.py:23-38 and
fusion_pointwise.py:206) and has no switches.
"""
from __future__ import annotations

import os
from typing import Callable

import torch


def _flag(name: str, default: bool) -> bool:
    v = os.environ.get(name)
    return default if v is None else v not in ("0", "false", "False", "")


EXTENSIONS = _flag("B200_EXTENSIONS", True)
ENABLE_EPILOGUE = _flag("B200_EPILOGUE", True)
ENABLE_POINTWISE = _flag("B200_POINTWISE", True)
ENABLE_ROWREDUCE = _flag("B200_ROWREDUCE", True)
ENABLE_ROPE = _flag("B200_ROPE", True)
ENABLE_GEMM_ROPE = _flag("B200_GEMM_ROPE", True)
ENABLE_PATCHIFY = _flag("B200_PATCHIFY", True)
# The attention kernel is parity-tested but measured slower than PyTorch's
# cuDNN SDPA on B200 (Llama-style prefill 327 vs 208 us, ViT-B/16 57 vs 35
# us per layer), so the pass is opt-in.
ENABLE_ATTENTION = _flag("B200_ATTENTION", False)
DUMP = _flag("B200_DUMP", False)
FAST_EPILOGUE = _flag("B200_FAST_EPILOGUE", True)  # compiled path for canonical GEMM epilogues
CUDA_GRAPHS = _flag("B200_CUDA_GRAPHS", True)  # replay compiled inference graphs as CUDA graphs
GRAPH_MIN_LAUNCHES = int(os.environ.get("B200_GRAPH_MIN_LAUNCHES", "16"))
GRAPH_MAX_OUTPUT_MB = int(os.environ.get("B200_GRAPH_MAX_OUTPUT_MB", "64"))

# Kernel library limits (include/b200k.h).
MAX_INPUTS = 8
MAX_DIMS = 6
LOADABLE_DTYPES = {
    torch.float32, torch.float16, torch.bfloat16, torch.float64,
    torch.int32, torch.int64, torch.bool, torch.uint8,
}
STORABLE_DTYPES = {torch.float32, torch.float16, torch.bfloat16, torch.float64}
GEMM_AB_DTYPES = {torch.float16, torch.bfloat16}


def gemm_ab_dtypes() -> set:
    """Operand dtypes the GEMM kernels take now: 16-bit always, fp32 when
    torch allows TF32 for matmuls (the kernels then run TF32 tensor cores,
    as cuBLAS would; the reference likewise lets its fp32 dots use TF32 only
    under that flag, compiler/optimization/fusion_epilogue.py:82-86)."""
    if torch.backends.cuda.matmul.allow_tf32:
        return GEMM_AB_DTYPES | {torch.float32}
    return GEMM_AB_DTYPES
GEMM_OUT_DTYPES = {torch.float16, torch.bfloat16, torch.float32}
ROW_DTYPES = {torch.float32, torch.float16, torch.bfloat16}

# The fusions fire only for tensors on this predicate's device: CUDA, as in the
# reference (fusion_pointwise.py:70, fusion_epilogue.py:41-42).  Tests that
# inspect the rewritten graph on a CPU-only machine swap it out.
_device_predicate: Callable[[torch.Tensor], bool] = lambda val: val.is_cuda


def on_target_device(val: torch.Tensor) -> bool:
    return _device_predicate(val)


def set_device_predicate(fn: Callable[[torch.Tensor], bool]) -> Callable[[torch.Tensor], bool]:
    """Replace the device predicate; returns the previous one."""
    global _device_predicate
    old = _device_predicate
    _device_predicate = fn
    return old
