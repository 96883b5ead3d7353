"""CPU oracle for the fused-kernel path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of what the reference backend's generated kernels compute
(aashrith-madasu/torch-compile-backend, compiler/optimization/
fusion_pointwise.py and fusion_epilogue.py), used by tests/, by
``__graft_entry__.smoke()`` and by bench.py's CPU-baseline leg as the checker.
The product (torch-compile-backend_b200/) never imports it.

Pinned against golden vectors produced by running the reference's own Triton
kernels (under Triton's CPU interpreter) on seeded inputs:
tests/golden/make_golden.py writes them, tests/test_oracle_golden.py checks
this module against them.  The row-reduction functions (rowreduce.py) and the
rotary embedding (rope.py) have no reference counterpart (the reference leaves
them to ATen); they restate eager PyTorch's decomposed-graph semantics and are
pinned against torch on CPU.
"""
from .bf16 import round_bf16, round_to
from .gemm import gemm_epilogue, hand_gemm, hand_gemm_swizzled
from .pointwise import OPS, eval_group, matrix_add
from .rope import rope
from .rowreduce import layer_norm, log_softmax, rms_norm, rms_norm_swiglu, softmax

__all__ = [
    "OPS", "eval_group", "matrix_add", "gemm_epilogue", "hand_gemm", "hand_gemm_swizzled",
    "rms_norm", "rms_norm_swiglu", "layer_norm", "softmax", "log_softmax", "round_bf16", "round_to", "rope",
]
