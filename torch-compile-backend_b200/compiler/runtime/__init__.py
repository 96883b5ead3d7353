"""Loader for the sm_100a kernel library and its PyTorch binding.

``load()`` registers ``torch.ops.b200.*`` from the in-tree ``_b200_ops.so``
(built by torch-compile-backend_b200/csrc/build.py) plus their fake (meta)
implementations, so AOTAutograd's FakeTensor propagation and the FX passes
can use them.  There is no fallback: if the binding is missing, importing the
backend fails with the build command to run.
"""
from __future__ import annotations

import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200k.so")
EXT_PATH = os.path.join(HERE, "_b200_ops.so")

_loaded = False


class LibraryMissing(RuntimeError):
    pass


def load() -> None:
    global _loaded
    if _loaded:
        return
    if not os.path.exists(EXT_PATH) or not os.path.exists(LIB_PATH):
        raise LibraryMissing(
            f"the B200 kernel library is not built ({EXT_PATH} missing); run "
            "`python torch-compile-backend_b200/csrc/build.py` (nvcc, sm_100a)"
        )
    torch.ops.load_library(EXT_PATH)
    _register_fakes()
    _loaded = True


def _register_fakes() -> None:
    lib = "b200::"

    @torch.library.register_fake(lib + "pointwise")
    def _(inputs, code, imm, out_shape, out_dtype, out_stride=()):
        if out_stride:
            return inputs[0].new_empty_strided(out_shape, out_stride, dtype=out_dtype)
        return inputs[0].new_empty(out_shape, dtype=out_dtype)

    @torch.library.register_fake(lib + "gemm_epilogue")
    def _(a, b, extras, code, imm, out_shape, out_dtype, form=()):
        return a.new_empty(out_shape, dtype=out_dtype)

    @torch.library.register_fake(lib + "rms_norm")
    def _(x, weight, eps, flags, out_dtype):
        return x.new_empty(x.shape, dtype=out_dtype)

    @torch.library.register_fake(lib + "rms_norm_swiglu")
    def _(x, weight, eps, flags, out_dtype):
        return x.new_empty((*x.shape[:-1], x.shape[-1] // 2), dtype=out_dtype)

    @torch.library.register_fake(lib + "layer_norm")
    def _(x, normalized_shape, weight, bias, eps):
        stat = (*x.shape[:-1], 1)
        return (
            x.new_empty(x.shape),
            x.new_empty(stat, dtype=torch.float32),
            x.new_empty(stat, dtype=torch.float32),
        )

    @torch.library.register_fake(lib + "softmax")
    def _(x, dim, half_to_float):
        return x.new_empty(x.shape, dtype=torch.float32 if half_to_float else x.dtype)

    @torch.library.register_fake(lib + "log_softmax")
    def _(x, dim, half_to_float):
        return x.new_empty(x.shape, dtype=torch.float32 if half_to_float else x.dtype)

    @torch.library.register_fake(lib + "attention")
    def _(q, k, v, causal, scale, out_stride=()):
        if out_stride:
            return q.new_empty_strided(q.shape, out_stride)
        return q.new_empty(q.shape)

    @torch.library.register_fake(lib + "rope")
    def _(x, cos, sin, out_stride=()):
        if out_stride:
            return x.new_empty_strided(x.shape, out_stride)
        return x.new_empty(x.shape)

    @torch.library.register_fake(lib + "gemm_rope")
    def _(a, b, cos, sin, period, out_shape):
        return a.new_empty(out_shape)


def gemm_status(device: int = 0, reset: bool = True) -> int:
    """The GEMM kernels' device status word (0 = ok, 6 = a wait timed out);
    synchronises with the device."""
    load()
    return int(torch.ops.b200.gemm_status(device, reset))


def check_status(device: int = 0) -> None:
    """Synchronises with the device and raises RuntimeError if a GEMM launched
    through ``torch.ops.b200.gemm_epilogue`` reported a device-side timeout
    since the last check (the word is then cleared)."""
    load()
    v = gemm_status(device, reset=True)
    if v != 0:
        raise RuntimeError(f"b200::gemm_epilogue on cuda:{device} reported status {v} "
                           "(6 = a device-side wait timed out): an earlier GEMM's output is incomplete")
