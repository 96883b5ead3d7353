"""In-tree build of the sm_100a kernel library and its PyTorch binding.

    python torch-compile-backend_b200/csrc/build.py [--force]

Produces, next to the Python runtime that loads them
(torch-compile-backend_b200/compiler/runtime/):

  libb200k.so    the C-ABI kernel library (include/b200k.h), nvcc for
                 sm_100a only, static CUDA runtime, no torch dependency;
  _b200_ops.so   the thin TORCH_LIBRARY binding that registers
                 torch.ops.b200.* and calls libb200k.so (rpath $ORIGIN).

Objects go to torch-compile-backend_b200/_build/.  A target is rebuilt when
any source or header it depends on is newer than it.  nvcc cross-compiles
here without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
INCLUDE = os.path.join(REPO, "include")
OUT_DIR = os.path.join(PKG, "compiler", "runtime")
BUILD_DIR = os.path.join(PKG, "_build")

# (source, object name, defines).  gemm_fast.cu is compiled once per
# (tile width, activation) that has compiled-epilogue kernels; the
# activations are B200K_ACT_NONE, GELU_ERF, GELU_TANH, SILU, RELU.
CU_UNITS = [(src, os.path.splitext(src)[0], []) for src in ("capi.cu", "pointwise.cu", "pointwise_jit.cu", "rowreduce.cu", "rowreduce16.cu",
                                                                  "rope.cu", "gemm_sm100.cu", "attention.cu")]
CU_UNITS += [("gemm_fast.cu", f"gemm_fast_{bn}_{act}", [f"-DB200K_FAST_BN={bn}", f"-DB200K_FAST_ACT={act}"])
             for bn in (256, 192, 128) for act in (0, 1, 2, 3, 4)]
# ... and once per activation for the CTA-pair kernels (2: 256 x 256 tiles,
# 4: 256 x 512 tiles)
CU_UNITS += [("gemm_fast.cu", f"gemm_fast_pair{w}_{act}", [f"-DB200K_FAST_BN={w}", f"-DB200K_FAST_ACT={act}"])
             for w in (2, 4) for act in (0, 1, 2, 3, 4)]
HEADERS = [os.path.join(HERE, h) for h in ("common.cuh", "host_common.h", "gemm_kernel.cuh", "rowreduce.cuh",
                                           "pointwise_jit.h")] + [
    os.path.join(INCLUDE, "b200k.h")]
LIB = os.path.join(OUT_DIR, "libb200k.so")
EXT = os.path.join(OUT_DIR, "_b200_ops.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I" + INCLUDE, "-I" + HERE]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")


def _compile_cu(unit: tuple[str, str, list[str]], force: bool, verbose: bool) -> str:
    src, name, defines = unit
    obj = os.path.join(BUILD_DIR, name + ".o")
    path = os.path.join(HERE, src)
    if force or _newer(obj, [path] + HEADERS):
        _run([NVCC] + NVCC_FLAGS + defines + ["-c", path, "-o", obj], verbose)
    return obj


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension as ce

    incs = ce.include_paths(device_type="cuda")
    libs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-I" + sysconfig.get_paths()["include"]]
    cflags += ["-I" + i for i in incs]
    ldflags = ["-L" + l for l in libs] + ["-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch"]
    ldflags += [f"-Wl,-rpath,{l}" for l in libs if "torch" in l]
    return cflags, ldflags


def build(force: bool = False, verbose: bool = False) -> tuple[str, str]:
    """Compile libb200k.so and _b200_ops.so if out of date; returns their paths."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    ext_src = os.path.join(HERE, "torch_ops.cpp")
    with cf.ThreadPoolExecutor(max_workers=min(len(CU_UNITS), os.cpu_count() or 4)) as pool:
        objs = list(pool.map(lambda u: _compile_cu(u, force, verbose), CU_UNITS))
        if force or _newer(LIB, objs):
            _run([NVCC] + ARCH_FLAGS + ["-shared", "-Xcompiler", "-fPIC", "-o", LIB] + objs + ["-ldl"], verbose)
        if force or _newer(EXT, [ext_src, LIB, os.path.join(INCLUDE, "b200k.h")]):
            cflags, ldflags = _torch_flags()
            cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-I" + INCLUDE] + cflags
            cmd += [ext_src, "-o", EXT, "-L" + OUT_DIR, "-l:libb200k.so", "-Wl,-rpath,$ORIGIN"] + ldflags
            _run(cmd, verbose)
    return LIB, EXT


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true", help="rebuild everything")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    lib, ext = build(force=args.force, verbose=args.verbose)
    print(lib)
    print(ext)


if __name__ == "__main__":
    main()
