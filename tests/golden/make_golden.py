"""Record golden vectors from the reference backend's own kernels.

Run where the reference checkout is available (read-only), not on the GPU box:

    python tests/golden/make_golden.py --reference <checkout of the reference>

Method.  The reference (aashrith-madasu/torch-compile-backend) is imported
from its checkout with TRITON_INTERPRET=1, so the Triton kernels it generates
(compiler/optimization/fusion_pointwise.py:132-169,
compiler/optimization/fusion_epilogue.py:72-151) run on CPU through Triton's
interpreter.  Four things are adjusted so it runs there, none of which
changes what a kernel computes:
  * the CUDA-only checks (`val.is_cuda` in _is_fusible, fusion_pointwise.py:70;
    _is_static_cuda, fusion_epilogue.py:41-42) accept CPU tensors;
  * the compile-time wall-clock gate (_epilogue_is_faster, :207-234) becomes
    the dtype rule it settles on for B200 (fp32 without TF32 -> cuBLAS, as its
    docstring says; fp16/bf16 -> fused), so the grouping is deterministic;
  * the autotuner gets one config (the interpreter cannot benchmark);
  * build_fused_op / build_epilogue_op are wrapped to record each kernel's
    group, argument order, inputs and output.
For every case in tests/golden/cases.py the script stores the reference's
grouping decisions, each fused kernel's inputs/outputs, and the compiled
model's output next to eager's.

Outputs (committed): reference_kernels.json + reference_kernels.npz.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.fx as fx  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from cases import CASES, make_case  # noqa: E402


def _spec(group, operand_index, acc_node=None):
    index = {n: j for j, n in enumerate(group)}
    spec = []
    for node in group:
        args = []
        for a in node.args:
            if isinstance(a, fx.Node):
                if a in index:
                    args.append(["node", index[a]])
                elif acc_node is not None and a is acc_node:
                    args.append(["acc"])
                else:
                    args.append(["in", operand_index[a]])
            else:
                args.append(float(a))
        if str(node.target) == "aten._to_copy.default":
            args.append(str(node.kwargs.get("dtype")).replace("torch.", ""))
        spec.append([str(node.target).replace("aten.", ""), args])
    return spec


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("B200_REFERENCE_DIR"),
                    required="B200_REFERENCE_DIR" not in os.environ,
                    help="checkout of the reference repository (or set B200_REFERENCE_DIR)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from compiler import backend as rb  # the reference's package
    from compiler.optimization import fusion_epilogue as fe
    from compiler.optimization import fusion_pointwise as fp

    def _is_fusible(node):
        if node.op != "call_function" or node.target not in fp.POINTWISE_OPS:
            return False
        if node.target == fp.aten._to_copy.default:
            if not fp._is_float_cast(node):
                return False
        elif node.kwargs:
            return False
        val = fp._tensor_meta(node)
        return val is not None and val.is_floating_point() and all(isinstance(s, int) for s in val.shape)

    fp._is_fusible = _is_fusible
    fe._is_static_cuda = lambda val: all(isinstance(s, int) for s in val.shape)
    fe._epilogue_is_faster = lambda group, matmul, inputs, op: fp._tensor_meta(matmul.args[-2]).dtype != torch.float32
    fe.AUTOTUNE_CONFIGS = (
        '[triton.Config({"BLOCK_M": 16, "BLOCK_N": 16, "BLOCK_K": 16, "GROUP_SIZE_M": 8}, num_warps=4, num_stages=3)]'
    )

    kernels: list[dict] = []
    arrays: dict[str, np.ndarray] = {}
    current: dict = {}

    orig_fused, orig_epi = fp.build_fused_op, fe.build_epilogue_op

    def rec_fused(group, inputs):
        op = orig_fused(group, inputs)
        entry = {
            "case": current["case"], "kind": "pointwise", "ops": [str(n.target) for n in group],
            "spec": _spec(group, {n: i for i, n in enumerate(inputs)}), "n_inputs": len(inputs),
            "out_dtype": str(fp._tensor_meta(group[-1]).dtype).replace("torch.", ""),
            "out_shape": list(fp._tensor_meta(group[-1]).shape), "calls": 0,
        }
        kernels.append(entry)
        k = len(kernels) - 1

        def wrapped(*tensors):
            out = op(*tensors)
            if entry["calls"] == 0 and current.get("record", True):
                entry["in_dtypes"] = [str(t.dtype).replace("torch.", "") for t in tensors]
                entry["in_strides"] = [list(t.stride()) for t in tensors]
                for i, t in enumerate(tensors):
                    arrays[f"k{k}_in{i}"] = t.detach().float().numpy() if t.dtype != torch.float64 else t.numpy()
                arrays[f"k{k}_out"] = out.detach().float().numpy()
                entry["calls"] = 1
            return out

        wrapped.__name__ = op.__name__
        return wrapped

    def rec_epi(group, matmul, inputs):
        op = orig_epi(group, matmul, inputs)
        entry = {
            "case": current["case"], "kind": "gemm_epilogue", "matmul": str(matmul.target),
            "ops": [str(n.target) for n in group],
            "spec": _spec(group, {n: i for i, n in enumerate(inputs)}, acc_node=matmul),
            "n_inputs": len(inputs), "bias_first": matmul.target == fp.aten.addmm.default,
            "out_dtype": str(fp._tensor_meta(group[-1]).dtype).replace("torch.", ""),
            "out_shape": list(fp._tensor_meta(group[-1]).shape), "calls": 0,
        }
        kernels.append(entry)
        k = len(kernels) - 1

        def wrapped(a, b, *tensors):
            out = op(a, b, *tensors)
            if entry["calls"] == 0:
                entry["ab_dtype"] = str(a.dtype).replace("torch.", "")
                entry["in_dtypes"] = [str(t.dtype).replace("torch.", "") for t in tensors]
                arrays[f"k{k}_a"] = a.detach().float().numpy()
                arrays[f"k{k}_b"] = b.detach().float().numpy()
                for i, t in enumerate(tensors):
                    arrays[f"k{k}_in{i}"] = t.detach().float().numpy()
                arrays[f"k{k}_out"] = out.detach().float().numpy()
                entry["calls"] = 1
            return out

        wrapped.__name__ = op.__name__
        return wrapped

    fp.build_fused_op = rec_fused
    fe.build_epilogue_op = rec_epi

    models = {}
    for case in CASES:
        current["case"] = case
        torch._dynamo.reset()
        mod, inputs = make_case(case)
        with torch.no_grad():
            eager = mod(*inputs)
            out = torch.compile(mod, backend=rb.custom_backend)(*inputs)
        for i, t in enumerate(inputs):
            arrays[f"{case}_x{i}"] = t.float().numpy()
        arrays[f"{case}_ref_out"] = out.float().numpy()
        arrays[f"{case}_eager_out"] = eager.float().numpy()
        groups = [(k["kind"], k["ops"]) for k in kernels if k["case"] == case and k["calls"]]
        models[case] = {"groups": groups, "out_dtype": str(out.dtype).replace("torch.", "")}
        err = (out.float() - eager.float()).abs().max().item()
        print(f"{case}: {len(groups)} fused kernels, |ref - eager| = {err:.3e}")

    with open(os.path.join(HERE, "reference_kernels.json"), "w") as f:
        json.dump({"kernels": kernels, "models": models,
                   "generator": "tests/golden/make_golden.py", "triton_interpret": True}, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "reference_kernels.npz"), **arrays)
    print(f"wrote {len(kernels)} kernels, {len(arrays)} arrays")


if __name__ == "__main__":
    main()
