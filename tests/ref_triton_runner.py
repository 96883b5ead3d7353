"""Runs the UNMODIFIED reference backend (installed in baseline/_ref) on the
benchmark's seeded inputs and saves its outputs, for the parity tests in
tests/test_gpu_parity_full.py.  A process of its own: the reference's
package is also named `compiler`.

    python tests/ref_triton_runner.py {sweep|mlp} OUT.pt
"""
from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import sweep_inputs as si  # noqa: E402
from compiler.backend import custom_backend  # noqa: E402  (the reference's package)


def main() -> None:
    case, out_path = sys.argv[1], sys.argv[2]
    torch._dynamo.config.recompile_limit = 64
    res = {}
    with torch.no_grad():
        if case == "sweep":
            for i in range(3 * len(si.SWEEP)):
                blk, x, r = si.sweep_point(i)
                torch._dynamo.reset()
                y = torch.compile(blk, backend=custom_backend)(x, r)
                res[i] = y[si.sample_rows(x.shape[0]).to(y.device)].cpu()
                del blk, x, r, y
                torch.cuda.empty_cache()
        elif case == "mlp":
            m, x = si.mlp()
            torch._dynamo.reset()
            res["mlp"] = torch.compile(m, backend=custom_backend)(x).cpu()
        else:
            raise SystemExit(f"unknown case {case}")
    torch.save(res, out_path)


if __name__ == "__main__":
    main()
