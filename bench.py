"""Benchmark: fused GEMM + epilogue sweep on B200 (the headline workload).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload sweep|gemm|chain|vit|llama|pointwise]
                    [--backend ours|eager|reference_triton|inductor]

One step of the default workload ("gemm_epilogue_sweep") runs the fused bf16
GEMM sweep once: Y = act(X W^T + b) + R for act in {none, gelu, silu} and
(M, N, K) in {512^3, 4096^3, 8192^3, (16384, 4096, 14336)} -- twelve launches
of the library's tcgen05 GEMM kernel with the epilogue fused.  `value` is the
sweep's total FLOPs (2MNK per GEMM) / device time, inputs resident in HBM.
`e2e` is the same metric through the public API (torch.compile with
custom_backend) with X and R copied in from pinned host memory and Y copied
back inside the timed region; the copies run on two copy streams, so one
GEMM's transfers overlap its neighbours' compute.

The same line carries the other half of the benchmark's metric: `models`
(ViT-B/16 batch 64 and the Llama-style prefill 8 x 2048, forward tokens/s
through this backend, eager PyTorch and, at N = 1, the reference Triton
backend), `chain` (RMSNorm+SwiGLU and softmax GB/s) and `cpu_baseline` (the
reference's CPU path on the host cores, N = 1).  --no-extras skips them.

Multi-GPU: one process per GPU (torchrun), each GPU runs the full sweep as an
independent replica (weak scaling, no data-path collective); the model
extras split their batch over the GPUs.  A gloo process group carries only
the barrier and the max-over-ranks time.  Each rank is bound to the host
CPUs of its GPU's NUMA node.

--impl reference times the reference's own CPU path of the sweep on the
host cores: the unmodified reference backend (baseline/_ref) compiling each
sweep block on CPU tensors, where it fuses nothing, i.e. eager PyTorch bf16
on the same ATen graph, on a bounded row sample of every sweep GEMM.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def _use_ours() -> None:
    p = os.path.join(ROOT, "torch-compile-backend_b200")
    if p not in sys.path:
        sys.path.insert(0, p)


def _use_reference_triton() -> None:
    """The unmodified reference backend installed in baseline/_ref (its package
    is also called `compiler`, so it runs in a process of its own)."""
    p = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(p, "compiler")):
        raise RuntimeError("reference not installed in baseline/_ref")
    sys.path.insert(0, p)


SWEEP = [(512, 512, 512), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 4096, 14336)]
ACTS = ["none", "gelu", "silu"]
DOMINANT = (16384, 4096, 14336)
L2_BYTES = 126 * 1024 * 1024


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# Kernel name per tile config of the dominant launch.
_DOMINANT_KERNELS = {3: "gemm_pair_kernel 256x256", 4: "gemm_pair_kernel 256x512"}


def _dominant_kernel() -> tuple[str]:
    """The kernel the library picks for the sweep's dominant launch."""
    from compiler.runtime import cabi

    cfg = cabi.library().b200k_gemm_pick_config(*DOMINANT)
    return (_DOMINANT_KERNELS.get(cfg, "gemm_epilogue_kernel"),)


# --------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.02)  # the timed region starts once sampling runs
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        rows = []
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        loaded = [r for r in rows if r[2] > 300.0] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


# --------------------------------------------------------------- distributed
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist

            dist.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            import torch.distributed as dist

            dist.destroy_process_group()


# --------------------------------------------------------------- sweep
def _sweep_problems(dev, gen):
    from bench_models import GemmEpilogueBlock, init_sweep_block

    probs = []
    for (M, N, K) in SWEEP:
        x = (0.02 * torch.randn(M, K, device=dev, generator=gen)).to(torch.bfloat16)
        r = (0.02 * torch.randn(M, N, device=dev, generator=gen)).to(torch.bfloat16)
        for act in ACTS:
            blk = GemmEpilogueBlock(K, N, act)
            init_sweep_block(blk, torch.Generator().manual_seed(len(probs)))
            blk = blk.to(dev, torch.bfloat16).eval()
            probs.append({"shape": (M, N, K), "act": act, "x": x, "r": r, "block": blk})
    return probs


def _pass_program(block, x, r):
    """The (code, imm) the FX passes build for this block: compile it with a
    backend that keeps the rewritten graph and read the fused node's args."""
    _use_ours()
    from torch._decomp import get_decompositions
    from torch._dynamo.backends.common import aot_autograd

    from compiler import backend as B

    found = []

    def comp(gm, example_inputs):
        f = B.compiler(gm, example_inputs)
        found.extend(n for n in gm.graph.nodes if n.op == "call_function"
                     and n.target == torch.ops.b200.gemm_epilogue.default)
        return f

    be = aot_autograd(fw_compiler=comp, decompositions=get_decompositions([torch.ops.aten.gelu, torch.ops.aten.silu]))
    torch._dynamo.reset()
    with torch.no_grad():
        torch.compile(block, backend=be)(x[:128], r[:128])
    if len(found) != 1:
        raise RuntimeError(f"expected one fused GEMM+epilogue node, got {len(found)}")
    n = found[0]
    return list(n.args[3]), list(n.args[4]), list(n.args[7]) if len(n.args) > 7 else []


def _smi_id(local: int) -> str:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(ids):
            return ids[local]
    return str(local)


def run_sweep(args, dist: Dist) -> dict:
    _use_ours()
    from compiler import runtime
    from compiler.backend import custom_backend

    runtime.load()
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(0)
    probs = _sweep_problems(dev, gen)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)

    # Device-resident step: the exact op the compiled graph calls.
    outs = []
    for p in probs:
        M, N, K = p["shape"]
        code, imm, form = _pass_program(p["block"], p["x"], p["r"])
        p["form"] = form
        lin = p["block"].lin
        p["call"] = (lambda x=p["x"], w=lin.weight, b=lin.bias, r=p["r"], c=code, i=imm, s=[M, N], f=form:
                     torch.ops.b200.gemm_epilogue(x, w.t(), [b, r], c, i, s, torch.bfloat16, f))
    flops = sum(2.0 * p["shape"][0] * p["shape"][1] * p["shape"][2] for p in probs)

    def step(record=None):
        for j, p in enumerate(probs):
            if record is not None:
                _gpu_lead()  # the events then bracket the kernel, not the host's enqueue
                record[j][0].record()
            out = p["call"]()
            if record is not None:
                record[j][1].record()
        return out

    for _ in range(args.warmup):
        flush.zero_()
        step()
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in probs]
          for _ in range(args.steps)]
    torch.cuda.synchronize()
    dist.barrier()
    with ClockSampler(_smi_id(dist.local)) as clk:
        torch.cuda.synchronize()
        for k in range(args.steps):
            flush.zero_()  # L2 flush between steps (outside the per-launch events)
            step(ev[k])
        torch.cuda.synchronize()
    dist.barrier()
    per = [[ev[k][j][0].elapsed_time(ev[k][j][1]) for k in range(args.steps)] for j in range(len(probs))]
    step_ms = sum(sum(per[j][k] for j in range(len(probs))) for k in range(args.steps)) / args.steps
    step_ms = dist.max(step_ms)

    # Correctness spot check of the timed op against the fp32 reference (8 rows).
    p = probs[4]
    lin = p["block"].lin
    y = p["call"]()
    ref = torch.nn.functional.gelu(p["x"][:8].float() @ lin.weight.float().t() + lin.bias.float()) + p["r"][:8].float()
    err = ((y[:8].float() - ref).abs().max() / ref.abs().max()).item()

    # End to end through torch.compile(custom_backend) with host buffers.
    # The twelve blocks are instances of one class, so dynamo compiles the
    # same frame once per block: its recompile limit (8 by default) would
    # send the last blocks to eager PyTorch, and its automatic dynamic shapes
    # would compile the blocks after a shape change with symbolic sizes,
    # which the fusion passes (static shapes) leave to ATen.  Raise the limit
    # and make hitting it an error, compile with static shapes, and check
    # below that every block's graph holds a fused GEMM.
    torch._dynamo.reset()
    torch._dynamo.config.recompile_limit = max(torch._dynamo.config.recompile_limit, 4 * len(probs))
    torch._dynamo.config.fail_on_recompile_limit_hit = True
    compiled = [torch.compile(p["block"], backend=custom_backend, dynamic=False) for p in probs]
    host = []
    for p in probs:
        M, N, K = p["shape"]
        host.append((p["x"].cpu().pin_memory(), p["r"].cpu().pin_memory(),
                     torch.empty(M, N, dtype=torch.bfloat16).pin_memory()))
    h2d = sum(hx.numel() * 2 + hr.numel() * 2 for hx, hr, _ in host)
    d2h = sum(hy.numel() * 2 for _, _, hy in host)

    # The copies run on their own streams, so the PCIe transfers of one GEMM
    # overlap the compute of its neighbours (as a serving loop would run it):
    # host->device on `up`, the compiled call on the current stream, the
    # result's device->host on `down`.  record_stream keeps the caching
    # allocator from reusing a buffer before the stream that reads it is done.
    compute = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()

    def e2e_step():
        for (hx, hr, hy), f in zip(host, compiled):
            with torch.cuda.stream(up):
                x = hx.to(dev, non_blocking=True)
                r = hr.to(dev, non_blocking=True)
            compute.wait_stream(up)
            x.record_stream(compute)
            r.record_stream(compute)
            with torch.no_grad():
                y = f(x, r)
            down.wait_stream(compute)
            with torch.cuda.stream(down):
                hy.copy_(y, non_blocking=True)
            y.record_stream(down)

    from compiler import backend as _backend

    graphs0, gemms0 = _backend.GRAPHS_COMPILED, _backend.GEMMS_FUSED
    for _ in range(max(1, args.warmup)):
        e2e_step()
    compute.wait_stream(down)
    e2e_graphs = _backend.GRAPHS_COMPILED - graphs0
    e2e_gemms = _backend.GEMMS_FUSED - gemms0
    if e2e_graphs < len(probs) or e2e_gemms < len(probs):
        raise RuntimeError(f"{e2e_graphs} graphs with {e2e_gemms} fused GEMMs for {len(probs)} e2e blocks")
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    up.wait_stream(compute)  # no copy starts before e0
    for _ in range(args.steps):
        e2e_step()
    compute.wait_stream(down)  # e1 follows the last result's copy to the host
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_ms = dist.max(e0.elapsed_time(e1) / args.steps)

    peaks, src = load_peaks()
    dom = [j for j, p in enumerate(probs) if p["shape"] == DOMINANT and p["act"] == "gelu"][0]
    M, N, K = DOMINANT
    dom_ms = statistics.mean(per[dom])
    achieved = 2.0 * M * N * K / (dom_ms * 1e-3) / 1e12
    # Each launch is timed on its own (events around it), so the burst peak
    # is the denominator; the sustained figure is reported beside it.
    peak = peaks["bf16_tflops"]
    sustained = peaks.get("bf16_tflops_sustained")
    sweep_detail = []
    for (M, N, K) in SWEEP:
        for act in ACTS:
            j = [i for i, p in enumerate(probs) if p["shape"] == (M, N, K) and p["act"] == act][0]
            ms = statistics.mean(per[j])
            sweep_detail.append({"M": M, "N": N, "K": K, "act": act, "ms": round(ms, 4),
                                 "tflops": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 1)})
    n = dist.world
    return {
        "metric": "fused GEMM+epilogue TFLOP/s",
        "value": round(n * flops / (step_ms * 1e-3) / 1e12, 2),
        "unit": "TFLOP/s",
        "n_gpus": n,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) X/W/R, N(0,0.01) b)",
        "config": {"workload": "gemm_epilogue_sweep", "shapes": SWEEP, "acts": ACTS,
                   "epilogue": "act(X W^T + b) + R, bf16 in/out, fp32 accumulate",
                   "l2": "256 MB flush between steps (outside the per-launch events)",
                   "timing": "CUDA events per launch, each after a ~100 us GPU spin (outside the events) so "
                             "the host's enqueue is not timed",
                   "parallelism": f"replicas x{n}"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 3), "peak_source": f"{src} bf16_tflops (burst)",
                     "frac_of_sustained": round(achieved / sustained, 3) if sustained else None,
                     "kernel": _dominant_kernel()[0] + " 16384x4096x14336 gelu",
                     "algorithmic_bytes": 2 * (M * K + N * K + 2 * M * N) + 2 * N,
                     "traffic": None,
                     "traffic_note": "not measured by this run (ncu cannot run inside it); the ncu "
                                     "capture of this kernel is summarised under profiles/"},
        "e2e": {"value": round(n * flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
                "graphs_compiled": e2e_graphs, "gemms_fused": e2e_gemms,
                "copy_gbs": round((h2d + d2h) / (e2e_ms * 1e-3) / 1e9, 1)},
        "gpu_launches": args.steps * len(probs),
        "clocks": clk.summary(),
        "sweep": sweep_detail,
        "epilogue_paths": sorted({"compiled" if p["form"] else "interpreted" for p in probs}),
        "spot_check_max_rel_err": round(err, 5),
    }


def run_sweep_backend(args, dist: Dist) -> dict:
    """The sweep through torch.compile with another backend (the reference
    Triton backend from baseline/_ref, eager, or inductor), inputs resident
    on the device: each block's call timed with CUDA events, an L2 flush
    between steps, value = sweep FLOPs / summed device time.  The blocks are
    the default workload's (same shapes, seeds and epilogues)."""
    from bench_models import GemmEpilogueBlock, init_sweep_block

    be = _backend(args.backend)
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(0)
    torch._dynamo.config.recompile_limit = max(torch._dynamo.config.recompile_limit, 64)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    calls, flops = [], 0.0
    t0 = time.perf_counter()
    for (M, N, K) in SWEEP:
        x = (0.02 * torch.randn(M, K, device=dev, generator=gen)).to(torch.bfloat16)
        r = (0.02 * torch.randn(M, N, device=dev, generator=gen)).to(torch.bfloat16)
        for act in ACTS:
            blk = GemmEpilogueBlock(K, N, act)
            init_sweep_block(blk, torch.Generator().manual_seed(len(calls)))
            blk = blk.to(dev, torch.bfloat16).eval()
            # static shapes: the blocks share one class, and dynamo's automatic
            # dynamic shapes would hand every block after the first shape change
            # to the backend with symbolic sizes, which both backends' fusion
            # passes leave to ATen
            f = blk if be is None else torch.compile(blk, backend=be, dynamic=False)
            calls.append((f, x, r))
            flops += 2.0 * M * N * K
    with torch.no_grad():
        for f, x, r in calls:  # compile (and, for the reference, autotune) each block
            f(x, r)
        torch.cuda.synchronize()
        compile_s = time.perf_counter() - t0
        per = [_time_device(lambda f=f, x=x, r=r: f(x, r), args.steps, args.warmup, flush, lead=True)
               for f, x, r in calls]
    total_ms = sum(statistics.median(t) for t in per)
    return {"metric": "fused GEMM+epilogue TFLOP/s", "value": round(flops / (total_ms * 1e-3) / 1e12, 2),
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms, 4), "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "gemm_epilogue_sweep", "backend": args.backend},
            "compile_s": round(compile_s, 1)}


def _reference_triton_sweep(steps: int, warmup: int) -> dict:
    """run_sweep_backend with the reference Triton backend, in a process of
    its own (its package is also named `compiler`)."""
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--workload", "sweep", "--backend", "reference_triton",
           "--steps", str(steps), "--warmup", str(warmup)]
    env = dict(os.environ)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    except subprocess.TimeoutExpired:
        return {"unavailable": "timed out after 900 s"}
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode == 0 and lines:
        d = json.loads(lines[-1])
        return {"value": d["value"], "unit": d["unit"], "ms": d["ms_per_step"], "compile_s": d["compile_s"]}
    err = [ln for ln in r.stderr.splitlines() if "Error" in ln or "error" in ln]
    return {"unavailable": (err[-1] if err else f"exit code {r.returncode}")[:300]}


def run_single_gemm(args, dist: Dist) -> dict:
    """One sweep point on its own: --shape M,N,K --act none|gelu|silu [--tile-config c].
    Used for ncu captures and for measuring the tile table."""
    _use_ours()
    from bench_models import GemmEpilogueBlock, init_sweep_block
    from compiler import runtime

    runtime.load()
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    M, N, K = (int(v) for v in args.shape.split(","))
    gen = torch.Generator(device=dev).manual_seed(0)
    x = (0.02 * torch.randn(M, K, device=dev, generator=gen)).to(torch.bfloat16)
    r = (0.02 * torch.randn(M, N, device=dev, generator=gen)).to(torch.bfloat16)
    blk = GemmEpilogueBlock(K, N, args.act)
    init_sweep_block(blk, torch.Generator().manual_seed(0))
    blk = blk.to(dev, torch.bfloat16).eval()
    code, imm, form = _pass_program(blk, x, r)
    if args.interpret:
        form = []
    w, b = blk.lin.weight, blk.lin.bias
    if args.plain:  # out = x w^T alone, against torch.mm (cuBLAS) in the eager leg
        from compiler.optimization.program import OP

        code, imm, form = [OP["MOV"] * 10], [0.0], [1, -1, 0, -1, -1, -1]

        def call():
            return torch.ops.b200.gemm_epilogue(x, w.t(), [], code, imm, [M, N], torch.bfloat16, form)
    elif args.tile_config >= 0:
        from compiler.runtime import cabi

        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)

        def call():
            cabi.gemm_epilogue(x, w.t(), [b, r], code, imm, out, tile_config=args.tile_config, form=form)
            return out
    else:
        def call():
            return torch.ops.b200.gemm_epilogue(x, w.t(), [b, r], code, imm, [M, N], torch.bfloat16, form)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        call()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    # host cost per call: back-to-back calls, one sync at the end
    t0 = time.perf_counter()
    for _ in range(50):
        call()
    torch.cuda.synchronize()
    wall_us = (time.perf_counter() - t0) / 50 * 1e6
    ms = statistics.median(times)
    # the same block in eager PyTorch (cuBLAS addmm + ATen epilogue kernels)
    with torch.no_grad():
        eager = (lambda: torch.mm(x, w.t())) if args.plain else (lambda: blk(x, r))
        eager_ms = statistics.median(_time_device(eager, args.steps, args.warmup, flush))
    return {"metric": "fused GEMM+epilogue TFLOP/s", "value": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 1),
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "gemm" if args.plain else "gemm_epilogue", "M": M, "N": N, "K": K,
                       "act": "none (no epilogue)" if args.plain else args.act,
                       "tile_config": args.tile_config, "program_len": len(code),
                       "epilogue_path": "compiled" if form else "interpreted"},
            "back_to_back_us_per_call": round(wall_us, 1),
            "eager_ms": round(eager_ms, 4), "eager_tflops": round(2.0 * M * N * K / (eager_ms * 1e-3) / 1e12, 1)}


def _backend(name: str):
    if name == "eager":
        return None
    if name == "ours":
        _use_ours()
        from compiler.backend import custom_backend

        return custom_backend
    if name == "reference_triton":
        _use_reference_triton()
        from compiler.backend import custom_backend

        return custom_backend
    if name == "inductor":
        return "inductor"
    raise ValueError(name)


LEAD_CYCLES = 200_000  # ~100 us of GPU spin at the B200's 1965 MHz


def _gpu_lead() -> None:
    """Queues a short GPU spin outside the timed events: while it runs the
    host enqueues the start event, the launch and the end event, so a
    launch whose host-side cost exceeds its kernel time (512^3) is timed as
    the kernel, not as the host's enqueue.  Both sweep legs (this library and
    the backends compared with it) use it."""
    torch.cuda._sleep(LEAD_CYCLES)


def _time_device(fn, steps: int, warmup: int, flush=None, lead: bool = False) -> list[float]:
    """Device time of each of `steps` calls (CUDA events on the current
    stream around the call, an L2 flush between calls).  The steps are queued
    back to back and synchronised once at the end, so the host's per-call
    cost overlaps the device's work, as in a running model; with `lead`, a
    GPU spin before each call keeps the host's enqueue out of the events."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = []
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        if lead:
            _gpu_lead()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        ev.append((e0, e1))
    torch.cuda.synchronize()
    return [e0.elapsed_time(e1) for e0, e1 in ev]


def run_model(args, dist: Dist) -> dict:
    """ViT-B/16 (batch 64) or Llama-style prefill (8 x 2048) forward, tokens/s,
    with --backend eager | ours | reference_triton | inductor."""
    import bench_models as bm

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    torch.manual_seed(0)
    gen = torch.Generator(device=dev).manual_seed(0)
    if args.workload == "vit":
        model = bm.ViT().to(dev, torch.bfloat16).eval()
        x = torch.randn(args.batch or 64, 3, 224, 224, device=dev, generator=gen).to(torch.bfloat16)
        tokens = x.shape[0] * 197
        flops = bm.vit_flops_per_image() * x.shape[0]
        cfg = {"workload": "vit_b16_forward", "batch": x.shape[0], "tokens": tokens}
    else:
        model = bm.Llama()
        bm.init_normal_(model, 0.02, torch.Generator().manual_seed(0))
        model = model.to(dev, torch.bfloat16).eval()
        x = torch.randint(0, 128256, (args.batch or 8, 2048), device=dev, generator=gen)
        tokens = x.numel()
        flops = bm.llama_flops_per_token() * tokens
        cfg = {"workload": "llama_prefill_forward", "batch": x.shape[0], "seq": 2048, "tokens": tokens}
    be = _backend(args.backend)
    t0 = time.perf_counter()
    f = model if be is None else torch.compile(model, backend=be)
    with torch.no_grad():
        f(x)
        torch.cuda.synchronize()
        compile_s = time.perf_counter() - t0
        times = _time_device(lambda: f(x), args.steps, args.warmup)
    ms = statistics.median(times)
    return {"metric": "forward tokens/s", "value": round(tokens / (ms * 1e-3), 1), "unit": "tokens/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic, random init",
            "config": dict(cfg, backend=args.backend),
            "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "compile_s": round(compile_s, 1)}


def run_chain(args, dist: Dist) -> dict:
    """RMSNorm -> split -> SiLU(gate)*up on h[16384, 8192] and softmax over
    [32768, 4096] (bf16), through the compiled graph; GB/s of algorithmic
    traffic (one read of the input, one write of the output)."""
    import torch.nn.functional as F

    import bench_models as bm

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(0)

    class RMSSwiGLU(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.norm = bm.RMSNorm(8192, 1e-6)

        def forward(self, h):
            y = self.norm(h)
            g, u = y.split(4096, dim=-1)
            return F.silu(g) * u

    class Softmax(torch.nn.Module):
        def forward(self, z):
            return torch.softmax(z, -1)

    m = RMSSwiGLU().to(dev)
    with torch.no_grad():
        m.norm.weight.copy_(1 + 0.02 * torch.randn(8192, device=dev, generator=gen))
    m = m.to(torch.bfloat16)
    h = torch.randn(16384, 8192, device=dev, generator=gen).to(torch.bfloat16)
    z = (2.0 * torch.randn(32768, 4096, device=dev, generator=gen)).to(torch.bfloat16)
    be = _backend(args.backend)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    out = {}
    with torch.no_grad():
        for name, mod, inp, nbytes in (("rmsnorm_swiglu", m, h, 16384 * 8192 * 2 + 8192 * 2 + 16384 * 4096 * 2),
                                       ("softmax", Softmax(), z, 2 * 32768 * 4096 * 2)):
            torch._dynamo.reset()
            f = mod if be is None else torch.compile(mod, backend=be)
            times = _time_device(lambda: f(inp), args.steps, args.warmup, flush)
            ms = statistics.median(times)
            out[name] = {"ms": round(ms, 4), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1), "bytes": nbytes}
    peaks, src = load_peaks()
    tot_bytes = sum(v["bytes"] for v in out.values())
    tot_ms = sum(v["ms"] for v in out.values())
    gbs = tot_bytes / (tot_ms * 1e-3) / 1e9
    return {"metric": "pointwise/reduction chain GB/s", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tot_ms, 4), "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic", "config": {"workload": "rmsnorm_swiglu+softmax",
                                                             "backend": args.backend},
            "kernels": out, "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 3),
                                         "peak_source": src + " hbm_gbs"}}


def run_pointwise(args, dist: Dist) -> dict:
    """Pointwise chains through the compiled graph (the pointwise pass and
    `b200k_pointwise`): `(x*sigmoid(x) + r) * w` in bf16 on [16384, 8192]
    with w [8192], `(a + b) * 0.5` in bf16 on [16384, 8192] and
    `(a + b) * c` in fp32 on [16384, 4096]; GB/s of algorithmic traffic
    (every input read once, the output written once)."""
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(0)

    class SiluResScale(torch.nn.Module):
        def forward(self, x, r, w):
            return (x * torch.sigmoid(x) + r) * w

    class AddHalf(torch.nn.Module):
        def forward(self, a, b):
            return (a + b) * 0.5

    class AddMul(torch.nn.Module):
        def forward(self, a, b, c):
            return (a + b) * c

    def rnd(*shape, dt=torch.bfloat16):
        return torch.randn(*shape, device=dev, generator=gen).to(dt)

    cases = (("silu_residual_scale_bf16", SiluResScale(), (rnd(16384, 8192), rnd(16384, 8192), rnd(8192))),
             ("add_half_bf16", AddHalf(), (rnd(16384, 8192), rnd(16384, 8192))),
             ("add_mul_f32", AddMul(), tuple(rnd(16384, 4096, dt=torch.float32) for _ in range(3))))
    be = _backend(args.backend)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    out = {}
    with torch.no_grad():
        for name, mod, inp in cases:
            nbytes = sum(t.numel() * t.element_size() for t in inp) + inp[0].numel() * inp[0].element_size()
            torch._dynamo.reset()
            f = mod if be is None else torch.compile(mod, backend=be)
            times = _time_device(lambda: f(*inp), args.steps, args.warmup, flush)
            ms = statistics.median(times)
            out[name] = {"ms": round(ms, 4), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1), "bytes": nbytes}
    peaks, src = load_peaks()
    tot_bytes = sum(v["bytes"] for v in out.values())
    tot_ms = sum(v["ms"] for v in out.values())
    gbs = tot_bytes / (tot_ms * 1e-3) / 1e9
    return {"metric": "pointwise chain GB/s", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tot_ms, 4), "higher_is_better": True,
            "dtype": "bf16+fp32", "data": "synthetic", "config": {"workload": "pointwise_chains", "backend": args.backend},
            "kernels": out, "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 3),
                                         "peak_source": src + " hbm_gbs"}}


def run_attention(args, dist: Dist) -> dict:
    """The attention kernel alone (torch.ops.b200.attention) against PyTorch's
    SDPA (cuDNN / flash) on the two model configs: the Llama prefill's causal
    grouped-query attention [8, 32 / 8 heads, 2048, 64] and ViT-B/16's
    [64, 12, 197, 64].  TFLOP/s counts the unmasked products only
    (4 B H L S D, halved for the causal mask)."""
    _use_ours()
    import torch.nn.functional as F

    from compiler import runtime

    runtime.load()
    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(0)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    out = {}
    for name, (B, H, Hkv, L, causal) in (("llama_prefill", (8, 32, 8, 2048, True)),
                                         ("vit_b16", (64, 12, 12, 197, False))):
        def mk(h):  # [B, S, H, D] memory, viewed [B, H, S, D] (the models' projections)
            return torch.randn(B, L, h, 64, device=dev, generator=gen).to(torch.bfloat16).transpose(1, 2)

        q, k, v = mk(H), mk(Hkv), mk(Hkv)
        stride = list(torch.empty(B, L, H, 64).transpose(1, 2).stride())
        flops = 4.0 * B * H * L * L * 64 * (0.5 if causal else 1.0)
        ours = statistics.median(_time_device(lambda: torch.ops.b200.attention(q, k, v, causal, -1.0, stride),
                                              args.steps, args.warmup, flush))
        theirs = statistics.median(_time_device(
            lambda: F.scaled_dot_product_attention(q, k, v, is_causal=causal, enable_gqa=H != Hkv),
            args.steps, args.warmup, flush))
        runtime.check_status(dist.local)
        out[name] = {"ms": round(ours, 4), "tflops": round(flops / (ours * 1e-3) / 1e12, 1),
                     "sdpa_ms": round(theirs, 4), "sdpa_tflops": round(flops / (theirs * 1e-3) / 1e12, 1)}
    peaks, src = load_peaks()
    ll = out["llama_prefill"]
    return {"metric": "attention TFLOP/s", "value": ll["tflops"], "unit": "TFLOP/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ll["ms"], "higher_is_better": True,
            "dtype": "bf16", "data": "synthetic N(0,1)", "config": {"workload": "attention"}, "kernels": out,
            "roofline": {"bound": "tensor", "achieved": ll["tflops"], "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": round(ll["tflops"] / peaks["bf16_tflops"], 3),
                         "peak_source": src + " bf16_tflops (burst)"}}


# --------------------------------------------------------------- CPU (reference) leg
def _host_threads() -> int:
    """Every host thread this process may run on (torchrun sets
    OMP_NUM_THREADS=1 for its ranks; the CPU leg overrides it)."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def run_reference_cpu(steps: int, warmup: int, rows: int, models: bool = True) -> dict:
    """The reference's own CPU path for the sweep on the host cores.

    Each block runs through ``torch.compile(block, backend=custom_backend)``
    with the UNMODIFIED reference backend from baseline/_ref.  On CPU tensors
    that backend fuses nothing (its passes require CUDA values,
    compiler/optimization/fusion_pointwise.py:70 and fusion_epilogue.py:41-42),
    so a step is eager PyTorch bf16 (oneDNN, AMX where the host has it) on the
    sweep's own ATen graph, with every host thread.  A step runs the first
    `rows` rows of each of the twelve sweep GEMMs (the 512^3 points whole);
    the value is the sampled FLOPs / median step time.  Without the reference
    install the same blocks run eagerly (kind "port").  With `models`, the
    MLP, ViT-B/16 and Llama-style forwards on the host cores are added
    (run_models_cpu)."""
    from bench_models import GemmEpilogueBlock, init_sweep_block

    threads = _host_threads()
    backend, kind = None, "port"
    try:
        _use_reference_triton()
        from compiler.backend import custom_backend as backend  # the reference's package

        kind = "reference"
    except Exception as e:  # noqa: BLE001 -- recorded in the line
        print(f"reference backend unavailable ({e}); timing eager PyTorch", file=sys.stderr)
    torch._dynamo.config.recompile_limit = max(torch._dynamo.config.recompile_limit, 64)
    gen = torch.Generator().manual_seed(0)
    work = []
    for (M, N, K) in SWEEP:
        m = min(rows, M)
        x = (0.02 * torch.randn(m, K, generator=gen)).to(torch.bfloat16)
        r = (0.02 * torch.randn(m, N, generator=gen)).to(torch.bfloat16)
        for act in ACTS:
            blk = GemmEpilogueBlock(K, N, act)
            init_sweep_block(blk, torch.Generator().manual_seed(len(work)))
            blk = blk.to(torch.bfloat16).eval()
            f = torch.compile(blk, backend=backend) if backend is not None else blk
            work.append((f, x, r, 2.0 * m * N * K))
    times = []
    with torch.no_grad():
        for _ in range(max(1, warmup)):
            for f, x, r, _ in work:
                f(x, r)
        for _ in range(max(1, steps)):
            t0 = time.perf_counter()
            for f, x, r, _ in work:
                f(x, r)
            times.append(time.perf_counter() - t0)
    flops = sum(w[3] for w in work)
    med = statistics.median(times)
    res = {"value": round(flops / med / 1e12, 4), "unit": "TFLOP/s", "cores": threads, "kind": kind,
           "sample": f"first {rows} rows of each of the 12 sweep GEMMs (512^3 whole), bf16, "
                     f"median of {len(times)} steps of {med * 1e3:.0f} ms; reference backend on CPU = "
                     "eager ATen graph", "ms_per_step": round(med * 1e3, 2)}
    if models:
        try:
            res["models"] = run_models_cpu()
        except Exception as e:  # noqa: BLE001 -- recorded in the line
            res["models"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    return res


def _median_s(fn, reps: int, warm: int) -> float:
    for _ in range(warm):
        fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts)


def _fill_cpu(model: torch.nn.Module) -> torch.nn.Module:
    """Materialises a meta-device model on the CPU in bf16: matrices and
    embeddings tile one seeded N(0, 0.02) block, vectors are ones (norm
    weights) or the same block (biases)."""
    model = model.to_empty(device="cpu").to(torch.bfloat16)
    block = (0.02 * torch.randn(1 << 20, generator=torch.Generator().manual_seed(0))).to(torch.bfloat16)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 1 and name.endswith("weight"):
                p.fill_(1.0)
                continue
            flat = p.view(-1)
            for i in range(0, flat.numel(), block.numel()):
                n = min(block.numel(), flat.numel() - i)
                flat[i:i + n].copy_(block[:n])
    return model


def run_models_cpu() -> dict:
    """The benchmark's models forward on the host cores: the eager graph,
    i.e. the ATen ops the reference backend leaves unfused on CPU (its passes
    need CUDA values), run without the compile step to keep the leg short.
    The MLP runs at its full configuration (x[64,1024] fp32, median of 20);
    ViT-B/16 on 2 of the 64 images and the Llama-style prefill on one
    256-token sequence (bf16, median of 3): tokens/s of those samples."""
    import bench_models as bm

    out = {}
    with torch.no_grad():
        torch.manual_seed(0)
        mlp = bm.MLP().eval()
        x = torch.randn(64, 1024, generator=torch.Generator().manual_seed(0))
        t = _median_s(lambda: mlp(x), 20, 3)
        out["mlp"] = {"ms": round(t * 1e3, 3), "rows_per_s": round(64 / t, 1),
                      "tflops": round(bm.mlp_flops() / t / 1e12, 4), "sample": "full config, fp32"}
        # The big models are built on the meta device and filled by tiling one
        # seeded N(0, 0.02) block: drawing 1.5e9 values one by one takes minutes
        # on the host, and the timing does not depend on the values.
        with torch.device("meta"):
            vit, llama = bm.ViT(), bm.Llama()
        vit, llama = _fill_cpu(vit), _fill_cpu(llama)
        llama.reset_rope()
        vit.eval()
        img = torch.randn(2, 3, 224, 224, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
        t = _median_s(lambda: vit(img), 3, 1)
        out["vit"] = {"ms": round(t * 1e3, 2), "tokens_per_s": round(2 * 197 / t, 1),
                      "tflops": round(2 * bm.vit_flops_per_image() / t / 1e12, 4), "sample": "batch 2 of 64, bf16"}
        del vit
        llama.eval()
        ids = torch.randint(0, 128256, (1, 256), generator=torch.Generator().manual_seed(0))
        t = _median_s(lambda: llama(ids), 3, 1)
        out["llama"] = {"ms": round(t * 1e3, 1), "tokens_per_s": round(256 / t, 1),
                        "tflops": round(bm.llama_flops_per_token(seq=256) * 256 / t / 1e12, 4),
                        "sample": "1 sequence x 256 tokens of 8 x 2048, bf16"}
    return out


def _cpu_baseline_subprocess(rows: int) -> dict | None:
    """run_reference_cpu in a process of its own (the reference's package is
    also named `compiler`), with no GPU visible."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT", "OMP_NUM_THREADS"):
        env.pop(k, None)
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "3", "--warmup", "1",
           "--cpu-rows", str(rows)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
        line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1]
        return json.loads(line)["cpu_baseline"]
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unavailable": f"{type(e).__name__}: {e}"[:300]}


# --------------------------------------------------------------- model extras
def _reference_triton_model(workload: str, batch: int, steps: int, warmup: int) -> dict:
    """--workload vit|llama through the reference Triton backend, in a process
    of its own; its JSON line, or the error it stopped with."""
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--workload", workload, "--backend", "reference_triton",
           "--batch", str(batch), "--steps", str(steps), "--warmup", str(warmup)]
    env = dict(os.environ)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    except subprocess.TimeoutExpired:
        return {"unavailable": "timed out after 900 s"}
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode == 0 and lines:
        d = json.loads(lines[-1])
        return {"tokens_per_s": d["value"], "ms": d["ms_per_step"], "compile_s": d.get("compile_s")}
    err = [ln for ln in r.stderr.splitlines() if "Error" in ln or "error" in ln]
    return {"unavailable": (err[-1] if err else f"exit code {r.returncode}")[:300]}


def run_model_extras(args, dist: Dist) -> dict:
    """ViT-B/16 (batch 64) and the Llama-style prefill (8 x 2048) forward,
    split by batch over the N GPUs (64/N images, 8/N sequences per GPU;
    strong scaling), this backend and eager PyTorch on each GPU; tokens/s =
    all ranks' tokens / the slowest rank's median step.  At N = 1 the
    reference Triton backend runs the same configs in a subprocess."""
    out = {}
    for wl, full in (("vit", 64), ("llama", 8)):
        per = max(1, full // dist.world)
        res = {"batch_per_gpu": per, "global_batch": per * dist.world}
        for be in ("ours", "eager"):
            ns = argparse.Namespace(workload=wl, backend=be, batch=per, steps=args.model_steps,
                                    warmup=max(3, args.warmup))
            torch._dynamo.reset()
            dist.barrier()
            d = run_model(ns, dist)
            ms = dist.max(d["ms_per_step"])
            tokens = d["config"]["tokens"] * dist.world
            res[be] = {"tokens_per_s": round(tokens / (ms * 1e-3), 1), "ms": round(ms, 3),
                       "tflops": round(d["tflops"] * dist.world * d["ms_per_step"] / ms, 1)}
            if be == "ours":
                from compiler import runtime

                runtime.check_status(dist.local)
        if dist.world == 1 and args.reference_models:
            res["reference_triton"] = _reference_triton_model(wl, per, args.model_steps, max(3, args.warmup))
        out[wl] = res
    torch._dynamo.reset()
    return out


def run_chain_extra(args, dist: Dist) -> dict:
    ns = argparse.Namespace(workload="chain", backend="ours", steps=args.model_steps, warmup=max(3, args.warmup))
    torch._dynamo.reset()
    d = run_chain(ns, dist)
    return {"GB/s": d["value"], "frac": d["roofline"]["frac"], "kernels": d["kernels"]}


def bind_to_gpu_numa(local: int) -> list[int] | None:
    """Restrict this rank to the host CPUs local to its GPU (sysfs
    local_cpulist of the GPU's PCI device), so that its pinned host buffers
    are first touched on the GPU's own NUMA node.  Returns the CPUs, or None
    when the topology is not readable."""
    try:
        prop = torch.cuda.get_device_properties(local)
        bus = f"{prop.pci_domain_id:04x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/local_cpulist") as f:
            spec = f.read().strip()
        cpus = []
        for part in spec.split(","):
            a, _, b = part.partition("-")
            cpus.extend(range(int(a), int(b or a) + 1))
        if cpus:
            os.sched_setaffinity(0, cpus)
            return cpus
    except (OSError, ValueError, AttributeError):
        pass
    return None


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="sweep",
                    choices=["sweep", "gemm", "vit", "llama", "chain", "pointwise", "attention"])
    ap.add_argument("--backend", default="ours", choices=["ours", "eager", "reference_triton", "inductor"],
                    help="sweep/vit/llama/chain workloads: which torch.compile backend runs the model")
    ap.add_argument("--batch", type=int, default=0, help="vit/llama batch (default: the benchmark config)")
    ap.add_argument("--shape", default="4096,4096,4096", help="M,N,K for --workload gemm")
    ap.add_argument("--act", default="gelu", choices=ACTS, help="epilogue activation for --workload gemm")
    ap.add_argument("--tile-config", type=int, default=-1, help="force a GEMM tile config (gemm workload)")
    ap.add_argument("--interpret", action="store_true", help="gemm workload: interpret the epilogue program")
    ap.add_argument("--plain", action="store_true",
                    help="gemm workload: out = x w^T with no epilogue, against torch.mm in the eager leg")
    ap.add_argument("--cpu-rows", type=int, default=1024, help="rows of each sweep GEMM the CPU leg runs")
    ap.add_argument("--model-steps", type=int, default=10, help="timed steps of each model extra")
    ap.add_argument("--no-cpu-models", dest="cpu_models", action="store_false",
                    help="reference arm: skip the MLP / ViT / Llama forward on the host cores")
    ap.add_argument("--no-extras", action="store_true",
                    help="sweep only: skip the ViT/Llama/chain extras and the CPU baseline")
    ap.add_argument("--no-reference-models", dest="reference_models", action="store_false",
                    help="skip the reference Triton backend's ViT/Llama runs in the extras")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)

    dist_env_rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if dist_env_rank != 0:
            return
        base = run_reference_cpu(args.steps, args.warmup, args.cpu_rows, args.cpu_models)
        line = {"impl": "reference", "metric": "fused GEMM+epilogue TFLOP/s", "value": base["value"],
                "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": base["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,0.02) X/W/R, N(0,0.01) b)",
                "config": {"workload": "gemm_epilogue_sweep", "shapes": SWEEP, "acts": ACTS,
                           "epilogue": "act(X W^T + b) + R, bf16 in/out", "sample_rows": args.cpu_rows},
                "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample", "models")
                                 if k in base},
                "e2e": {"value": base["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    dist = Dist()
    try:
        cpus = bind_to_gpu_numa(dist.local) if torch.cuda.is_available() else None
        if args.workload == "gemm":
            print(json.dumps(run_single_gemm(args, dist)))
            return
        if args.workload in ("vit", "llama"):
            print(json.dumps(run_model(args, dist)))
            return
        if args.workload == "chain":
            print(json.dumps(run_chain(args, dist)))
            return
        if args.workload == "pointwise":
            print(json.dumps(run_pointwise(args, dist)))
            return
        if args.workload == "attention":
            print(json.dumps(run_attention(args, dist)))
            return
        if args.backend != "ours":
            print(json.dumps(run_sweep_backend(args, dist)))
            return
        res = run_sweep(args, dist)
        res["host_cpus_bound"] = len(cpus) if cpus else None
        if not args.no_extras:
            res["models"] = run_model_extras(args, dist)
            res["chain"] = run_chain_extra(args, dist)
            if dist.world == 1 and args.reference_models:
                res["sweep_reference_triton"] = _reference_triton_sweep(args.model_steps, max(3, args.warmup))
        if dist.rank == 0:
            if dist.world == 1 and not args.no_extras:
                res["cpu_baseline"] = _cpu_baseline_subprocess(args.cpu_rows)
            print(json.dumps(res))
    finally:
        dist.close()


if __name__ == "__main__":
    main()
