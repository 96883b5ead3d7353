"""Benchmark: fused GEMM + epilogue sweep on B200 (the headline workload).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload sweep|gemm|chain|vit|llama] [--backend ours|eager|reference_triton|inductor]

One step of the default workload ("gemm_epilogue_sweep") runs the fused bf16
GEMM sweep once: Y = act(X W^T + b) + R for act in {none, gelu, silu} and
(M, N, K) in {512^3, 4096^3, 8192^3, (16384, 4096, 14336)} -- twelve launches
of the library's tcgen05 GEMM kernel with the epilogue fused.  `value` is the
sweep's total FLOPs (2MNK per GEMM) / device time, inputs resident in HBM.
`e2e` is the same metric through the public API (torch.compile with
custom_backend) with X and R copied in from pinned host memory and Y copied
back inside the timed region; the copies run on two copy streams, so one
GEMM's transfers overlap its neighbours' compute.

Multi-GPU: one process per GPU (torchrun), each GPU runs the full sweep as an
independent replica (weak scaling, no data-path collective); a gloo process
group carries only the barrier and the max-over-ranks time.

--impl reference times the CPU implementation of the same path on the host
cores: the oracle restatement of the reference kernels' arithmetic (numpy
fp32 GEMM + epilogue), on a bounded row sample of every sweep GEMM.
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


# Kernel and ncu summary (profiles/<name>.md) per tile config of the dominant launch.
_DOMINANT_KERNELS = {3: ("gemm_pair_kernel 256x256", "gemm_pair_16384x4096x14336_gelu"),
                     4: ("gemm_pair_kernel 256x512", "gemm_pair_wide_16384x4096x14336_gelu")}


def _dominant_kernel() -> tuple[str, str | None]:
    """The kernel the library picks for the sweep's dominant launch and the
    name of its ncu summary under profiles/ (None when there is none)."""
    from compiler.runtime import cabi

    cfg = cabi.library().b200k_gemm_pick_config(*DOMINANT)
    return _DOMINANT_KERNELS.get(cfg, ("gemm_epilogue_kernel", None))


def profile_traffic(name: str):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name>.md
    (line 'dram_bytes_per_launch: <int>'), or None."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


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
    # send the last blocks to eager PyTorch.  Raise it for this run and make
    # hitting it an error, so every e2e call goes through the backend.
    torch._dynamo.reset()
    torch._dynamo.config.recompile_limit = max(torch._dynamo.config.recompile_limit, 4 * len(probs))
    torch._dynamo.config.fail_on_recompile_limit_hit = True
    compiled = [torch.compile(p["block"], backend=custom_backend) for p in probs]
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

    graphs0 = _backend.GRAPHS_COMPILED
    for _ in range(max(1, args.warmup)):
        e2e_step()
    compute.wait_stream(down)
    e2e_graphs = _backend.GRAPHS_COMPILED - graphs0
    if e2e_graphs < len(probs):
        raise RuntimeError(f"only {e2e_graphs} of {len(probs)} e2e blocks compiled through the backend")
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
    peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
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
                   "parallelism": f"replicas x{n}"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 3), "peak_source": f"{src} bf16_tflops_sustained",
                     "frac_of_burst": round(achieved / peaks["bf16_tflops"], 3),
                     "kernel": _dominant_kernel()[0] + " 16384x4096x14336 gelu",
                     "traffic": profile_traffic(_dominant_kernel()[1]) if _dominant_kernel()[1] else None},
        "e2e": {"value": round(n * flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
                "graphs_compiled": e2e_graphs},
        "gpu_launches": args.steps * len(probs),
        "clocks": clk.summary(),
        "sweep": sweep_detail,
        "epilogue_paths": sorted({"compiled" if p["form"] else "interpreted" for p in probs}),
        "spot_check_max_rel_err": round(err, 5),
    }


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


def _time_device(fn, steps: int, warmup: int, flush=None) -> list[float]:
    """Device time of each of `steps` calls (CUDA events on the current
    stream around the call, an L2 flush between calls).  The steps are queued
    back to back and synchronised once at the end, so the host's per-call
    cost overlaps the device's work, as in a running model."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = []
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
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


# --------------------------------------------------------------- CPU (oracle) leg
def cpu_sweep(rows: int, reps: int) -> dict:
    """The oracle's GEMM + epilogue (numpy fp32, every host core via BLAS) on
    the first `rows` rows of every sweep GEMM."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(0)
    gelu = [["mul.Tensor", [["acc"], 0.5]], ["mul.Tensor", [["acc"], 0.7071067811865476]],
            ["erf.default", [["node", 1]]], ["add.Tensor", [["node", 2], 1.0]],
            ["mul.Tensor", [["node", 0], ["node", 3]]]]
    silu = [["sigmoid.default", [["acc"]]], ["mul.Tensor", [["acc"], ["node", 0]]]]
    work = []
    for (M, N, K) in SWEEP:
        m = min(rows, M)
        x = oracle.round_bf16((0.02 * rng.standard_normal((m, K))).astype(np.float32))
        w = oracle.round_bf16((0.02 * rng.standard_normal((K, N))).astype(np.float32))
        b = oracle.round_bf16((0.01 * rng.standard_normal(N)).astype(np.float32))
        r = oracle.round_bf16((0.02 * rng.standard_normal((m, N))).astype(np.float32))
        for act, spec in (("none", []), ("gelu", gelu), ("silu", silu)):
            s = list(spec) + [["add.Tensor", [["node", len(spec) - 1] if spec else ["acc"], ["in", 1]]]]
            work.append((x, w, b, r, s, 2.0 * m * N * K))
    t0 = time.perf_counter()
    for _ in range(reps):
        for x, w, b, r, s, _ in work:
            oracle.gemm_epilogue(x, w, s, [b, r], "bfloat16", bias=b)
    dt = time.perf_counter() - t0
    flops = reps * sum(f for *_, f in work)
    return {"value": round(flops / dt / 1e12, 4), "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"first {rows} rows of each of the 12 sweep GEMMs, x{reps}; {dt:.1f} s",
            "seconds": round(dt, 2)}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="sweep", choices=["sweep", "gemm", "vit", "llama", "chain", "pointwise"])
    ap.add_argument("--backend", default="ours", choices=["ours", "eager", "reference_triton", "inductor"],
                    help="vit/llama/chain workloads: which torch.compile backend runs the model")
    ap.add_argument("--batch", type=int, default=0, help="vit/llama batch (default: the benchmark config)")
    ap.add_argument("--shape", default="4096,4096,4096", help="M,N,K for --workload gemm")
    ap.add_argument("--act", default="gelu", choices=ACTS, help="epilogue activation for --workload gemm")
    ap.add_argument("--tile-config", type=int, default=-1, help="force a GEMM tile config (gemm workload)")
    ap.add_argument("--interpret", action="store_true", help="gemm workload: interpret the epilogue program")
    ap.add_argument("--plain", action="store_true",
                    help="gemm workload: out = x w^T with no epilogue, against torch.mm in the eager leg")
    ap.add_argument("--cpu-rows", type=int, default=256)
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)

    dist_env_rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if dist_env_rank != 0:
            return
        base = cpu_sweep(args.cpu_rows, max(1, args.steps // 5))
        line = {"impl": "reference", "metric": "fused GEMM+epilogue TFLOP/s", "value": base["value"],
                "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic", "config": {"workload": "gemm_epilogue_sweep", "shapes": SWEEP, "acts": ACTS},
                "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": base["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    dist = Dist()
    try:
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
        res = run_sweep(args, dist)
        if dist.rank == 0:
            if dist.world == 1:
                base = cpu_sweep(args.cpu_rows, 1)
                res["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
            print(json.dumps(res))
    finally:
        dist.close()


if __name__ == "__main__":
    main()
