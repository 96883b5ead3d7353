"""The bench's multi-process path on CPU (gloo, world size 2): the replica
harness exchanges only a barrier and the max-over-ranks time, and under
torchrun only rank 0 prints the result line."""
import json
import os
import socket
import subprocess
import sys

import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import bench

    d = bench.Dist()
    try:
        d.barrier()
        q.put((rank, d.max(float(10 * rank + 1))))
        d.barrier()
    finally:
        d.close()


def test_dist_barrier_and_max_over_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    assert got == [(0, 11.0), (1, 11.0)]  # every rank sees the slowest rank's time


def test_reference_arm_under_torchrun_prints_once():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0",
           "--cpu-rows", "4", "--no-cpu-models"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [line for line in r.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["unit"] == "TFLOP/s"
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["e2e"]["h2d_bytes_per_step"] == 0
    # torchrun pins OMP_NUM_THREADS=1; the CPU leg uses every host thread anyway
    assert d["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))


def test_cpu_model_baselines():
    """The reference arm's model leg: the MLP config and the ViT / Llama
    samples run forward on the host cores and report tokens/s."""
    sys.path.insert(0, ROOT)
    import bench

    d = bench.run_models_cpu()
    assert d["mlp"]["rows_per_s"] > 0 and "full config" in d["mlp"]["sample"]
    assert d["vit"]["tokens_per_s"] > 0 and d["llama"]["tokens_per_s"] > 0
    assert all(0 < d[k]["tflops"] < 100 for k in ("mlp", "vit", "llama"))
