"""The N>1 host logic of bench.py on CPU: two gloo ranks exercise the rank
slice and the max-over-ranks timing reduction, and the reference arm is run
under torchrun with two ranks (rank 0 alone measures and prints)."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, str(ROOT))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    base = bench.rank_index_base(rank, 1000)
    slowest = bench.max_over_ranks(1.5 * (rank + 1), world)
    out.put((rank, base, slowest))
    dist.destroy_process_group()


def test_two_gloo_ranks_slice_and_max_reduction():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == [(0, 0, 3.0), (1, 1000, 3.0)]


def test_max_over_ranks_single_process_is_identity():
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.max_over_ranks(2.5, 1) == 2.5


def test_reference_arm_two_ranks_under_torchrun():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), "bench.py",
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3",
           "--workload", "c1", "--cpu-rows", "2"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.splitlines()
    assert len(lines) == 1 and lines[0].startswith("{"), r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_library_output_on_fd1_goes_to_stderr():
    """A banner a library writes straight to file descriptor 1 (as NCCL does
    with its version line) must not reach stdout, which holds only the JSON
    result line."""
    code = ("import os, sys; sys.path.insert(0, '.'); import bench; bench.claim_stdout(); "
            "os.write(1, b'NCCL version banner\\n'); print('stray print'); "
            "bench.emit({'value': 1.0})")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.splitlines() == ['{"value": 1.0}'], r.stdout
    assert "NCCL version banner" in r.stderr and "stray print" in r.stderr
