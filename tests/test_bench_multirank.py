"""CPU: the multi-rank logic of bench.py under two gloo ranks (no GPU).

bench.py runs one process per GPU; each rank decodes its own replica and the
reported time is the maximum over ranks, the value the whole-job token rate.
These tests run that reduction on two CPU ranks, and the reference arm under
torchrun with two ranks: rank 0 alone prints one JSON line, rank 1 exits 0.
"""
import json
import os
import socket
import subprocess
import sys

import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    per_rank_ms = [12.5, 20.0][rank]
    t_max = bench.max_over_ranks(per_rank_ms, dist, "cpu")
    out[rank] = (t_max, bench.aggregate_tok_s(world, 64 * 10, t_max / 1000.0))
    dist.barrier()
    dist.destroy_process_group()


def test_max_over_ranks_and_aggregate_gloo():
    world, port = 2, _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    assert res[0] == res[1]                      # every rank sees the same maximum
    t_max, value = res[0]
    assert t_max == 20.0
    assert abs(value - 2 * 640 / 0.020) < 1e-6   # all ranks' tokens over the slowest rank's time


def test_max_over_ranks_single_process():
    import bench
    assert bench.max_over_ranks(3.5, None) == 3.5


def test_reference_arm_two_ranks_prints_once():
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"),
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0", "--ref-sample-steps", "1"]
    env = dict(os.environ, OMP_NUM_THREADS="2")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"
