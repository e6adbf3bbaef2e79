"""The multi-process side of bench.py on CPU: world size 2 over gloo.

With N > 1 the bench runs one replica per GPU (bs1 Qwen2 does not shard: its
all-gathers would be latency-bound, so the decode is replicated), takes the
slowest rank's device time for the whole job and reports world x tokens per
rank / that time.  Here two gloo ranks with different timings check that every
rank gets the same maximum, and that the reference arm runs on rank 0 only.
"""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, queue):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        secs = bench.max_over_ranks(dist, 0.5 + rank, "cpu")  # rank 1 is the slow one
        e2e = bench.max_over_ranks(dist, 2.0 - rank, "cpu")   # rank 0 is the slow one
        queue.put((rank, secs, e2e, bench.job_throughput(world, 128, 20, secs)))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_job_throughput_gloo_world_2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(queue.get(timeout=10) for _ in range(2))
    for rank, secs, e2e, value in got:
        assert secs == 1.5 and e2e == 2.0, (rank, secs, e2e)
        assert value == pytest.approx(2 * 128 * 20 / 1.5)


def test_single_process_needs_no_process_group():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks(None, 0.25, "cpu") == 0.25
    assert bench.job_throughput(1, 128, 20, 2.0) == 1280.0


def test_reference_arm_runs_on_rank_zero_only():
    """A non-zero rank of the reference arm exits 0 without work or output."""
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


@pytest.mark.slow
def test_reference_arm_line_on_rank_zero():
    """Rank 0 of the reference arm prints one JSON line (reference CPU path,
    or the unavailable line when the harness is not built)."""
    env = dict(os.environ, RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    if "unavailable" not in line:
        assert line["metric"].startswith("decode tok/s") and line["value"] > 0
        assert line["e2e"]["h2d_bytes_per_step"] == 0
        # the same workload description as the repo arm's line
        sys.path.insert(0, ROOT)
        import bench
        assert line["config"] == bench.config_for(1)
        assert "positions 68..71" in line["cpu_baseline"]["sample"]  # after one warm-up step
