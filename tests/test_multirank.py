"""The multi-GPU host logic on CPU, two `gloo` ranks in spawned processes.

The benchmark partitions the batched encoder by rank with no collective on
the data path: every rank draws its own 64 segments (seed + rank) and runs
them on its own GPU; the job's figures come from one reduction at the end,
the time as the max over ranks and the work (int8 ops, audio seconds) as the
sum. These tests run exactly that host code (bench.segments, bench.products,
bench.job_totals) with the gloo backend on 127.0.0.1.
"""
from __future__ import annotations

import datetime
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, queue) -> None:
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        segs = bench.segments(rank)
        prods = bench.products(segs)
        ops = bench.step_ops(prods)
        audio = bench.audio_seconds(segs)
        ms = 10.0 + 3.0 * rank  # a stand-in per-rank step time
        totals = bench.job_totals(dist, torch.device("cpu"), ms, ops, audio)
        queue.put({"rank": rank, "ops": ops, "audio": audio, "ms": ms, "totals": totals,
                   "frames": [s[3] for s in segs]})
    finally:
        dist.destroy_process_group()


def _run(world: int) -> list[dict]:
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    out = [queue.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out, key=lambda r: r["rank"])


@pytest.fixture(scope="module")
def two_ranks() -> list[dict]:
    return _run(2)


def test_each_rank_its_own_segments(two_ranks):
    a, b = two_ranks
    assert len(a["frames"]) == bench.SEGMENTS and len(b["frames"]) == bench.SEGMENTS
    assert a["frames"] != b["frames"]
    # the draw is the rank's alone: the same rank draws the same segments again
    assert [s[3] for s in bench.segments(1)] == b["frames"]
    # encoder frames 25..375 a segment (2..30 s at 80 ms)
    assert all(25 <= f <= 376 for f in a["frames"] + b["frames"])


def test_job_totals_max_time_sum_work(two_ranks):
    a, b = two_ranks
    want = (max(a["ms"], b["ms"]), a["ops"] + b["ops"], a["audio"] + b["audio"])
    for r in two_ranks:
        ms, ops, audio = r["totals"]
        assert ms == pytest.approx(want[0])
        assert ops == pytest.approx(want[1], rel=1e-12)
        assert audio == pytest.approx(want[2], rel=1e-12)
    # the per-rank work differs, so rank 0's times the world size is not the job's
    assert a["ops"] != b["ops"]


def test_job_totals_alone():
    segs = bench.segments(0)
    ops, audio = bench.step_ops(bench.products(segs)), bench.audio_seconds(segs)
    assert bench.job_totals(None, None, 7.5, ops, audio) == (7.5, ops, audio)
