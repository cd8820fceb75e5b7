"""The multi-GPU host logic on CPU, two `gloo` ranks in spawned processes.

The benchmark partitions the batched encoder by rank with no collective on
the data path: the batch of 64 segments is dealt across the ranks longest
first (strong scaling; with weak scaling every rank takes the whole batch) and
each rank runs its share on its own GPU; the job's figures come from one
reduction at the end, the time as the max over ranks and the work (int8
ops, audio seconds) as the sum. These tests run exactly that host code
(bench.segments, bench.partition, bench.products, bench.job_totals) with
the gloo backend on 127.0.0.1.
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


def _rank_main(rank: int, world: int, port: int, queue, scaling: str = "strong") -> None:
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        segs = bench.segments(rank, world, scaling)
        prods = bench.products(segs)
        ops = bench.step_ops(prods)
        audio = bench.audio_seconds(segs)
        ms = 10.0 + 3.0 * rank  # a stand-in per-rank step time
        totals = bench.job_totals(dist, torch.device("cpu"), ms, ops, audio)
        queue.put({"rank": rank, "ops": ops, "audio": audio, "ms": ms, "totals": totals,
                   "frames": [s[3] for s in segs]})
    finally:
        dist.destroy_process_group()


def _run(world: int, scaling: str = "strong") -> list[dict]:
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue, scaling)) for r in range(world)]
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


@pytest.fixture(scope="module")
def two_ranks_weak() -> list[dict]:
    return _run(2, "weak")


def test_strong_scaling_deals_the_one_batch(two_ranks):
    a, b = two_ranks
    whole = [s[3] for s in bench.draw_segments(bench.SEED)]
    # the two shares together are the batch, each segment once
    assert sorted(a["frames"] + b["frames"]) == sorted(whole)
    assert len(a["frames"]) + len(b["frames"]) == bench.SEGMENTS
    # longest first to the lighter rank: the loads differ by at most one segment
    assert abs(sum(a["frames"]) - sum(b["frames"])) <= max(whole)
    # encoder frames 25..375 a segment (2..30 s at 80 ms)
    assert all(25 <= f <= 376 for f in whole)


def test_partition_at_every_width():
    segs = bench.draw_segments(bench.SEED)
    for world in (1, 2, 4, 8):
        shares = bench.partition(segs, world)
        assert sorted(i for s in shares for i in s) == list(range(bench.SEGMENTS))
        loads = [sum(segs[i][3] for i in s) for s in shares]
        assert max(loads) - min(loads) <= max(s[3] for s in segs)


def test_weak_scaling_every_rank_the_whole_batch(two_ranks_weak):
    a, b = two_ranks_weak
    assert len(a["frames"]) == bench.SEGMENTS and len(b["frames"]) == bench.SEGMENTS
    # every GPU the same batch: the work a GPU is the same at every world size
    assert a["frames"] == b["frames"] == [s[3] for s in bench.draw_segments(bench.SEED)]
    assert a["ops"] == b["ops"]
    # and the job's work is the world size times one batch's
    one = bench.step_ops(bench.products(bench.draw_segments(bench.SEED)))
    assert a["totals"][1] == pytest.approx(2 * one, rel=1e-12)


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
    # strong scaling: the job's work is the whole batch's
    whole = bench.step_ops(bench.products(bench.draw_segments(bench.SEED)))
    assert a["totals"][1] == pytest.approx(whole, rel=1e-12)


def test_job_totals_alone():
    segs = bench.segments(0)
    ops, audio = bench.step_ops(bench.products(segs)), bench.audio_seconds(segs)
    assert bench.job_totals(None, None, 7.5, ops, audio) == (7.5, ops, audio)
