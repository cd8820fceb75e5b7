"""The long-form workload's chunks: the committed
fixture is what the reference's own segmenter and chunker give for the
seeded hour, and the chunks the benchmark deals across GPUs are theirs."""
import json
import os

import pytest

from tests.golden import make_longform as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _doc():
    with open(L.OUT) as f:
        return json.load(f)


def test_chunks_tile_the_hour_and_fit_a_chunk():
    doc = _doc()
    c = doc["chunks"]
    assert c[0][0] == 0 and c[-1][1] == doc["seconds"] * doc["rate"]
    assert all(a[1] == b[0] for a, b in zip(c, c[1:]))
    assert all(0 < b - a <= doc["max_chunk_s"] * doc["rate"] for a, b in c)


@pytest.mark.skipif(not os.path.exists(L.CORE), reason="the reference's core is not built (make -C oracle ref)")
def test_fixture_is_the_references_cut():
    x, runs = L.recording()
    segs, chunks = L.cut(x, L.probabilities(runs, x.size))
    doc = _doc()
    assert doc["segments"] == len(segs)
    assert doc["chunks"] == [[int(a), int(b)] for a, b in chunks]


def test_benchmark_deals_every_chunk_once():
    import bench
    chunks = bench.longform_chunks()
    assert len(chunks) == len(_doc()["chunks"])
    for world in (1, 2, 4, 8):
        parts = bench.partition(chunks, world)
        assert sorted(i for p in parts for i in p) == list(range(len(chunks)))
        loads = [sum(chunks[i][3] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(c[3] for c in chunks)
