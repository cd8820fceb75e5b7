"""TDT's greedy search on the GPU (pkb_tdt_search_dev), the batch's segments
in lockstep, against the reference's own tokens and the oracle.

* The reference's tiny model (tests/golden/tdt_golden.npz, written by the
  reference's pk_decode through oracle/_ref/tdt_ref): all seven of its cases
  as one batch of segments of 1 to 400 frames, each segment's tokens the
  reference's: blanks that skip frames, durations 0 to 3, several tokens at
  one frame up to max_symbols, a one-frame segment, a segment of none.
* The model's real shapes (pred_hidden 640, joint 640, a vocabulary of 1,024
  here to keep the oracle's search fast, 5 durations) with seeded weights:
  a batch of 6 segments against the oracle's search, in two rounding modes.
* The token capacity: a segment that finds more tokens than the room given
  makes the call fail.
* Both ways the search runs: one cooperative launch for the whole search
  (the cases above, and a batch of 200 segments, its products' columns
  taken 64 at a time), and the rounds' launches replayed as a CUDA graph
  where the model's shapes do not fit the one launch's shared memory
  (pred_hidden 2048).
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden import make_tdt_golden as G

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "tdt_golden.npz")


def dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.cuda()


def device_model(pkb, m: dict):
    """The decoder's weights on the device: PK_Q8 matrices repacked to rows."""
    import torch
    P, L, J, nop = m["P"], m["L"], m["J"], m["n_out_pad"]
    keep = []

    def put(a):
        t = dev(a)
        keep.append(t)
        return t.data_ptr()

    def q8(w_pk, rows, n):
        src = dev(w_pk)
        out = torch.empty(rows * n, dtype=torch.int8, device="cuda")
        pkb.repack_q8_dev(out, src, rows, n)
        keep.extend([src, out])
        return out.data_ptr()

    t = pkb.TdtModel()
    t.P, t.L, t.J, t.V, t.n_dur, t.max_symbols, t.n_out_pad = P, L, J, m["V"], m["n_dur"], m["max_symbols"], nop
    for i, d in enumerate(m["dur"]):
        t.dur[i] = int(d)
    t.embed = put(m["embed"])
    for l in range(L):
        t.wx[l] = q8(m["wx"][l * 4 * P * P:(l + 1) * 4 * P * P], 4 * P, P)
        t.wh[l] = q8(m["wh"][l * 4 * P * P:(l + 1) * 4 * P * P], 4 * P, P)
        t.wxs[l] = put(m["wxs"][l * 4 * P:(l + 1) * 4 * P])
        t.whs[l] = put(m["whs"][l * 4 * P:(l + 1) * 4 * P])
        t.lb[l] = put(m["lb"][l * 4 * P:(l + 1) * 4 * P])
    t.jpred, t.jpreds, t.jpredb = q8(m["jpred"], J, P), put(m["jpreds"]), put(m["jpredb"])
    t.jout, t.jouts, t.joutb = q8(m["jout"], nop, J), put(m["jouts"]), put(m["joutb"])
    torch.cuda.synchronize()
    return t, keep


def search(pkb, t, frames: list, cap: int, rmode: int = O.RN):
    """The batch's segments (lists of [T][J] frames) through the device search:
    each segment's tokens as rows of (id, frame, duration)."""
    import torch
    J = t.J
    Ts = np.array([len(f) // J for f in frames], np.uint32)
    f0 = np.concatenate([[0], np.cumsum(Ts)[:-1]]).astype(np.uint32)
    f = dev(np.concatenate([np.asarray(x, np.float32) for x in frames] + [np.zeros(J, np.float32)]))
    S = len(frames)
    toks = torch.full((S * cap * 3,), -7, dtype=torch.int32, device="cuda")
    ntok = torch.zeros(S, dtype=torch.int32, device="cuda")
    work = torch.empty(pkb.tdt_work_bytes(t, S) // 4 + 64, dtype=torch.float32, device="cuda")
    pkb.tdt_search_dev(t, f, f0, Ts, toks, ntok, cap, work, rmode)
    torch.cuda.synchronize()
    tk = toks.view(S, cap, 3).cpu().numpy()
    n = ntok.cpu().numpy()
    return [tk[s, :n[s]] for s in range(S)]


def golden_model():
    g = np.load(GOLDEN)
    return g, G.model(g)


def test_the_references_tokens_on_its_tiny_model(pkb, cuda_device):
    g, m = golden_model()
    t, keep = device_model(pkb, m)
    frames, want = [], []
    for i, (T, seed, scale) in enumerate(G.CASES):
        frames.append(G.frames(T, m["J"], seed, float(g[f"case/{i}/scale"][0])))
        want.append(g[f"case/{i}/toks"])
    frames.append(np.zeros(0, np.float32))  # a segment of no frames: no tokens
    want.append(np.zeros((0, 3), np.int32))
    got = search(pkb, t, frames, cap=2048)
    for (T, seed, _), a, b in zip(G.CASES + [(0, 0, 0)], got, want):
        assert a.shape == b.shape and (a == b).all(), (T, seed)


def synthetic_model(P=640, J=640, V=1024, L=2, n_dur=5, seed=3):
    """The model's shapes with seeded weights (PK_Q8 bytes uniform, scales
    and biases in the ranges the real model's have)."""
    g = np.random.default_rng(seed)
    nop = (V + 1 + n_dur + 15) // 16 * 16

    def q8(rows, n):
        return O.pack_q8(g.integers(-127, 128, (rows, n), dtype=np.int8))

    def sc(n, lo=2e-3, hi=2e-2):
        return (lo + (hi - lo) * g.random(n)).astype(np.float32)
    m = dict(P=P, L=L, J=J, V=V, n_dur=n_dur, max_symbols=10, n_out_pad=nop,
             dur=np.array([0, 1, 2, 3, 4][:n_dur], np.uint32),
             embed=(g.standard_normal((V + 1) * P) * 0.5).astype(np.float32))
    m["wx"] = np.concatenate([q8(4 * P, P) for _ in range(L)])
    m["wh"] = np.concatenate([q8(4 * P, P) for _ in range(L)])
    m["wxs"], m["whs"] = sc(L * 4 * P, 1e-4, 1e-3), sc(L * 4 * P, 1e-4, 1e-3)
    m["lb"] = (g.standard_normal(L * 4 * P) * 0.1).astype(np.float32)
    m["jpred"], m["jpreds"], m["jpredb"] = q8(J, P), sc(J, 1e-4, 1e-3), (g.standard_normal(J) * 0.1).astype(np.float32)
    m["jout"], m["jouts"], m["joutb"] = q8(nop, J), sc(nop, 1e-4, 1e-3), (g.standard_normal(nop) * 0.1).astype(np.float32)
    return m


@pytest.mark.parametrize("rmode", [O.RN, O.RZ])
def test_the_oracles_tokens_at_the_models_shapes(pkb, cuda_device, rmode):
    m = synthetic_model()
    t, keep = device_model(pkb, m)
    g = np.random.default_rng(11 + rmode)
    Ts = [1, 9, 40, 64, 17, 100]
    frames = [(g.standard_normal(T * m["J"]) * 2.0).astype(np.float32) for T in Ts]
    n0 = pkb.launch_count()
    got = search(pkb, t, frames, cap=1024, rmode=rmode)
    # the embedding's quantization, the states' set-up, the search: one launch
    assert pkb.launch_count() - n0 == 3
    total = 0
    for T, f, a in zip(Ts, frames, got):
        want = O.tdt_search(m, f, T, rmode)
        assert a.shape == want.shape and (a == want).all(), T
        total += len(want)
    assert total > 50  # the prediction network stepped on real tokens


def test_a_batch_of_200_segments_in_one_launch(pkb, cuda_device):
    """200 segments at the model's shapes: the one launch takes a product's
    columns 64 segments at a time, so its shared memory does not grow with
    the batch; every segment's tokens are still the oracle's."""
    m = synthetic_model()
    t, keep = device_model(pkb, m)
    g = np.random.default_rng(23)
    Ts = [int(x) for x in g.integers(0, 5, 200)]
    frames = [(g.standard_normal(T * m["J"]) * 2.0).astype(np.float32) for T in Ts]
    n0 = pkb.launch_count()
    got = search(pkb, t, frames, cap=64)
    assert pkb.launch_count() - n0 == 3
    total = 0
    for T, f, a in zip(Ts, frames, got):
        want = O.tdt_search(m, f, T, O.RN)
        assert a.shape == want.shape and (a == want).all(), T
        total += len(want)
    assert total > 20


def test_a_prediction_network_past_one_launchs_shared_memory_takes_the_rounds_launches(pkb, cuda_device):
    """pred_hidden 2048: a job's weight rows and a chunk's inputs would need
    more shared memory than a CTA has, so the rounds run as launches (the
    product kernel and the rounds' kernels); every segment's tokens are
    still the oracle's."""
    m = synthetic_model(P=2048, V=256, seed=5)
    t, keep = device_model(pkb, m)
    g = np.random.default_rng(29)
    Ts = [1, 3, 4, 2]
    frames = [(g.standard_normal(T * m["J"]) * 2.0).astype(np.float32) for T in Ts]
    n0 = pkb.launch_count()
    got = search(pkb, t, frames, cap=64)
    assert pkb.launch_count() - n0 > 10
    total = 0
    for T, f, a in zip(Ts, frames, got):
        want = O.tdt_search(m, f, T, O.RN)
        assert a.shape == want.shape and (a == want).all(), T
        total += len(want)
    assert total > 3


def test_a_segment_past_its_token_room_fails_the_call(pkb, cuda_device):
    g, m = golden_model()
    t, keep = device_model(pkb, m)
    i = 2  # 300 frames, 265 tokens
    f = G.frames(G.CASES[i][0], m["J"], G.CASES[i][1], float(g[f"case/{i}/scale"][0]))
    with pytest.raises(pkb.PkbError):
        search(pkb, t, [f], cap=100)
