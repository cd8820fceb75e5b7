"""The oracle pinned before it is trusted (CPU only).

* Against the committed golden vectors (tests/golden/q8_golden.npz), which
  the reference's own ref backend wrote (tests/golden/make_golden.py).
* Against the reference's ref backend live, where oracle/_ref was built from
  the reference's sources in this checkout.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests import cases as C

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q8_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def keys(g, prefix):
    return sorted({k.split("/")[1] for k in g.files if k.startswith(prefix + "/")}, key=lambda s: (len(s), s))


def test_golden_quantize(golden):
    for i in keys(golden, "qc"):
        T, n, qb, xs = (int(v) for v in golden[f"qc/{i}/shape"])
        q, d = O.quantize(golden[f"qc/{i}/x"], n, qb, T=T, xs=xs)
        assert np.array_equal(q, golden[f"qc/{i}/q"]), i
        assert d.tobytes() == golden[f"qc/{i}/d"].tobytes(), i
    q, d = O.quantize(golden["qx/nonfinite/x"], 64, 32)
    assert np.array_equal(q, golden["qx/nonfinite/q"]) and d.tobytes() == golden["qx/nonfinite/d"].tobytes()
    assert not q.any() and not d.any()
    n = golden["qx/tiny/x"].size // 2
    q, d = O.quantize(golden["qx/tiny/x"], n, 32)
    assert np.array_equal(q, golden["qx/tiny/q"]) and d.tobytes() == golden["qx/tiny/d"].tobytes()


def test_golden_q8check_products(golden):
    for j in keys(golden, "g8"):
        shape = tuple(int(v) for v in golden[f"g8/{j}/shape"])
        rmode = int(golden[f"g8/{j}/rmode"])
        c = C.q8check_case(*shape)
        o = c["out"].copy()
        O.gemm_q8(o, c["os"], c["w"], c["ws"], c["bias"], c["rows"], c["q"], c["d"], c["n"], c["qb"], c["T"],
                  c["add"], rmode)
        assert o.tobytes() == golden[f"g8/{j}/out"].tobytes(), (shape, rmode)


def test_golden_random_products(golden):
    for i in keys(golden, "gr"):
        p = f"gr/{i}/"
        rows, n, T, qb, add, bias, r0, os_ = (int(v) for v in golden[p + "meta"])
        o = golden[p + "out_in"].copy()
        b = golden[p + "bias"][r0:] if bias else None
        O.gemm_q8(o[r0:], os_, golden[p + "w"][r0 * n:], golden[p + "ws"][r0:], b, rows - r0, golden[p + "q"],
                  golden[p + "d"], n, qb, T, bool(add))
        assert o.tobytes() == golden[p + "out"].tobytes(), i


def test_block_sums_exact():
    """The integer sums equal an int64 definition (tests/kcheck.c:217-239)."""
    rng = np.random.default_rng(3)
    rows, n, T, qb = 32, 256, 5, 32
    w_rm = rng.integers(-128, 128, (rows, n)).astype(np.int8)
    q = rng.integers(-127, 128, (T, n)).astype(np.int8)
    s = O.block_sums(O.pack_q8(w_rm), rows, q, n, qb, T)
    want = np.einsum("tbk,rbk->trb", q.reshape(T, n // qb, qb).astype(np.int64),
                     w_rm.reshape(rows, n // qb, qb).astype(np.int64))
    assert np.array_equal(s, want)


def test_pack_roundtrip():
    w = O.uniform_weights(48, 640, 1)
    assert np.array_equal(O.unpack_q8(O.pack_q8(w), 48, 640), w)


needs_ref = pytest.mark.skipif(not O.have_ref(), reason="oracle/_ref not built (reference sources absent)")


@needs_ref
@pytest.mark.parametrize("rmode", [O.RN, O.RD, O.RU, O.RZ])
def test_live_reference_products(rmode):
    """The oracle's product equals the reference's ref in every rounding mode."""
    for seed, (rows, n, T, qb) in enumerate([(32, 128, 5, 32), (48, 1024, 7, 64), (16, 640, 3, 640),
                                             (64, 4096, 9, 32), (32, 96, 2, 96), (16, 16384, 3, 32)]):
        g = np.random.default_rng(seed)
        x = (g.standard_normal(T * n) * g.choice([1.0, 1e4, 1e-38], T * n)).astype(np.float32)
        q, d = O.ref_quantize(x, n, qb)
        w = O.pack_q8(g.integers(-128, 128, (rows, n)).astype(np.int8))
        ws = (g.random(rows) - 0.3).astype(np.float32)
        b = g.standard_normal(rows).astype(np.float32)
        for add in (False, True):
            o1 = g.standard_normal(T * (rows + 3)).astype(np.float32)
            o2 = o1.copy()
            O.gemm_q8(o1, rows + 3, w, ws, b, rows, q, d, n, qb, T, add, rmode)
            O.ref_gemm_q8(o2, rows + 3, w, ws, b, rows, q, d, n, qb, T, add, rmode)
            assert o1.tobytes() == o2.tobytes(), (seed, add)


@needs_ref
def test_live_reference_quantize_rn():
    for seed, (T, n, qb, xs) in enumerate([(5, 128, 32, 160), (7, 1024, 64, 1024), (3, 640, 640, 672),
                                           (9, 4096, 32, 4096), (13, 16384, 32, 16384)]):
        g = np.random.default_rng(100 + seed)
        x = (g.standard_normal(T * xs + n) * g.choice([1.0, 1e4, 1e-38], T * xs + n)).astype(np.float32)
        x[g.integers(0, x.size, 4)] = np.float32(1e-40)
        q1, d1 = O.quantize(x, n, qb, T=T, xs=xs)
        q2, d2 = O.ref_quantize(x, n, qb, T=T, xs=xs)
        assert np.array_equal(q1, q2) and d1.tobytes() == d2.tobytes()


@needs_ref
def test_reference_quantize_directed_modes_differs_only_in_rint():
    """Under RD/RU the reference's ref, as gcc compiles it for baseline
    x86-64, rounds |v * id| and restores the sign (its inline rintf), so a
    negative value rounds toward zero under RD and away from it under RU,
    where IEEE rint (the contract's rint, backend/kernels.h:52, which the
    oracle and the CUDA path follow) rounds down and up. The reference's own
    checks never quantize in a directed mode. This pins that the two differ
    there and nowhere else: the scales agree, every byte of a non-negative
    input agrees, and a negative input's bytes are at most one step apart."""
    n, qb, T = 1024, 32, 8
    x = np.random.default_rng(7).standard_normal(T * n).astype(np.float32) * 100
    neg = x.reshape(T, n) < 0
    for rmode in (O.RD, O.RU):
        q1, d1 = O.quantize(x, n, qb, rmode=rmode)
        q2, d2 = O.ref_quantize(x, n, qb, rmode=rmode)
        assert d1.tobytes() == d2.tobytes()
        assert np.array_equal(q1[~neg], q2[~neg])
        diff = q2[neg].astype(np.int32) - q1[neg].astype(np.int32)
        assert np.all(np.abs(diff) <= 1) and np.any(diff != 0)


@needs_ref
def test_reference_quantize_every_mode_with_its_rint():
    """With the oracle's rintf rounding as the reference's baseline build
    rounds it (|x| in the mode, the sign put back), the oracle's quantize is
    the reference's ref byte for byte in every mode: rint is the whole
    difference."""
    n, qb, T = 1024, 32, 8
    x = np.random.default_rng(8).standard_normal(T * n).astype(np.float32) * 100
    for rmode in (O.RN, O.RD, O.RU, O.RZ):
        with O.rint_style():
            q1, d1 = O.quantize(x, n, qb, rmode=rmode)
        q2, d2 = O.ref_quantize(x, n, qb, rmode=rmode)
        assert np.array_equal(q1, q2) and d1.tobytes() == d2.tobytes()


# ---------------------------------------------------- the fused producers --

PRODUCERS = os.path.join(os.path.dirname(__file__), "golden", "producers_golden.npz")


@pytest.fixture(scope="module")
def producers():
    return np.load(PRODUCERS)


def producer_cases(g):
    """(kind, prefix, meta, rounding modes stored) for every fixture case"""
    for k in sorted(g.files):
        if k.endswith("/meta"):
            p = k[:-4]
            modes = sorted(int(f[len(p) + 1:]) for f in g.files if f.startswith(p + "q"))
            yield p.split("/")[0], p, [int(v) for v in g[k]], modes


def run_producer(g, kind, p, meta, rmode):
    """the oracle on a fixture case: (q, d, floats or None)"""
    if kind == "ln":
        T, n, qb, xs = meta
        return (*O.layernorm_quantize(g[p + "x"], xs, T, n, qb, g[p + "w"], g[p + "b"], float(g[p + "eps"]), rmode),
                None)
    if kind == "si":
        T, n, qb, us = meta
        return (*O.silu_quantize(g[p + "u"], us, T, n, qb, rmode), None)
    T, C, K, glu, qb, xs = meta
    return O.dwconv_quantize(g[p + "x"], xs, T, C, g[p + "w"], g[p + "b"], K, bool(glu), qb, rmode)


def same_as_fixture(g, p, rmode, q, d, o) -> bool:
    return (np.array_equal(q, g[p + f"q{rmode}"]) and d.tobytes() == g[p + f"d{rmode}"].tobytes()
            and (o is None or o.tobytes() == g[p + f"o{rmode}"].tobytes()))


def test_golden_producers(producers):
    """normq, siluq_tile and glu_item + dw_item as the reference's ref wrote
    them (tests/golden/make_producers_golden.py): the oracle with the
    reference's build of rintf matches every case in every mode, and with
    IEEE's rint (what the CUDA path computes) every case in RN and RZ."""
    n_cases = 0
    for kind, p, meta, modes in producer_cases(producers):
        for rmode in modes:
            with O.rint_style():
                assert same_as_fixture(producers, p, rmode, *run_producer(producers, kind, p, meta, rmode)), (p, rmode)
            if rmode in (O.RN, O.RZ):
                assert same_as_fixture(producers, p, rmode, *run_producer(producers, kind, p, meta, rmode)), (p, rmode)
            n_cases += 1
    assert n_cases >= 40


@needs_ref
@pytest.mark.parametrize("rmode", [O.RN, O.RD, O.RU, O.RZ])
def test_live_reference_producers(rmode):
    """The oracle's three producers against the reference's own, composed as
    its encoder composes them, on fresh shapes in every mode."""
    g = np.random.default_rng(50 + rmode)
    for T, n, qb, xs in [(6, 256, 32, 272), (3, 2048, 64, 2048), (11, 160, 32, 160)]:
        x = (g.standard_normal(T * xs + n) * 4 + 1).astype(np.float32)
        w, b = g.standard_normal(n).astype(np.float32), g.standard_normal(n).astype(np.float32)
        with O.rint_style():
            q1, d1 = O.layernorm_quantize(x, xs, T, n, qb, w, b, 1e-5, rmode)
        q2, d2 = O.ref_layernorm_quantize(x, xs, T, n, qb, w, b, 1e-5, rmode)
        assert np.array_equal(q1, q2) and d1.tobytes() == d2.tobytes()
        with O.rint_style():
            q1, d1 = O.silu_quantize(x * 5, xs, T, n, qb, rmode)
        q2, d2 = O.ref_silu_quantize(x * 5, xs, T, n, qb, rmode)
        assert np.array_equal(q1, q2) and d1.tobytes() == d2.tobytes()
    for T, C, K, glu, qb in [(13, 192, 9, 1, 64), (4, 96, 7, 0, 32), (30, 64, 15, 1, 32)]:
        xs = 2 * C + 8
        x = g.standard_normal(T * xs).astype(np.float32)
        w, b = (g.standard_normal(C * K) * 0.5).astype(np.float32), g.standard_normal(C).astype(np.float32)
        with O.rint_style():
            r1 = O.dwconv_quantize(x, xs, T, C, w, b, K, bool(glu), qb, rmode)
        r2 = O.ref_dwconv_quantize(x, xs, T, C, w, b, K, bool(glu), qb, rmode)
        assert all(a.tobytes() == c.tobytes() for a, c in zip(r1, r2))


def test_exp_and_sigmoid_properties():
    """pk_expf and pk_sigmoidf as restated: exact at 0, within 1 and 2 ulp
    of the double-precision functions on a sweep (the accuracy the reference
    states, core/vmath.h:19-31), the clamp's ends, and a NaN taken to the
    low end."""
    x = np.linspace(-87, 88, 200001, dtype=np.float32)
    e = O.expf(x)
    ref = np.exp(x.astype(np.float64)).astype(np.float32)
    ulp = np.abs(e.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    assert ulp.max() <= 1
    s = O.sigmoidf(x)
    sref = (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)
    assert np.abs(s.view(np.int32).astype(np.int64) - sref.view(np.int32).astype(np.int64)).max() <= 2
    special = np.array([0.0, np.nan, np.inf, -np.inf, 1000.0, -1000.0], np.float32)
    e = O.expf(special)
    assert e[0] == 1.0 and e[1] == e[5] == e[3] and e[2] == e[4] and np.isfinite(e).all()


# ------------------------------------------------------ the attention's panels --

def test_golden_panels():
    """The oracle's K/P panel layout is the reference's pk_panels_tile's
    (tests/golden/make_panels_golden.py), padding zeros included."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "panels_golden.npz"))
    cases = sorted({k.split("/")[1] for k in g.files})
    assert len(cases) >= 5
    for i in cases:
        n, np_, D, dk = (int(v) for v in g[f"kp/{i}/meta"])
        assert O.panels_kp(g[f"kp/{i}/src"], n, np_, D, dk).tobytes() == g[f"kp/{i}/dst"].tobytes(), i


@pytest.mark.skipif(not O.have_passes(), reason="oracle/_ref/libpkpasses.so not built")
def test_live_reference_panels():
    g = np.random.default_rng(5)
    for n, D, dk in [(750, 1024, 128), (1499, 1024, 128), (63, 192, 64)]:
        for np_ in ((n + 15) // 16 * 16, (n + 15) // 16 * 16 + 16):
            src = g.standard_normal(n * D).astype(np.float32)
            assert O.panels_kp(src, n, np_, D, dk).tobytes() == O.ref_panels_kp(src, n, np_, D, dk).tobytes()


@pytest.mark.skipif(not O.have_fast(), reason="the reference's backends are not built here")
@pytest.mark.parametrize("T,rows,n,qb,add,bias", [(750, 4096, 1024, 32, 0, 0), (301, 1024, 4096, 64, 1, 0),
                                                  (129, 640, 1024, 1024, 0, 1), (64, 256, 256, 32, 1, 1)])
def test_fast_checker_is_the_oracle(T, rows, n, qb, add, bias):
    """The full-size checker (the reference's picked backend, threaded as its
    passes deal work) gives the oracle's bits: it may stand in for the
    oracle where the oracle's scalar loops are too slow."""
    x = O.seeded_normal(T * n, T + n)
    q, d = O.fast_quantize(x, n, qb, T)
    qo, do = O.quantize(x, n, qb)
    assert np.array_equal(q, qo) and d.tobytes() == do.tobytes()
    w = O.pack_q8(O.uniform_weights(rows, n, rows))
    ws = (1e-3 + 9e-3 * np.random.default_rng(rows).random(rows)).astype(np.float32)
    b = np.random.default_rng(n).standard_normal(rows).astype(np.float32) if bias else None
    out0 = np.random.default_rng(T).standard_normal(T * rows).astype(np.float32)
    got, want = out0.copy(), out0.copy()
    O.fast_gemm_q8(got, rows, w, ws, b, rows, q, d, n, qb, T, bool(add))
    O.gemm_q8(want, rows, w, ws, b, rows, qo, do, n, qb, T, bool(add))
    assert got.tobytes() == want.tobytes()


# ------------------------------------------- the attention's float products --

ATT_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "attention_golden.npz")


@pytest.fixture(scope="module")
def att_golden():
    return np.load(ATT_GOLDEN)


def test_golden_gemm_f32_and_softmax(att_golden):
    """k_gemm_f32 and k_softmax as restated give the reference's ref bits on
    its kcheck-style cases (tests/golden/make_attention_golden.py): runs of
    panels from inside a row, odd n and strides, no bias / one / a bias a
    column written in place, ReLU, and awkward values (zeros of both signs,
    subnormals, large ones)."""
    from tests.golden import make_attention_golden as G
    n = 0
    for i, (meta, w, x, b) in enumerate(G.gemm_f32_cases()):
        assert G.run_gemm_f32(O.gemm_f32, meta, w, x, b).tobytes() == att_golden[f"gf/{i}/out"].tobytes(), meta
        n += 1
    for i, s in enumerate(G.softmax_cases()):
        O.softmax(s, s.size, 1, s.size, 0.0883883476)
        assert s.tobytes() == att_golden[f"sm/{i}/y"].tobytes(), i
        n += 1
    assert n == 64


def test_golden_attention(att_golden):
    """att_item restated query by query equals the reference's own blocked
    run of it (blocks of 16, the position window from a panel boundary)."""
    from tests.golden import make_attention_golden as G
    for i, (T, D, H) in enumerate(G.ATT):
        q, kp, pp, vp, bu, bv = G.att_inputs(T, D, H, 300 + i)
        o = O.attention(q, D, kp, pp, vp, bu, bv, T, D, H)
        assert o.tobytes() == att_golden[f"att/{i}/o"].tobytes(), (T, D, H)


@needs_ref
@pytest.mark.parametrize("rmode", [O.RN, O.RD, O.RU, O.RZ])
def test_live_reference_gemm_f32_and_softmax(rmode):
    """The same restatements against the reference's ref live, in every
    rounding mode (the softmax's exp with the compiled ref's rint)."""
    from tests.golden import make_attention_golden as G
    for meta, w, x, b in G.gemm_f32_cases():
        got = G.run_gemm_f32(lambda *a, **k: O.gemm_f32(*a, rmode=rmode, **k), meta, w, x, b)
        want = G.run_gemm_f32(lambda *a, **k: O.ref_gemm_f32(*a, rmode=rmode, **k), meta, w, x, b)
        assert got.tobytes() == want.tobytes(), (meta, rmode)
    for s in G.softmax_cases():
        s1, s2 = s.copy(), s.copy()
        with O.rint_style():
            O.softmax(s1, s.size, 1, s.size, 0.0883883476, rmode)
        O.ref_softmax(s2, s.size, 1, s.size, 0.0883883476, rmode)
        assert s1.tobytes() == s2.tobytes(), (s.size, rmode)


@needs_ref
def test_live_reference_attention():
    from tests.golden import make_attention_golden as G
    for T, D, H in [(3, 32, 1), (31, 128, 2), (48, 64, 4), (70, 128, 1)]:
        q, kp, pp, vp, bu, bv = G.att_inputs(T, D, H, T + D)
        want = O.ref_attention(q, D, kp, pp, vp, bu, bv, T, D, H)
        assert O.attention(q, D, kp, pp, vp, bu, bv, T, D, H).tobytes() == want.tobytes(), (T, D, H)


# ------------------------------------------------ the TDT decoder's search --

TDT_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "tdt_golden.npz")


def test_golden_tdt_search():
    """The search restated (predict, joint, the label-looping loop of
    core/decoder.c:125-179, with the oracle's quantize, gemm_q8, sigmoid,
    tanh and LSTM cell) gives the reference's own tokens on its tiny model
    (tests/golden/make_tdt_golden.py): blanks that skip frames, durations 0
    to 3, several tokens at one frame."""
    from tests.golden import make_tdt_golden as G
    g = np.load(TDT_GOLDEN)
    m = G.model(g)
    durs = set()
    for i in range(len(G.CASES)):
        T, seed = (int(v) for v in g[f"case/{i}/meta"])
        f = G.frames(T, m["J"], seed, float(g[f"case/{i}/scale"][0]))
        want = g[f"case/{i}/toks"]
        got = O.tdt_search(m, f, T)
        assert got.shape == want.shape and (got == want).all(), (T, seed)
        durs |= set(want[:, 2].tolist())
    assert {0, 1, 2, 3} <= durs


@pytest.mark.skipif(not os.path.exists(O.TDT_REF), reason="oracle/_ref/tdt_ref not built")
def test_live_reference_tdt_search(tmp_path):
    for T, seed, scale in [(77, 11, 2.0), (250, 12, 6.0)]:
        m = O.ref_tdt(T, seed, scale, str(tmp_path / "t.bin"))
        got = O.tdt_search(m, m["f"], T)
        assert got.shape == m["toks"].shape and (got == m["toks"]).all()


def test_tanh_properties():
    """pk_tanhf as restated: odd, within 2 ulp of tanh, 0 and the ends."""
    x = np.linspace(-12, 12, 100001, dtype=np.float32)
    y = O.tanhf(x)
    ref = np.tanh(x.astype(np.float64)).astype(np.float32)
    assert np.abs(y.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64)).max() <= 2
    assert (O.tanhf(-x) == -y).all()
    e = O.tanhf(np.array([0.0, -0.0, 100.0, -100.0], np.float32))
    assert e[0] == 0 and e[2] == 1.0 and e[3] == -1.0
