"""The attention's float work on the GPU, bit for bit against the oracle
(every rounding mode) and against the reference's own outputs
(tests/golden/attention_golden.npz, round to nearest), through the C ABI.

  pkb_gemm_f32_dev        k_gemm_f32 (backend/ref/kernels.c:90-105)
  pkb_softmax_dev         k_softmax (backend/ref/kernels.c:134-147)
  pkb_attention_dev       att_item (core/encoder.c:280-326) over one segment,
                          K, P and V in the reference's panel layouts
  pkb_attention_rows_dev  the same over a batch of segments, K, P and V as
                          the products' plain rows

Cases: the reference's own kcheck draws for gemm_f32 (runs of panels from
inside a row, odd n, strides, no bias / one bias / a bias a column written in
place, ReLU, awkward values) and softmax (1 to 700 awkward scores), then the
attention at the model's shapes (D 1024, 8 heads of 128) with T across the
block size's edges (1, 15, 16, 17) up to the longest chunk (384 frames), a
head of 64 and one of 48, and a batch of segments of ragged lengths.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden import make_attention_golden as G

pytestmark = pytest.mark.gpu

MODES = [O.RN, O.RD, O.RU, O.RZ]
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "attention_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32).reshape(-1)).cuda()


def host(t) -> np.ndarray:
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def gpu_gemm_f32(pkb, meta, w, x, b, rmode):
    rows, ld, k0, n, T, xs, bias_kind, relu, os_ = meta
    out = dev(b)
    bias = (out if bias_kind == 2 else dev(b)) if bias_kind else None
    pkb.gemm_f32_dev(out, os_, dev(w), ld, rows, n, dev(x), xs, T, bias, os_ if bias_kind == 2 else 0, bool(relu),
                     rmode, w_off=16 * k0)
    return host(out)


def test_gemm_f32_reference_cases(pkb, cuda_device, golden):
    """kcheck's gemm_f32 draws: the reference's bits (round to nearest)."""
    for i, (meta, w, x, b) in enumerate(G.gemm_f32_cases()):
        assert gpu_gemm_f32(pkb, meta, w, x, b, O.RN).tobytes() == golden[f"gf/{i}/out"].tobytes(), meta


@pytest.mark.parametrize("rmode", MODES)
def test_gemm_f32_every_mode(pkb, cuda_device, rmode):
    for meta, w, x, b in G.gemm_f32_cases():
        want = G.run_gemm_f32(lambda *a, **k: O.gemm_f32(*a, rmode=rmode, **k), meta, w, x, b)
        assert gpu_gemm_f32(pkb, meta, w, x, b, rmode).tobytes() == want.tobytes(), (meta, rmode)


@pytest.mark.parametrize("rows,ld,n,T", [(400, 128, 128, 16), (128, 384, 384, 16), (1024, 640, 640, 1),
                                         (16, 1, 1, 70), (2560, 640, 640, 3)])
def test_gemm_f32_shapes(pkb, cuda_device, rows, ld, n, T):
    """The attention's and the decoder's shapes: scores over 400 keys, the
    weighted sum over 384, a gemv (T 1, strides not read), n of 1."""
    g = np.random.default_rng(rows + n + T)
    w = g.standard_normal(rows * ld).astype(np.float32)
    x = g.standard_normal(T * n + 3).astype(np.float32)
    b = g.standard_normal(rows).astype(np.float32)
    for bias, relu in ((None, False), (b, True)):
        want = np.full(T * rows, 7.0, np.float32)
        O.gemm_f32(want, rows, w, ld, rows, n, x, n, T, bias, 0, relu)
        out = dev(np.full(T * rows, 7.0, np.float32))
        pkb.gemm_f32_dev(out, 0 if T == 1 else rows, dev(w), ld, rows, n, dev(x), 0 if T == 1 else n, T,
                         None if bias is None else dev(bias), 0, relu)
        assert host(out).tobytes() == want.tobytes()


def test_softmax_reference_cases(pkb, cuda_device, golden):
    for i, s in enumerate(G.softmax_cases()):
        x = dev(s)
        pkb.softmax_dev(x, s.size, 1, s.size, 0.0883883476)
        assert host(x).tobytes() == golden[f"sm/{i}/y"].tobytes(), s.size


@pytest.mark.parametrize("rmode", MODES)
def test_softmax_every_mode(pkb, cuda_device, rmode):
    """Every mode against the oracle (IEEE rint in pk_expf), one row a call
    and many rows at a stride; rows of constants, of -inf and NaN, one huge."""
    for s in G.softmax_cases():
        want = s.copy()
        O.softmax(want, s.size, 1, s.size, 0.0883883476, rmode)
        x = dev(s)
        pkb.softmax_dev(x, s.size, 1, s.size, 0.0883883476, rmode)
        assert host(x).tobytes() == want.tobytes(), (s.size, rmode)
    g = np.random.default_rng(9 + rmode)
    T, n, xs = 53, 375, 384
    x0 = (g.standard_normal(T * xs) * 30).astype(np.float32)
    x0[0 * xs:0 * xs + n] = 3.5
    x0[1 * xs:1 * xs + n] = -np.inf
    x0[2 * xs + 7] = np.nan
    x0[3 * xs + 5] = np.inf
    x0[4 * xs + 11] = 1e30
    want = x0.copy()
    O.softmax(want, xs, T, n, 0.0883883476, rmode)
    x = dev(x0)
    pkb.softmax_dev(x, xs, T, n, 0.0883883476, rmode)
    assert host(x).tobytes() == want.tobytes()


def test_attention_reference_cases(pkb, cuda_device, golden):
    """The reference's own blocked att_item (16 queries a block, its position
    window from a panel boundary) on every golden case."""
    for i, (T, D, H) in enumerate(G.ATT):
        q, kp, pp, vp, bu, bv = G.att_inputs(T, D, H, 300 + i)
        o = dev(np.full(T * D, 5.0, np.float32))
        pkb.attention_dev(o, D, dev(q), D, dev(kp), dev(pp), dev(vp), dev(bu), dev(bv), T, D, H)
        assert host(o).tobytes() == golden[f"att/{i}/o"].tobytes(), (T, D, H)


@pytest.mark.parametrize("T,D,H,rmode", [(1, 1024, 8, O.RN), (15, 1024, 8, O.RN), (16, 1024, 8, O.RD),
                                         (17, 1024, 8, O.RU), (100, 1024, 8, O.RZ), (384, 1024, 8, O.RN),
                                         (77, 512, 8, O.RN), (50, 192, 4, O.RU), (33, 256, 1, O.RN)])
def test_attention_panels(pkb, cuda_device, T, D, H, rmode):
    """att_item over one segment at the model's shapes, across the block's
    edges up to the longest chunk (384 frames); heads of 128, 64, 48 and 256;
    o at a row stride beyond D, its other floats untouched."""
    q, kp, pp, vp, bu, bv = G.att_inputs(T, D, H, 7 * T + D)
    want = O.attention(q, D, kp, pp, vp, bu, bv, T, D, H, rmode)
    os_ = D + 16
    o = dev(np.full(T * os_, 5.0, np.float32))
    pkb.attention_dev(o, os_, dev(q), D, dev(kp), dev(pp), dev(vp), dev(bu), dev(bv), T, D, H, rmode)
    got = host(o).reshape(T, os_)
    assert got[:, :D].tobytes() == want.tobytes()
    assert (got[:, D:] == 5.0).all()


def rows_to_panels(k: np.ndarray, T: int, D: int, dk: int, np_: int) -> np.ndarray:
    """K or P rows [T][D] as the reference's K/P panels (pk_panels_tile)."""
    return O.panels_kp(np.ascontiguousarray(k, np.float32).reshape(-1), T, np_, D, dk)


def rows_to_vpanels(v: np.ndarray, T: int, D: int) -> np.ndarray:
    return np.ascontiguousarray(v.reshape(T, D // 16, 16).transpose(1, 0, 2)).reshape(-1)


@pytest.mark.parametrize("rmode", [O.RN, O.RD])
def test_attention_rows_batch(pkb, cuda_device, rmode):
    """A batch of ragged segments in one launch, K, V and P as rows of the
    batch (K and V at their own strides, P's rows segment after segment):
    each segment's o is the oracle's for that segment alone."""
    D, H = 1024, 8
    dk = D // H
    Ts = [1, 17, 40, 100, 5, 64, 16, 233]
    g = np.random.default_rng(41 + rmode)
    M, Rsum = sum(Ts), sum(2 * t - 1 for t in Ts)
    ks, vs, ps = D + 4, D + 8, D
    q = g.standard_normal(M * D).astype(np.float32)
    k = g.standard_normal(M * ks).astype(np.float32)
    v = g.standard_normal(M * vs).astype(np.float32)
    p = g.standard_normal(Rsum * ps).astype(np.float32)
    bu = (g.standard_normal(D) * 0.1).astype(np.float32)
    bv = (g.standard_normal(D) * 0.1).astype(np.float32)
    segs, f, r = [], 0, 0
    for T in Ts:
        segs.append((T, f, r))
        f += T
        r += 2 * T - 1
    o = dev(np.full(M * D, 5.0, np.float32))
    pkb.attention_rows_dev(o, D, dev(q), D, dev(k), ks, dev(v), vs, dev(p), ps, dev(bu), dev(bv), D, H, segs, rmode)
    got = host(o).reshape(M, D)
    for T, f, r in segs:
        R = 2 * T - 1
        Tp, Pp = (T + 15) // 16 * 16, (R + 15) // 16 * 16 + 16
        kr = k.reshape(M, ks)[f:f + T, :D]
        vr = v.reshape(M, vs)[f:f + T, :D]
        pr = p.reshape(Rsum, ps)[r:r + R, :D]
        want = O.attention(q.reshape(M, D)[f:f + T], D, rows_to_panels(kr, T, D, dk, Tp),
                           rows_to_panels(pr, R, D, dk, Pp), rows_to_vpanels(vr, T, D), bu, bv, T, D, H, rmode)
        assert got[f:f + T].tobytes() == want.tobytes(), T


def test_attention_refuses_what_it_cannot_take(pkb, cuda_device):
    """Heads that are not whole panels, and a segment too long for a block's
    shared memory, are refused with PKB_EINVAL before any launch."""
    import torch
    buf = torch.zeros(4096 * 1024 * 3, device="cuda")
    launches = pkb.launch_count()
    with pytest.raises(pkb.PkbError):
        pkb.attention_dev(buf, 1000, buf, 1000, buf, buf, buf, buf, buf, 10, 1000, 8)  # dk 125
    with pytest.raises(pkb.PkbError):
        pkb.attention_dev(buf, 1024, buf, 1024, buf, buf, buf, buf, buf, 4000, 1024, 8)  # T 4000
    assert pkb.launch_count() == launches


def test_host_entries_of_the_table(pkb, cuda_device, golden):
    """pkb_gemm_f32_host and pkb_softmax_host (the cuda-b200-f32 table's
    gemm_f32 and softmax) on host memory: kcheck's draws, a bias a column
    written in place among them, the reference's bits; the bytes of out
    between the rows left as they were."""
    import ctypes
    lib = pkb.lib()
    for i, (meta, w, x, b) in enumerate(G.gemm_f32_cases()):
        rows, ld, k0, n, T, xs, bias_kind, relu, os_ = meta
        out = b.copy()
        bias = (out if bias_kind == 2 else b) if bias_kind else None
        rc = lib.pkb_gemm_f32_host(out.ctypes.data, os_, w.ctypes.data + 64 * k0, ld, rows, n, x.ctypes.data, xs, T,
                                   0 if bias is None else bias.ctypes.data, os_ if bias_kind == 2 else 0, relu, O.RN)
        assert rc == 0, pkb.lib().pkb_last_error()
        assert out.tobytes() == golden[f"gf/{i}/out"].tobytes(), meta
    for i, s in enumerate(G.softmax_cases()):
        x = s.copy()
        assert lib.pkb_softmax_host(x.ctypes.data, x.size, ctypes.c_float(0.0883883476), O.RN) == 0
        assert x.tobytes() == golden[f"sm/{i}/y"].tobytes(), s.size


def test_attention_rows_more_segments_than_a_launch_takes(pkb, cuda_device):
    """130 short segments (a launch takes 128): the call splits them over two
    launches; every segment's o is the oracle's."""
    D, H = 256, 4
    dk = D // H
    g = np.random.default_rng(77)
    Ts = [1 + (i * 7) % 11 for i in range(130)]
    M, Rsum = sum(Ts), sum(2 * t - 1 for t in Ts)
    q, k, v = (g.standard_normal(M * D).astype(np.float32) for _ in range(3))
    p = g.standard_normal(Rsum * D).astype(np.float32)
    bu, bv = (g.standard_normal(D) * 0.1).astype(np.float32), (g.standard_normal(D) * 0.1).astype(np.float32)
    segs, f, r = [], 0, 0
    for T in Ts:
        segs.append((T, f, r))
        f += T
        r += 2 * T - 1
    launches = pkb.launch_count()
    o = dev(np.full(M * D, 5.0, np.float32))
    pkb.attention_rows_dev(o, D, dev(q), D, dev(k), D, dev(v), D, dev(p), D, dev(bu), dev(bv), D, H, segs)
    got = host(o).reshape(M, D)
    assert pkb.launch_count() - launches == 2
    for T, f, r in segs:
        R = 2 * T - 1
        Tp, Pp = (T + 15) // 16 * 16, (R + 15) // 16 * 16 + 16
        want = O.attention(q.reshape(M, D)[f:f + T], D, rows_to_panels(k.reshape(M, D)[f:f + T], T, D, dk, Tp),
                           rows_to_panels(p.reshape(Rsum, D)[r:r + R], R, D, dk, Pp),
                           rows_to_vpanels(v.reshape(M, D)[f:f + T], T, D), bu, bv, T, D, H)
        assert got[f:f + T].tobytes() == want.tobytes(), T
