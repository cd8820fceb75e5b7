"""The fused producers of the product's int8 inputs on the GPU, bit for bit
against the oracle (IEEE rint: every mode) and against the reference's own
outputs (tests/golden/producers_golden.npz: RN and RZ, where the reference's
baseline build of rintf is IEEE's), through the C ABI.

  pkb_layernorm_quantize_dev  normq (core/encoder.c:112-130)
  pkb_silu_quantize_dev       siluq_tile (core/encoder.c:150-158)
  pkb_dwconv_quantize_dev     glu_item + dw_item (core/encoder.c:160-183)

Cases follow the reference's own float-kernel checks (tests/kcheck.c's
awkward values, rows of constants, non-finite inputs, strides beyond the
row) plus what the kernels' layout makes edges: an odd count of rows (a
warp takes two), rows and channel counts not a multiple of the tile, the
taps of a convolution longer than the sequence, misaligned buffers (the
scalar-load and 4-byte-store forms).
"""
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MODES = [O.RN, O.RD, O.RU, O.RZ]
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "producers_golden.npz")


def dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.cuda() if dtype is None else t.to(dtype).cuda()


def host(t) -> np.ndarray:
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def empty(n, kind, off=0):
    """a device buffer of n elements starting `off` elements into a larger
    one (for misaligned starts), filled with a marker"""
    import torch
    if kind == "q":
        base = torch.full((n + 16,), 77, dtype=torch.int8, device="cuda")
    else:
        base = torch.full((n + 16,), 1234.5, dtype=torch.float32, device="cuda")
    return base, base[off:off + n]


def awkward_rows(g, T, xs, n, scale=1.0):
    x = (g.standard_normal(T * xs + n) * scale + g.standard_normal()).astype(np.float32)
    return x


def gpu_ln(pkb, x, xs, T, n, qb, w, b, eps, rmode, xoff=0, qoff=0, woff=0):
    xb, xd = empty(x.size, "f", xoff)
    xd.copy_(dev(x))
    wb, wd = empty(n, "f", woff)
    wd.copy_(dev(w))
    bb, bd = empty(n, "f", woff)
    bd.copy_(dev(b))
    qbuf, qd = empty(T * n, "q", qoff)
    dbuf, dd = empty(T * (n // qb), "f")
    pkb.layernorm_quantize_dev(qd, dd, xd, xs, T, n, qb, wd, bd, eps, rmode)
    qh = host(qbuf)
    assert (qh[:qoff] == 77).all() and (qh[qoff + T * n:] == 77).all(), "bytes outside q written"
    return qh[qoff:qoff + T * n].reshape(T, n), host(dd).reshape(T, -1)


def gpu_silu(pkb, u, us, T, n, qb, rmode, uoff=0, qoff=0):
    ub, ud = empty(u.size, "f", uoff)
    ud.copy_(dev(u))
    qbuf, qd = empty(T * n, "q", qoff)
    dbuf, dd = empty(T * (n // qb), "f")
    pkb.silu_quantize_dev(qd, dd, ud, us, T, n, qb, rmode)
    qh = host(qbuf)
    assert (qh[:qoff] == 77).all() and (qh[qoff + T * n:] == 77).all(), "bytes outside q written"
    return qh[qoff:qoff + T * n].reshape(T, n), host(dd).reshape(T, -1)


def gpu_dw(pkb, x, xs, T, C, w, b, K, glu, qb, rmode, with_out=True, os_=None):
    os_ = C if os_ is None else os_
    xd = dev(x)
    qbuf, qd = empty(T * C, "q")
    dbuf, dd = empty(T * (C // qb), "f")
    ob = None
    if with_out:
        ob, od = empty(T * os_, "f")
    pkb.dwconv_quantize_dev(qd, dd, od if with_out else None, os_, xd, xs, T, C, dev(w), dev(b), K, glu, qb, rmode)
    qh = host(qbuf)
    assert (qh[T * C:] == 77).all(), "bytes outside q written"
    o = None
    if with_out:
        oh = host(ob)[:T * os_].reshape(T, os_)
        assert (oh[:, C:] == 1234.5).all(), "floats between rows written"
        o = np.ascontiguousarray(oh[:, :C])
    return qh[:T * C].reshape(T, C), host(dd).reshape(T, -1), o


def same(a, b) -> bool:
    return a.tobytes() == b.tobytes()


def same_floats(a, b) -> bool:
    """the same bits, except that a NaN matches any NaN: the payload of a
    NaN an operation makes is the platform's (x86's default NaN has the sign
    bit set, the GPU's canonical one not), not the reference's contract"""
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb)) and a[~na].tobytes() == b[~nb].tobytes()


# ---------------------------------------------------------------- golden --

def golden_cases():
    g = np.load(GOLDEN)
    out = []
    for k in sorted(g.files):
        if k.endswith("/meta"):
            p = k[:-4]
            for f in g.files:
                if f.startswith(p + "q"):
                    m = int(f[len(p) + 1:])
                    if m in (O.RN, O.RZ):
                        out.append((p, m))
    return out


@pytest.mark.parametrize("p,rmode", golden_cases())
def test_golden(pkb, cuda_device, p, rmode):
    g = np.load(GOLDEN)
    meta = [int(v) for v in g[p + "meta"]]
    kind = p.split("/")[0]
    if kind == "ln":
        T, n, qb, xs = meta
        q, d = gpu_ln(pkb, g[p + "x"], xs, T, n, qb, g[p + "w"], g[p + "b"], float(g[p + "eps"]), rmode)
        o = None
    elif kind == "si":
        T, n, qb, us = meta
        q, d = gpu_silu(pkb, g[p + "u"], us, T, n, qb, rmode)
        o = None
    else:
        T, C, K, glu, qb, xs = meta
        q, d, o = gpu_dw(pkb, g[p + "x"], xs, T, C, g[p + "w"], g[p + "b"], K, bool(glu), qb, rmode)
    assert np.array_equal(q, g[p + f"q{rmode}"])
    assert same(d, g[p + f"d{rmode}"])
    if o is not None:
        assert same_floats(o, g[p + f"o{rmode}"])


# ------------------------------------------------------------- layer norm --

LN_SHAPES = [(1, 32, 32, 32), (2, 64, 64, 64), (3, 96, 32, 100), (37, 1024, 32, 1024), (750, 1024, 32, 1024),
             (33, 1024, 64, 1040), (5, 4096, 32, 4096), (3, 8192, 64, 8192), (17, 160, 32, 161)]


@pytest.mark.parametrize("T,n,qb,xs", LN_SHAPES)
@pytest.mark.parametrize("rmode", MODES)
def test_layernorm_quantize(pkb, cuda_device, T, n, qb, xs, rmode):
    g = np.random.default_rng(T * 31 + n + qb + rmode)
    x = awkward_rows(g, T, xs, n, scale=g.choice([0.01, 1.0, 300.0]))
    if T > 3:
        x[xs: xs + n] = np.float32(-2.5)  # a constant row: variance 0
        x[2 * xs + 7] = np.nan
    w = g.standard_normal(n).astype(np.float32)
    b = (g.standard_normal(n) * 0.1).astype(np.float32)
    q, d = gpu_ln(pkb, x, xs, T, n, qb, w, b, 1e-5, rmode)
    qo, do = O.layernorm_quantize(x, xs, T, n, qb, w, b, 1e-5, rmode)
    assert np.array_equal(q, qo)
    assert same(d, do)


@pytest.mark.parametrize("xoff,qoff,woff", [(1, 0, 0), (0, 4, 0), (0, 0, 1), (3, 12, 2)])
def test_layernorm_quantize_misaligned(pkb, cuda_device, xoff, qoff, woff):
    """x not 16-byte aligned (scalar loads), q not 8-byte aligned (4-byte
    stores), w and b not 16-byte aligned (scalar loads)"""
    T, n, qb = 9, 1024, 32
    g = np.random.default_rng(xoff + 10 * qoff + 100 * woff)
    x = awkward_rows(g, T, n, n, 3.0)
    w, b = g.standard_normal(n).astype(np.float32), g.standard_normal(n).astype(np.float32)
    q, d = gpu_ln(pkb, x, n, T, n, qb, w, b, 1e-6, O.RN, xoff=xoff, qoff=qoff, woff=woff)
    qo, do = O.layernorm_quantize(x, n, T, n, qb, w, b, 1e-6, O.RN)
    assert np.array_equal(q, qo) and same(d, do)


def test_layernorm_quantize_extremes(pkb, cuda_device):
    """rows whose sums overflow, whose variance underflows to eps alone,
    subnormal rows, infinite inputs, and eps of 0 on a constant row (1/0)"""
    T, n, qb = 8, 256, 32
    g = np.random.default_rng(3)
    x = g.standard_normal(T * n).astype(np.float32)
    x[0:n] *= np.float32(3e38)
    x[n:2 * n] *= np.float32(1e-30)
    x[2 * n:3 * n] = (g.standard_normal(n) * 1e-40).astype(np.float32)
    x[3 * n + 5] = np.inf
    x[4 * n:5 * n] = np.float32(7.0)
    w, b = g.standard_normal(n).astype(np.float32), g.standard_normal(n).astype(np.float32)
    for eps in (1e-5, 0.0):
        for rmode in MODES:
            q, d = gpu_ln(pkb, x, n, T, n, qb, w, b, eps, rmode)
            qo, do = O.layernorm_quantize(x, n, T, n, qb, w, b, eps, rmode)
            assert np.array_equal(q, qo) and same(d, do), (eps, rmode)


# ------------------------------------------------------------------- SiLU --

SILU_SHAPES = [(1, 32, 32, 32), (3, 64, 64, 64), (750, 4096, 32, 4096), (11, 4096, 64, 4160), (7, 96, 32, 97),
               (1499, 1024, 32, 1024)]


@pytest.mark.parametrize("T,n,qb,us", SILU_SHAPES)
@pytest.mark.parametrize("rmode", MODES)
def test_silu_quantize(pkb, cuda_device, T, n, qb, us, rmode):
    g = np.random.default_rng(T + n + us + rmode)
    u = (g.standard_normal(T * us + n) * g.choice([1.0, 10.0, 60.0])).astype(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 87.0, -87.0, 88.0, -88.0, 87.3, -87.3, 1e-40, -1e-40,
                        3e38, -3e38], np.float32)
    u[g.integers(0, u.size, special.size)] = special
    q, d = gpu_silu(pkb, u, us, T, n, qb, rmode)
    qo, do = O.silu_quantize(u, us, T, n, qb, rmode)
    assert np.array_equal(q, qo)
    assert same(d, do)


@pytest.mark.parametrize("uoff,qoff", [(1, 0), (0, 4), (2, 4)])
def test_silu_quantize_misaligned(pkb, cuda_device, uoff, qoff):
    T, n, qb = 13, 1024, 64
    u = (np.random.default_rng(uoff + qoff).standard_normal(T * n) * 6).astype(np.float32)
    q, d = gpu_silu(pkb, u, n, T, n, qb, O.RU, uoff=uoff, qoff=qoff)
    qo, do = O.silu_quantize(u, n, T, n, qb, O.RU)
    assert np.array_equal(q, qo) and same(d, do)


def test_silu_every_exponent(pkb, cuda_device):
    """SiLU of a float of every exponent and both signs, and the values
    either side of the exp argument's clamp, one value a block (so each
    byte is 127 or 0 and the scale carries the value): the device's exp and
    sigmoid are the reference's bit for bit wherever the result is finite"""
    vals = []
    for e in range(-149, 128):
        for m in (1.0, 1.2345678, 1.9999999):
            v = np.float32(m * 2.0 ** e) if e > -127 else np.float32(2.0 ** e)
            vals += [v, -v]
    vals += list(np.linspace(-88.5, 88.5, 4001, dtype=np.float32))
    v = np.array(vals, np.float32)
    T = v.size
    u = np.zeros((T, 32), np.float32)
    u[:, 0] = v
    for rmode in MODES:
        q, d = gpu_silu(pkb, u.reshape(-1), 32, T, 32, 32, rmode)
        qo, do = O.silu_quantize(u.reshape(-1), 32, T, 32, 32, rmode)
        assert np.array_equal(q, qo) and same(d, do), rmode


# ---------------------------------------------------------------- dwconv --

DW_SHAPES = [(1, 32, 9, 0, 32), (2, 64, 9, 1, 64), (5, 96, 9, 1, 32), (40, 1024, 9, 1, 32), (750, 1024, 9, 1, 32),
             (33, 1024, 9, 0, 64), (100, 256, 31, 1, 32), (64, 64, 63, 0, 64), (31, 160, 3, 1, 32), (8, 64, 1, 1, 64),
             (97, 512, 15, 0, 32)]


@pytest.mark.parametrize("T,C,K,glu,qb", DW_SHAPES)
@pytest.mark.parametrize("rmode", MODES)
def test_dwconv_quantize(pkb, cuda_device, T, C, K, glu, qb, rmode):
    g = np.random.default_rng(T * 3 + C + K + glu + rmode)
    xs = (2 * C if glu else C) + (8 if T % 2 else 0)
    x = (g.standard_normal(T * xs) * 2).astype(np.float32)
    w = (g.standard_normal(C * K) * 0.3).astype(np.float32)
    b = (g.standard_normal(C) * 0.2).astype(np.float32)
    if T > 10:
        x[5 * xs + 3] = np.nan
    if C >= 128:
        w[70 * K] = np.inf  # channel 70's first tap: past the start at frame 0, so skipped there
    q, d, o = gpu_dw(pkb, x, xs, T, C, w, b, K, bool(glu), qb, rmode)
    qo, do, oo = O.dwconv_quantize(x, xs, T, C, w, b, K, bool(glu), qb, rmode)
    assert same_floats(o, oo)
    assert np.array_equal(q, qo)
    assert same(d, do)


def test_dwconv_quantize_without_floats_and_strided_out(pkb, cuda_device):
    T, C, K, qb = 45, 256, 9, 32
    g = np.random.default_rng(9)
    x = g.standard_normal(T * 2 * C).astype(np.float32)
    w, b = (g.standard_normal(C * K) * 0.3).astype(np.float32), g.standard_normal(C).astype(np.float32)
    qo, do, oo = O.dwconv_quantize(x, 2 * C, T, C, w, b, K, True, qb, O.RN)
    q, d, _ = gpu_dw(pkb, x, 2 * C, T, C, w, b, K, True, qb, O.RN, with_out=False)
    assert np.array_equal(q, qo) and same(d, do)
    q, d, o = gpu_dw(pkb, x, 2 * C, T, C, w, b, K, True, qb, O.RN, os_=C + 24)
    assert np.array_equal(q, qo) and same(d, do) and same_floats(o, oo)


def test_producers_on_a_side_stream(pkb, cuda_device):
    """enqueued on the caller's stream, not the default one"""
    import torch
    T, n, qb = 64, 1024, 32
    x = np.random.default_rng(4).standard_normal(T * n).astype(np.float32)
    w, b = np.ones(n, np.float32), np.zeros(n, np.float32)
    s = torch.cuda.Stream()
    xd, wd, bd = dev(x), dev(w), dev(b)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        q = torch.empty(T * n, dtype=torch.int8, device="cuda")
        d = torch.empty(T * n // qb, dtype=torch.float32, device="cuda")
        pkb.layernorm_quantize_dev(q, d, xd, n, T, n, qb, wd, bd, 1e-5, O.RN, stream=s.cuda_stream)
        q2 = torch.empty_like(q)
        d2 = torch.empty_like(d)
        pkb.silu_quantize_dev(q2, d2, xd, n, T, n, qb, O.RN, stream=s.cuda_stream)
    s.synchronize()
    qo, do = O.layernorm_quantize(x, n, T, n, qb, w, b, 1e-5, O.RN)
    assert np.array_equal(q.cpu().numpy().reshape(T, n), qo) and same(d.cpu().numpy().reshape(T, -1), do)
    qo, do = O.silu_quantize(x, n, T, n, qb, O.RN)
    assert np.array_equal(q2.cpu().numpy().reshape(T, n), qo) and same(d2.cpu().numpy().reshape(T, -1), do)


@pytest.mark.parametrize("rmode", MODES)
def test_sigmoid_reciprocal_exhaustive(pkb, cuda_device, rmode):
    """The sigmoid's branch-free reciprocal (Markstein's method) is the
    correctly rounded 1/y for every finite float y >= 1 (1 + e^-x reaches
    1.7e38, whose reciprocal is subnormal), in each rounding mode: no
    mismatch over 1.07e9 floats."""
    mismatches, first = pkb.rcp_selftest(rmode)
    assert mismatches == 0, f"{mismatches} floats differ, the first 0x{first:08x}"


@pytest.mark.parametrize("rmode", MODES)
def test_layernorm_floats(pkb, cuda_device, rmode):
    """k_layernorm alone (the encoder's out norm): the floats against the
    oracle in every mode, at the model's width and an odd one, rows at a
    stride, and in place as the reference runs it."""
    import torch
    g = np.random.default_rng(60 + rmode)
    for T, n, xs in [(37, 1024, 1024), (9, 160, 200), (1, 4096, 4096)]:
        x = (g.standard_normal(T * xs) * 3 + 500.0 * (n == 160)).astype(np.float32)
        w, b = g.standard_normal(n).astype(np.float32), g.standard_normal(n).astype(np.float32)
        want = O.layernorm(x, xs, T, n, w, b, 1e-5, rmode)
        out = torch.full((T * (n + 8),), 7.0, device="cuda")
        pkb.layernorm_dev(out, n + 8, dev(x), xs, T, n, dev(w), dev(b), 1e-5, rmode)
        got = host(out).reshape(T, n + 8)
        assert got[:, :n].tobytes() == want.tobytes(), (T, n)
        assert (got[:, n:] == 7.0).all()
        xi = dev(x)
        pkb.layernorm_dev(xi, xs, xi, xs, T, n, dev(w), dev(b), 1e-5, rmode)
        inplace = host(xi).reshape(T, xs)
        assert inplace[:, :n].tobytes() == want.tobytes(), (T, n, "in place")
