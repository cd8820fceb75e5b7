"""The CUDA path against the oracle, bit for bit, through the C ABI.

Every comparison is of bytes (float32 bit patterns, int8 values): the
reference's contract is ref's bits, not ref's answer to a tolerance
(backend/kernels.h:9-24). Cases follow the reference's own checks:
tests/q8check.c (edges, output stride 35, rounding modes, no columns) and
tests/kcheck.c (random products on awkward values, runs of panels, blocks
of 32, 64 and a whole row).
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests import cases as C

pytestmark = pytest.mark.gpu


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    return a.tobytes() == b.tobytes()


def first_diff(a: np.ndarray, b: np.ndarray) -> str:
    av, bv = a.reshape(-1).view(np.uint32), b.reshape(-1).view(np.uint32)
    i = int(np.nonzero(av != bv)[0][0])
    return f"element {i}: {a.reshape(-1)[i]!r} vs oracle {b.reshape(-1)[i]!r} ({int((av != bv).sum())} differ)"


# ------------------------------------------------------------- quantize --

QUANT_SHAPES = [(1, 32, 32, 32), (5, 128, 32, 160), (20, 1024, 32, 1024), (7, 1024, 64, 1056),
                (3, 640, 640, 640), (2, 96, 96, 96), (13, 4096, 32, 4096), (4, 16384, 16384, 16384),
                (750, 1024, 32, 1024), (33, 256, 64, 257)]


@pytest.mark.parametrize("T,n,qb,xs", QUANT_SHAPES)
@pytest.mark.parametrize("rmode", [O.RN, O.RD, O.RU, O.RZ])
def test_quantize_host(pkb, cuda_device, T, n, qb, xs, rmode):
    rng = O.XorShift(0x1234 + T * 7 + n + qb + rmode)
    scale = 1e4 if (T + n) % 3 == 0 else 1.0
    x = C.awkward_array(rng, T * xs + n, scale)
    if T > 1:
        x[:qb] = 0.0  # a block of zeros: scale 0
    x[min(5, x.size - 1)] = np.float32(1e-40)
    q, d = pkb.quantize_host(x, n, qb, T=T, xs=xs, rmode=rmode)
    qo, do = O.quantize(x, n, qb, T=T, xs=xs, rmode=rmode)
    assert np.array_equal(q, qo)
    assert same_bits(d, do), first_diff(d, do)
    assert q.min() >= -127 or rmode in (O.RU, O.RD)


def test_quantize_nonfinite_and_tiny(pkb, cuda_device):
    # tests/kcheck.c:120-175: non-finite inputs and amax either side of 2^-121
    T, n, qb = 2, 64, 32
    x = np.array([O.XorShift(9).frand() for _ in range(T * n)], np.float32)
    x[3], x[40], x[n + 5], x[n + 45] = np.nan, np.inf, -np.inf, np.nan
    q, d = pkb.quantize_host(x, n, qb)
    assert not q.any() and not d.any()
    tops = np.array([2.0**-140, 2.0**-130, 2.0**-122, np.float32(float.fromhex('0x1.fffffep-122')), 2.0**-121, 2.0**-120,
                     2.0**-100], np.float32)
    n = 32 * len(tops)
    rng = O.XorShift(77)
    x = np.empty(2 * n, np.float32)
    for t in range(2):
        for b, top in enumerate(tops):
            v = np.array([top * np.float32(rng.frand()) for _ in range(32)], np.float32)
            v[rng.rnd() % 32] = -top if t else top
            x[t * n + 32 * b: t * n + 32 * b + 32] = v
    q, d = pkb.quantize_host(x, n, 32)
    qo, do = O.quantize(x, n, 32)
    assert np.array_equal(q, qo) and same_bits(d, do)
    assert ((d.reshape(2, -1) == 0) == (tops < 2.0**-121)[None, :]).all()


def test_quantize_dev_matches_host(pkb, cuda_device):
    import torch
    T, n, qb = 300, 4096, 32
    x = O.seeded_normal(T * n, 5)
    xd = torch.from_numpy(x).cuda()
    q = torch.empty(T * n, dtype=torch.int8, device="cuda")
    d = torch.empty(T * n // qb, dtype=torch.float32, device="cuda")
    pkb.quantize_dev(q, d, xd, n, T, n, qb)
    torch.cuda.synchronize()
    qo, do = O.quantize(x, n, qb)
    assert np.array_equal(q.cpu().numpy().reshape(T, n), qo)
    assert same_bits(d.cpu().numpy().reshape(T, -1), do)


@pytest.mark.parametrize("qoff", [0, 4, 8, 12])
@pytest.mark.parametrize("qb", [32, 64])
def test_quantize_dev_q_alignment(pkb, cuda_device, qoff, qb):
    # the interface asks q to be 4-byte aligned; 8-byte stores of q are only
    # taken where it is 8-byte aligned, so both forms must give ref's bytes
    import torch
    T, n = 37, 1024
    x = O.seeded_normal(T * n, 11 + qoff + qb)
    xd = torch.from_numpy(x).cuda()
    qbuf = torch.full((T * n + 16,), 99, dtype=torch.int8, device="cuda")
    d = torch.empty(T * n // qb, dtype=torch.float32, device="cuda")
    pkb.quantize_dev(qbuf[qoff:], d, xd, n, T, n, qb, rmode=O.RD)
    torch.cuda.synchronize()
    qo, do = O.quantize(x, n, qb, rmode=O.RD)
    got = qbuf.cpu().numpy()
    assert np.array_equal(got[qoff:qoff + T * n].reshape(T, n), qo)
    assert (got[:qoff] == 99).all() and (got[qoff + T * n:] == 99).all()
    assert same_bits(d.cpu().numpy().reshape(T, -1), do)


# ---------------------------------------------------------------- gemm_q8 --

def run_host_case(pkb, c, rmode=O.RN):
    got = c["out"].copy()
    pkb.gemm_q8_host(got, c["os"], c["w"], c["ws"], c["bias"], c["rows"], c["q"], c["d"], c["n"], c["qb"], c["T"],
                     c["add"], rmode)
    want = c["out"].copy()
    O.gemm_q8(want, c["os"], c["w"], c["ws"], c["bias"], c["rows"], c["q"], c["d"], c["n"], c["qb"], c["T"],
              c["add"], rmode)
    return got, want


@pytest.mark.parametrize("shape", C.q8check_shapes(), ids=lambda s: "n%d-qb%d-T%d-f%d" % s)
def test_q8check_edges(pkb, cuda_device, shape):
    got, want = run_host_case(pkb, C.q8check_case(*shape))
    assert same_bits(got, want), first_diff(got, want)  # the floats between columns too


@pytest.mark.parametrize("rmode", [O.RD, O.RU, O.RZ])
@pytest.mark.parametrize("shape", C.q8check_mode_shapes(), ids=lambda s: "n%d-qb%d-T%d-f%d" % s)
def test_q8check_rounding_modes(pkb, cuda_device, shape, rmode):
    got, want = run_host_case(pkb, C.q8check_case(*shape), rmode)
    assert same_bits(got, want), first_diff(got, want)


def test_no_columns(pkb, cuda_device):
    out = np.array([-0.0], np.float32)
    lib = pkb.lib()
    rc = lib.pkb_gemm_q8_host(out.ctypes.data, 16, None, None, None, 16, None, None, 32, 32, 0, 0, 0)
    assert rc == 0 and out.tobytes() == np.array([-0.0], np.float32).tobytes()
    rc = lib.pkb_quantize_host(None, None, 32, 32, 0, None, 32, 0)
    assert rc == 0


RANDOM = [(rows, n, T, qb, add, bias)
          for i, (rows, n, T, qb) in enumerate([
              (16, 32, 1, 32), (48, 64, 7, 32), (64, 96, 13, 96), (32, 256, 37, 32), (384, 640, 3, 640),
              (64, 1024, 20, 32), (208, 1024, 1, 1024), (64, 4096, 9, 32), (16, 4096, 37, 4096),
              (128, 1024, 129, 64), (256, 256, 200, 64), (48, 640, 31, 64), (64, 4096, 48, 64),
              (32, 1024, 193, 32), (16, 4096, 101, 4096), (2048, 1024, 5, 32)])
          for add in (0, 1) for bias in (0, 1) if (i + add + bias) % 2 == 0 or T == 1]


@pytest.mark.parametrize("rows,n,T,qb,add,bias", RANDOM)
def test_random_products(pkb, cuda_device, rows, n, T, qb, add, bias):
    c = C.random_gemm_case(rows * 31 + n + T * 7 + qb + add * 3 + bias, rows, n, T, qb, bool(add), bool(bias))
    r0, nr = c["r0"], rows - c["r0"]
    got = c["out"].copy()
    b = None if c["bias_full"] is None else c["bias_full"][r0:]
    pkb.gemm_q8_host(got[r0:], c["os"], c["w_full"][r0 * n:], c["ws_full"][r0:], b, nr, c["q"], c["d"], n, qb, T,
                     bool(add))
    want = C.gemm_oracle(c)
    assert same_bits(got, want), first_diff(got, want)


def test_one_column_reads_no_stride(pkb, cuda_device):
    """The reference's decoder quantizes and multiplies one column at a time
    with output stride 0 (core/decoder.c:53-63): the contract's out[t os + r]
    and x + t xs read no stride for t = 0, so any stride is accepted there,
    on host and device buffers."""
    import torch
    n, rows, qb = 640, 2560, 640
    x = O.seeded_normal(n, 41)
    q, d = pkb.quantize_host(x, n, qb, T=1, xs=0)
    qo, do = O.quantize(x, n, qb)
    assert np.array_equal(q, qo) and same_bits(d, do)
    w = O.pack_q8(O.uniform_weights(rows, n, 42))
    ws = np.linspace(1e-3, 1e-2, rows).astype(np.float32)
    b = np.linspace(-1, 1, rows).astype(np.float32)
    want = np.full(rows, 3.0, np.float32)
    O.gemm_q8(want, rows, w, ws, b, rows, qo, do, n, qb, 1, True)
    got = np.full(rows, 3.0, np.float32)
    pkb.gemm_q8_host(got, 0, w, ws, b, rows, q, d, n, qb, 1, True)
    assert same_bits(got, want), first_diff(got, want)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    wp = torch.empty(rows * n, dtype=torch.int8, device="cuda")
    pkb.repack_q8_dev(wp, dev(w), rows, n)
    out = torch.full((rows,), 3.0, device="cuda")
    pkb.gemm_q8_dev(out, 0, wp, dev(ws), dev(b), rows, dev(qo), dev(do), n, qb, 1, True)
    torch.cuda.synchronize()
    assert same_bits(out.cpu().numpy(), want)


def test_table_entry(pkb, cuda_device):
    """pk_kernels_cuda_b200, called as the reference's passes call a backend."""
    tab = pkb.Table()
    assert tab.id == "cuda-b200"
    T, n, qb, rows = 37, 1024, 32, 64
    x = O.seeded_normal(T * n, 11)
    q = np.zeros(T * n, np.int8)
    d = np.zeros(T * n // qb, np.float32)
    act = pkb.PkAct(q.ctypes.data, d.ctypes.data, n, qb, T)
    tab.quantize(act, x, n)
    qo, do = O.quantize(x, n, qb)
    assert np.array_equal(q.reshape(T, n), qo) and same_bits(d.reshape(T, -1), do)
    w = O.pack_q8(O.uniform_weights(rows, n, 3))
    ws = np.linspace(1e-3, 1e-2, rows).astype(np.float32)
    out = np.full(T * rows, 7.0, np.float32)
    tab.gemm_q8(out, rows, w, ws, None, rows, act, True)
    want = np.full(T * rows, 7.0, np.float32)
    O.gemm_q8(want, rows, w, ws, None, rows, qo, do, n, qb, T, True)
    assert same_bits(out, want), first_diff(out, want)


def test_weights_changed_in_place(pkb, cuda_device):
    """A matrix rewritten at the same host address is uploaded again."""
    T, n, qb, rows = 9, 256, 32, 32
    x = O.seeded_normal(T * n, 2)
    q, d = O.quantize(x, n, qb)
    w = O.pack_q8(O.uniform_weights(rows, n, 4))
    ws = np.full(rows, 0.01, np.float32)
    for seed in (4, 5):
        w[:] = O.pack_q8(O.uniform_weights(rows, n, seed))
        got = np.zeros(T * rows, np.float32)
        pkb.gemm_q8_host(got, rows, w, ws, None, rows, q, d, n, qb, T, False)
        want = np.zeros(T * rows, np.float32)
        O.gemm_q8(want, rows, w, ws, None, rows, q, d, n, qb, T, False)
        assert same_bits(got, want)
    pkb.forget(w)


@pytest.mark.parametrize("T,rows,n,qb", [(750, 4096, 1024, 32), (750, 1024, 4096, 64), (1499, 1024, 1024, 32),
                                         (300, 640, 1024, 1024)])
def test_device_path_full_layer_shapes(pkb, cuda_device, T, rows, n, qb):
    """Encoder shapes at a minute of audio (T = 750, the position table's
    1499), on device buffers, against the oracle."""
    import torch
    x = O.seeded_normal(T * n, T + rows)
    q, d = O.quantize(x, n, qb)
    w_pk = O.pack_q8(O.uniform_weights(rows, n, rows + n))
    ws = (1e-3 + 9e-3 * np.random.default_rng(rows).random(rows)).astype(np.float32)
    bias = np.random.default_rng(n).standard_normal(rows).astype(np.float32)
    out0 = np.random.default_rng(T).standard_normal(T * rows).astype(np.float32)
    add = qb != 32
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    wpack = torch.empty(rows * n, dtype=torch.int8, device="cuda")
    pkb.repack_q8_dev(wpack, dev(w_pk), rows, n)
    out = dev(out0)
    pkb.gemm_q8_dev(out, rows, wpack, dev(ws), dev(bias), rows, dev(q), dev(d), n, qb, T, add)
    torch.cuda.synchronize()
    assert pkb.device_errors(0) == 0
    got = out.cpu().numpy()
    want = out0.copy()
    O.gemm_q8(want, rows, w_pk, ws, bias, rows, q, d, n, qb, T, add)
    assert same_bits(got, want), first_diff(got, want)


# ------------------------------------------------ page-locked host buffers --

def pinned_like(a: np.ndarray) -> tuple[object, np.ndarray]:
    """a copy of a in page-locked host memory (the tensor keeps it alive)"""
    import torch
    t = torch.empty(a.size, dtype={np.dtype(np.float32): torch.float32, np.dtype(np.int8): torch.int8}[a.dtype],
                    pin_memory=True)
    v = t.numpy()
    v[:] = a.reshape(-1)
    return t, v


@pytest.mark.parametrize("rmode", [O.RN, O.RU])
@pytest.mark.parametrize("os_,add", [(272, 1), (256, 1), (256, 0)])
def test_host_calls_on_page_locked_buffers(pkb, cuda_device, rmode, os_, add):
    """Page-locked activations and results take the direct-DMA path (no
    host staging): several chunks; a strided output with the floats between
    rows untouched, or rows back to back; a product that adds to its output
    or overwrites it, with bias; the same bytes as the oracle."""
    lib = pkb.lib()
    T, n, qb, xs, rows = 40000, 1024, 32, 1040, 256
    g = np.random.default_rng(17 + rmode)
    x = g.standard_normal(T * xs).astype(np.float32)
    keep_x, xp = pinned_like(x)
    keep_q, qp = pinned_like(np.zeros(T * n, np.int8))
    keep_d, dp = pinned_like(np.zeros(T * n // qb, np.float32))
    assert lib.pkb_quantize_host(qp.ctypes.data, dp.ctypes.data, n, qb, T, xp.ctypes.data, xs, rmode) == 0
    qo, do = O.quantize(x, n, qb, T=T, xs=xs, rmode=rmode)
    assert np.array_equal(qp.reshape(T, n), qo) and same_bits(dp.reshape(T, -1), do)
    w_rm = g.integers(-127, 128, (rows, n), dtype=np.int8)
    w = O.pack_q8(w_rm)
    ws = (1e-3 + 9e-3 * g.random(rows)).astype(np.float32)
    bias = g.standard_normal(rows).astype(np.float32)
    out0 = g.standard_normal(T * os_).astype(np.float32)
    keep_o, op = pinned_like(out0)
    assert lib.pkb_gemm_q8_host(op.ctypes.data, os_, w.ctypes.data, ws.ctypes.data, bias.ctypes.data, rows,
                                qp.ctypes.data, dp.ctypes.data, n, qb, T, add, rmode) == 0
    want = out0.copy()
    O.gemm_q8(want, os_, w, ws, bias, rows, qo, do, n, qb, T, bool(add), rmode)
    assert same_bits(op, want), first_diff(op, want)
    pkb.forget(w)


# -------------------------------------------- the decoder's products, batched --

# The TDT decoder's int8 products (core/decoder.c:53-79, 149-156) with T the
# number of segments stepped in lockstep: each LSTM layer's wx and wh
# (4P x P, the second added to the first), jpred (J x P, bias), jout
# (vocab + 1 + durations, padded to 16, x J, bias), every input a whole row a
# block (qb = n); and jenc (J x D, qb = D, bias) over a chunk's frames.
DECODER = [(2560, 640, 640, 0, 0), (2560, 640, 640, 1, 0), (640, 640, 640, 0, 1), (8208, 640, 640, 0, 1),
           (640, 1024, 1024, 0, 1)]


@pytest.mark.parametrize("T", [1, 7, 64])
@pytest.mark.parametrize("rows,n,qb,add,bias", DECODER)
def test_decoder_products_batched(pkb, cuda_device, rows, n, qb, add, bias, T):
    import torch
    g = np.random.default_rng(rows + n + T + add)
    x = (g.standard_normal(T * n) * 3).astype(np.float32)
    qo, do = O.quantize(x, n, qb)
    w_rm = g.integers(-127, 128, (rows, n), dtype=np.int8)
    w = O.pack_q8(w_rm)
    ws = (1e-3 + 9e-3 * g.random(rows)).astype(np.float32)
    b = g.standard_normal(rows).astype(np.float32) if bias else None
    out0 = g.standard_normal(T * rows).astype(np.float32)
    want = out0.copy()
    O.gemm_q8(want, rows, w, ws, b, rows, qo, do, n, qb, T, bool(add))
    # on the device: quantize, repack, product, as a decode step runs them
    xd = torch.from_numpy(x).cuda()
    q = torch.empty(T * n, dtype=torch.int8, device="cuda")
    d = torch.empty(T * n // qb, dtype=torch.float32, device="cuda")
    pkb.quantize_dev(q, d, xd, n, T, n, qb)
    wp = torch.empty(rows * n, dtype=torch.int8, device="cuda")
    pkb.repack_q8_dev(wp, torch.from_numpy(w).cuda(), rows, n)
    out = torch.from_numpy(out0).cuda()
    pkb.gemm_q8_dev(out, rows, wp, torch.from_numpy(ws).cuda(), None if b is None else torch.from_numpy(b).cuda(),
                    rows, q, d, n, qb, T, bool(add))
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy().reshape(T, n), qo) and same_bits(d.cpu().numpy().reshape(T, -1), do)
    got = out.cpu().numpy()
    assert same_bits(got, want), first_diff(got, want)


# ------------------------------------------------- the attention's panels --

PANELS = [(37, 256, 1024, 32, 64, 48), (750, 1024, 1024, 32, 128, 752), (1499, 1024, 1024, 32, 128, 1520),
          (129, 128, 256, 64, 32, 144), (5, 64, 640, 640, 16, 16),
          (1407, 256, 1024, 32, 128, 1424),  # P's padding reaching a tile past the frames
          (100, 144, 512, 32, 48, 112),  # heads of 48: a group of 32 columns spans two heads; rows % 32 = 16
          (300, 80, 256, 32, 16, 336)]  # heads of 16, padding past a whole panel of frames


@pytest.mark.parametrize("T,rows,n,qb,dk,tpad", PANELS)
@pytest.mark.parametrize("rmode", [O.RN, O.RZ])
@pytest.mark.parametrize("off", [0, 1])
def test_product_into_panels(pkb, cuda_device, T, rows, n, qb, dk, tpad, rmode, off):
    """The product straight into the attention's panels: K/P as
    pk_panels_tile lays them (from the product's rows, padding zeros), V as
    pk_gemm_panels_on's one call a 16-row panel; the floats beyond V's
    panels (ps > 16 T) untouched. off 0: 16-byte aligned panels, the TMA
    stores of panel-shaped maps where n / qb is a multiple of 4; off 1: the
    panels one float in, the plain-store path."""
    import torch
    g = np.random.default_rng(T + rows + dk + rmode)
    x = g.standard_normal(T * n).astype(np.float32)
    qo, do = O.quantize(x, n, qb)
    w = O.pack_q8(g.integers(-127, 128, (rows, n), dtype=np.int8))
    ws = (1e-3 + 9e-3 * g.random(rows)).astype(np.float32)
    ws[::5] *= -1  # negative row scales: padding must still be +0
    plain = np.zeros(T * rows, np.float32)
    O.gemm_q8(plain, rows, w, ws, None, rows, qo, do, n, qb, T, False, rmode)
    want_kp = O.panels_kp(plain, T, tpad, rows, dk)
    ps = 16 * T + 48
    want_v = np.full((rows // 16 - 1) * ps + 16 * T + 48, 7.5, np.float32)
    got_v_oracle = O.panels_v(w, ws, rows, qo, do, n, qb, T, ps, rmode)
    for r in range(0, rows, 16):
        want_v[(r // 16) * ps:(r // 16) * ps + 16 * T] = got_v_oracle[(r // 16) * ps:(r // 16) * ps + 16 * T]
    qd, dd = torch.from_numpy(qo.reshape(-1)).cuda(), torch.from_numpy(do.reshape(-1)).cuda()
    wp = torch.empty(rows * n, dtype=torch.int8, device="cuda")
    pkb.repack_q8_dev(wp, torch.from_numpy(w).cuda(), rows, n)
    wsd = torch.from_numpy(ws).cuda()
    kp = torch.full((want_kp.size + off,), float("nan"), device="cuda")[off:]
    pkb.gemm_q8_panels_dev(kp, pkb.PANELS_KP, 0, dk, tpad, wp, wsd, rows, qd, dd, n, qb, T, rmode)
    vp = torch.full((want_v.size + off,), 7.5, device="cuda")[off:]
    pkb.gemm_q8_panels_dev(vp, pkb.PANELS_V, ps, 0, 0, wp, wsd, rows, qd, dd, n, qb, T, rmode)
    torch.cuda.synchronize()
    assert pkb.device_errors(0) == 0
    got_kp, got_v = kp.cpu().numpy(), vp.cpu().numpy()
    assert same_bits(got_kp, want_kp), first_diff(got_kp, want_kp)
    assert same_bits(got_v, want_v), first_diff(got_v, want_v)


# ------------------------------------------ blocks of whole stages (WIDE) --

WIDE = [(300, 640, 1024, 1024, 0, 1), (129, 256, 512, 256, 1, 0), (1500, 384, 2048, 512, 1, 1),
        (64, 8208, 640, 640, 0, 1), (257, 128, 1536, 384, 0, 0), (700, 512, 4096, 2048, 1, 0)]


@pytest.mark.parametrize("T,rows,n,qb,add,bias", WIDE)
@pytest.mark.parametrize("rmode", [O.RN, O.RD, O.RU, O.RZ])
@pytest.mark.parametrize("off", [0, 1])
def test_wide_blocks_on_device(pkb, cuda_device, T, rows, n, qb, add, bias, rmode, off):
    """Blocks that span whole TMA boxes of K (qb = 256, 384, ... n: the
    decoder's and the joint's products take qb = n), on the staged path that
    issues a stage's four K steps unrolled into one accumulator; off 0 with
    the results through TMA stores, off 1 (the results one float in) through
    plain stores. Every rounding mode, against the oracle."""
    import torch
    g = np.random.default_rng(T + rows + n + qb + add + rmode)
    x = (g.standard_normal(T * n) * 2).astype(np.float32)
    qo, do = O.quantize(x, n, qb, rmode=rmode)
    w = O.pack_q8(g.integers(-128, 128, (rows, n), dtype=np.int8))
    ws = (1e-3 + 9e-3 * g.random(rows)).astype(np.float32)
    ws[::7] *= -1
    b = g.standard_normal(rows).astype(np.float32) if bias else None
    out0 = g.standard_normal(T * rows + off).astype(np.float32)
    want = out0.copy()
    O.gemm_q8(want[off:], rows, w, ws, b, rows, qo, do, n, qb, T, bool(add), rmode=rmode)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    wp = torch.empty(rows * n, dtype=torch.int8, device="cuda")
    pkb.repack_q8_dev(wp, dev(w), rows, n)
    out = dev(out0)
    pkb.gemm_q8_dev(out[off:], rows, wp, dev(ws), None if b is None else dev(b), rows, dev(qo), dev(do), n, qb, T,
                    bool(add), rmode=rmode)
    torch.cuda.synchronize()
    assert pkb.device_errors(0) == 0
    got = out.cpu().numpy()
    assert same_bits(got, want), first_diff(got, want)
