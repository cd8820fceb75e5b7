"""Parity cases shared by the CPU and GPU tests: inputs built the way the
reference's own checks build theirs (tests/q8check.c:83-161,
tests/kcheck.c:96-241, 496-577), restated here as data generators."""
from __future__ import annotations

import numpy as np

from oracle import oracle as O


def q8check_case(n: int, qb: int, T: int, flags: int):
    """The int8 product at its edges (tests/q8check.c:83-129): 32 rows whose
    weights are all -128, all 127, or alternate (127, -127) / (127, -128);
    activations of +-127 patterns; block scales with zeros every fifth;
    row scales +-1/32 alternating; biases (r % 7) - 3.25; 35 floats between
    output columns, pre-set to 0.125 / -0 alternating. flags & 1: bias,
    flags & 2: add."""
    rows, os_ = 32, 35
    nb = n // qb
    w_rm = np.empty((rows, n), np.int8)
    k = np.arange(n)
    for r in range(rows):
        if r % 4 == 0:
            w_rm[r] = -128
        elif r % 4 == 1:
            w_rm[r] = 127
        elif r % 4 == 2:
            w_rm[r] = np.where(k % 2 == 1, -127, 127)
        else:
            w_rm[r] = np.where(k % 2 == 1, -128, 127)
    q = np.empty((T, n), np.int8)
    d = np.empty((T, nb), np.float32)
    for t in range(T):
        q[t] = 127 if t % 3 == 0 else (-127 if t % 3 == 1 else np.where(k % 2 == 1, -127, 127))
        for b in range(nb):
            d[t, b] = np.float32(0.0) if (b + t) % 5 == 0 else np.float32((b + t) % 13 + 1) / np.float32(127.0)
    ws = np.array([(-1 if r % 2 else 1) * 0.03125 for r in range(rows)], np.float32)
    bias = np.array([(r % 7) - 3.25 for r in range(rows)], np.float32)
    out = np.array([-0.0 if i % 2 else 0.125 for i in range(T * os_)], np.float32)
    return dict(w=O.pack_q8(w_rm), ws=ws, bias=bias if flags & 1 else None, rows=rows, os=os_,
                q=q, d=d, n=n, qb=qb, T=T, add=bool(flags & 2), out=out)


def q8check_shapes():
    """(n, qb, T, flags) of tests/q8check.c:131-145 in RN."""
    out = []
    for n in (32, 64, 96, 128, 1024, 4096):
        for qb in (32, 64):
            if n % qb == 0:
                for T in range(1, 10):
                    for f in range(4):
                        out.append((n, qb, T, f))
    for qb in (32, 64):
        out += [(4096, qb, 49, 3), (4096, qb, 50, 3), (1024, qb, 193, 3), (1024, qb, 194, 3),
                (16384, qb, 13, 3), (16384, qb, 14, 3)]
    return out


def q8check_mode_shapes():
    """the rounding-mode cases of tests/q8check.c:146-155"""
    return [(128, 32, 5, 0), (128, 64, 5, 3), (128, 32, 37, 0), (128, 64, 37, 3)]


def awkward_array(rng: O.XorShift, count: int, scale: float) -> np.ndarray:
    return np.array([rng.awkward(scale) for _ in range(count)], np.float32)


def random_gemm_case(seed: int, rows: int, n: int, T: int, qb: int, add: bool, bias: bool, sliced: bool = True):
    """kcheck's random product (tests/kcheck.c:183-216): weights uniform in
    [-127, 127] with 127 a third of the time, some zero row scales,
    awkward biases and activations (quantized by the oracle), an output
    stride of rows or rows + 16, and a run of panels from the middle."""
    g = np.random.default_rng(seed)
    w_rm = np.where(g.integers(0, 3, (rows, n)) > 0, g.integers(-127, 128, (rows, n)), 127).astype(np.int8)
    ws = np.where(g.integers(0, 8, rows) > 0, 0.01 * (g.random(rows) * 2 - 1 + 1.5), 0.0).astype(np.float32)
    xr = O.XorShift(seed * 2654435761 + 1)
    b = awkward_array(xr, rows, 1.0)
    x = awkward_array(xr, T * n, 2.0)
    q, d = O.quantize(x, n, qb)
    os_ = rows + 16 * int(g.integers(0, 2))
    out = awkward_array(xr, T * os_, 1.0)
    r0 = 16 * int(g.integers(0, rows // 16)) if (sliced and rows > 16 and g.integers(0, 2)) else 0
    return dict(w_full=O.pack_q8(w_rm), w_rm=w_rm, ws_full=ws, bias_full=b if bias else None, rows_full=rows,
                r0=r0, os=os_, q=q, d=d, n=n, qb=qb, T=T, add=add, out=out)


def gemm_oracle(case, out=None, rmode=O.RN):
    """The oracle's answer for a random_gemm_case, on a copy of its output."""
    o = case["out"].copy() if out is None else out
    r0, n = case["r0"], case["n"]
    rows = case["rows_full"] - r0
    w = case["w_full"][r0 * n:]
    bias = None if case["bias_full"] is None else case["bias_full"][r0:]
    O.gemm_q8(o[r0:], case["os"], w, case["ws_full"][r0:], bias, rows, case["q"], case["d"], n, case["qb"],
              case["T"], case["add"], rmode)
    return o
