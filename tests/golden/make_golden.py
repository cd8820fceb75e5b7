"""Writes tests/golden/q8_golden.npz: outputs of the reference's own `ref`
backend (backend/ref/kernels.c, compiled from the reference's sources by
oracle/Makefile into oracle/_ref/libpkref.so) on the cases below.

    make -C oracle ref && python tests/golden/make_golden.py

Needs the reference's sources (only in the build container); the fixture it
writes is committed, so the tests that read it run anywhere.

Cases:
  qc/*   quantize, RN: awkward values (zeros of both signs, subnormals,
         x30 outliers, ties), a zero block, column strides n and n+32,
         blocks of 32, 64 and a whole column (tests/kcheck.c:98-118, 496-504)
  qx/*   quantize of non-finite inputs and of blocks either side of 2^-121
         (tests/kcheck.c:120-175)
  g8/*   every product of tests/q8check.c's edge set (tests/cases.py
         q8check_case regenerates the inputs; only outputs are stored), RN,
         plus its rounding-mode cases under RD, RU, RZ
  gr/*   random products on awkward values, runs of panels from the middle
         (tests/kcheck.c:183-216), inputs and outputs stored
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from tests import cases as C  # noqa: E402

OUT = os.path.join(HERE, "q8_golden.npz")

QUANT = [(1, 32, 32, 32), (3, 64, 32, 96), (20, 1024, 32, 1056), (7, 640, 640, 640), (11, 256, 64, 288),
         (5, 4096, 32, 4096), (2, 96, 96, 128), (16, 128, 64, 128), (9, 1024, 1024, 1024), (4, 16384, 32, 16384)]

RANDOM = [(16, 32, 1, 32, 0, 1), (48, 64, 7, 32, 1, 0), (64, 96, 13, 96, 0, 0), (32, 256, 37, 32, 1, 1),
          (384, 640, 3, 640, 0, 1), (64, 1024, 20, 32, 1, 0), (208, 1024, 1, 1024, 0, 0), (64, 4096, 9, 32, 1, 1),
          (16, 4096, 37, 4096, 0, 1), (128, 1024, 29, 64, 1, 0), (48, 640, 31, 64, 0, 1), (32, 1024, 49, 64, 1, 1)]


def main() -> None:
    if not O.have_ref():
        raise SystemExit("oracle/_ref/libpkref.so is not built: make -C oracle ref")
    g: dict[str, np.ndarray] = {}

    for i, (T, n, qb, xs) in enumerate(QUANT):
        rng = O.XorShift(0xC0FFEE + i)
        x = C.awkward_array(rng, T * xs + n, 1e4 if i % 3 == 0 else 1.0)
        if i % 2:
            x[:qb] = 0.0
        q, d = O.ref_quantize(x, n, qb, T=T, xs=xs)
        g[f"qc/{i}/shape"] = np.array([T, n, qb, xs], np.int64)
        g[f"qc/{i}/x"], g[f"qc/{i}/q"], g[f"qc/{i}/d"] = x, q, d

    xr = O.XorShift(31)
    x = np.array([xr.frand() for _ in range(128)], np.float32)
    x[3], x[40], x[69], x[109] = np.nan, np.inf, -np.inf, np.nan
    q, d = O.ref_quantize(x, 64, 32)
    g["qx/nonfinite/x"], g["qx/nonfinite/q"], g["qx/nonfinite/d"] = x, q, d
    tops = np.array([2.0**-140, 2.0**-130, 2.0**-122, np.float32(float.fromhex('0x1.fffffep-122')), 2.0**-121, 2.0**-120,
                     2.0**-100], np.float32)
    n = 32 * len(tops)
    x = np.empty(2 * n, np.float32)
    for t in range(2):
        for b, top in enumerate(tops):
            v = np.array([top * np.float32(xr.frand()) for _ in range(32)], np.float32)
            v[xr.rnd() % 32] = -top if t else top
            x[t * n + 32 * b: t * n + 32 * b + 32] = v
    q, d = O.ref_quantize(x, n, 32)
    g["qx/tiny/x"], g["qx/tiny/q"], g["qx/tiny/d"] = x, q, d

    for j, shape in enumerate(C.q8check_shapes()):
        c = C.q8check_case(*shape)
        o = c["out"].copy()
        O.ref_gemm_q8(o, c["os"], c["w"], c["ws"], c["bias"], c["rows"], c["q"], c["d"], c["n"], c["qb"], c["T"],
                      c["add"])
        g[f"g8/{j}/shape"], g[f"g8/{j}/rmode"], g[f"g8/{j}/out"] = np.array(shape, np.int64), np.array(O.RN), o
    j = len(C.q8check_shapes())
    for rmode in (O.RD, O.RU, O.RZ):
        for shape in C.q8check_mode_shapes():
            c = C.q8check_case(*shape)
            o = c["out"].copy()
            O.ref_gemm_q8(o, c["os"], c["w"], c["ws"], c["bias"], c["rows"], c["q"], c["d"], c["n"], c["qb"],
                          c["T"], c["add"], rmode)
            g[f"g8/{j}/shape"], g[f"g8/{j}/rmode"], g[f"g8/{j}/out"] = np.array(shape, np.int64), np.array(rmode), o
            j += 1

    for i, (rows, n, T, qb, add, bias) in enumerate(RANDOM):
        c = C.random_gemm_case(1000 + i, rows, n, T, qb, bool(add), bool(bias))
        r0 = c["r0"]
        o = c["out"].copy()
        b = None if c["bias_full"] is None else c["bias_full"][r0:]
        O.ref_gemm_q8(o[r0:], c["os"], c["w_full"][r0 * n:], c["ws_full"][r0:], b, rows - r0, c["q"], c["d"], n, qb,
                      T, bool(add))
        p = f"gr/{i}/"
        g[p + "meta"] = np.array([rows, n, T, qb, add, bias, r0, c["os"]], np.int64)
        g[p + "w"], g[p + "ws"], g[p + "q"], g[p + "d"] = c["w_full"], c["ws_full"], c["q"], c["d"]
        g[p + "bias"] = c["bias_full"] if c["bias_full"] is not None else np.zeros(0, np.float32)
        g[p + "out_in"], g[p + "out"] = c["out"], o

    np.savez_compressed(OUT, **g)
    print(f"{OUT}: {len(g)} arrays, {os.path.getsize(OUT) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
