"""Writes tests/golden/producers_golden.npz: outputs of the reference's own
`ref` backend (oracle/_ref/libpkref.so, compiled from the reference's
sources by oracle/Makefile) for the encoder's three producers of int8
inputs, composed as the encoder composes them (oracle.ref_*):

    make -C oracle ref && python tests/golden/make_producers_golden.py

Cases (inputs and outputs stored; each case in the rounding mode it names):
  ln/*   normq (core/encoder.c:112-130): k_layernorm then pk_quant_part, on
         rows with a constant row (variance 0), a NaN, an infinity, values
         near 1e30 (sums overflow), near 1e-30 (the variance underflows to
         eps alone), subnormals; w and b with zeros and negatives
  si/*   siluq_tile (core/encoder.c:150-158): k_silu then pk_quant_part, on
         values across the exp clamp (+-87, +-88), +-0, +-inf, NaN,
         subnormals, large and tiny blocks
  dw/*   glu_item + dw_item (core/encoder.c:160-183): k_glu (when glu),
         k_dwconv per 64 channels, pk_quant_part per frame; T below and
         above K, an infinite tap weight, a NaN input frame; the
         convolution's floats are stored too

The reference's ref is built for baseline x86-64, where gcc's rintf rounds
|x| and puts the sign back; under RD and RU that differs from IEEE rint for
negative arguments (the exp's n, the quantizer's bytes), so the fixtures in
those modes are matched by the oracle's rint_style(), and the CUDA path is
held to them in RN and RZ.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "producers_golden.npz")

MODES = (O.RN, O.RD, O.RU, O.RZ)

# T, n, qb, xs, eps, modes
LN = [(3, 32, 32, 32, 1e-5, MODES), (9, 1024, 32, 1024, 1e-5, MODES), (4, 1024, 64, 1056, 1e-6, (O.RN,)),
      (2, 4096, 32, 4096, 1e-5, (O.RN, O.RZ)), (7, 96, 32, 96, 1e-3, MODES), (1, 8192, 64, 8192, 1e-5, (O.RN,))]
# T, n, qb, us, modes
SI = [(4, 64, 32, 64, MODES), (6, 4096, 32, 4096, (O.RN, O.RD)), (3, 1024, 64, 1088, MODES), (1, 32, 32, 32, MODES)]
# T, C, K, glu, qb, modes
DW = [(1, 32, 9, 0, 32, MODES), (5, 64, 9, 1, 64, MODES), (37, 96, 3, 0, 32, (O.RN, O.RU)),
      (20, 128, 31, 1, 32, (O.RN,)), (3, 1024, 9, 1, 64, (O.RN, O.RZ)), (12, 64, 1, 0, 64, MODES),
      (50, 256, 63, 1, 32, (O.RN,))]


def ln_rows(rng: np.random.Generator, T: int, xs: int, n: int) -> np.ndarray:
    x = (rng.standard_normal(T * xs + n) * rng.choice([0.1, 1.0, 10.0], T * xs + n) + rng.standard_normal()).astype(
        np.float32)
    kinds = ["const", "nan", "inf", "huge", "tiny", "sub"]
    for t in range(min(T, len(kinds)) if T > 2 else 0):
        r = x[t * xs: t * xs + n]
        k = kinds[t]
        if k == "const":
            r[:] = np.float32(3.25)
        elif k == "nan":
            r[rng.integers(n)] = np.nan
        elif k == "inf":
            r[rng.integers(n)] = -np.inf
        elif k == "huge":
            r *= np.float32(1e30)
        elif k == "tiny":
            r *= np.float32(1e-30)
        elif k == "sub":
            r[:] = (rng.standard_normal(n) * 1e-39).astype(np.float32)
    return x


def silu_rows(rng: np.random.Generator, T: int, us: int, n: int) -> np.ndarray:
    u = (rng.standard_normal(T * us + n) * 8).astype(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, 87.0, -87.0, 88.0, -88.0, 87.5, -87.5, 100.0, -100.0, 1e-40,
                        -1e-40, 1e-30, 20.0, -20.0, 0.5, -0.5], np.float32)
    idx = rng.integers(0, u.size, 3 * len(special))
    u[idx] = np.tile(special, 3)
    if T > 1:
        u[us + 5] = np.nan  # a block with a NaN: zeros
        u[:32] *= np.float32(1e-37)  # a block of tiny results
    return u


def main() -> None:
    if not O.have_ref():
        raise SystemExit("oracle/_ref/libpkref.so is not built: make -C oracle ref")
    g: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(2026)
    for i, (T, n, qb, xs, eps, modes) in enumerate(LN):
        x = ln_rows(rng, T, xs, n)
        w = rng.standard_normal(n).astype(np.float32)
        w[::7] = 0.0
        b = (rng.standard_normal(n) * 0.5).astype(np.float32)
        p = f"ln/{i}/"
        g[p + "meta"] = np.array([T, n, qb, xs], np.int64)
        g[p + "eps"] = np.array(eps, np.float32)
        g[p + "x"], g[p + "w"], g[p + "b"] = x, w, b
        for m in modes:
            q, d = O.ref_layernorm_quantize(x, xs, T, n, qb, w, b, eps, m)
            g[p + f"q{m}"], g[p + f"d{m}"] = q, d
    for i, (T, n, qb, us, modes) in enumerate(SI):
        u = silu_rows(rng, T, us, n)
        p = f"si/{i}/"
        g[p + "meta"] = np.array([T, n, qb, us], np.int64)
        g[p + "u"] = u
        for m in modes:
            q, d = O.ref_silu_quantize(u, us, T, n, qb, m)
            g[p + f"q{m}"], g[p + f"d{m}"] = q, d
    for i, (T, C, K, glu, qb, modes) in enumerate(DW):
        xs = (2 * C if glu else C) + (16 if i % 2 else 0)
        x = (rng.standard_normal(T * xs + 2 * C) * 2).astype(np.float32)
        w = (rng.standard_normal(C * K) * 0.4).astype(np.float32)
        b = (rng.standard_normal(C) * 0.3).astype(np.float32)
        if C >= 128:
            w[5 * K + K // 2] = np.inf  # channel 5's centre tap: its block of every frame is zeros
        if T > 8:
            x[3 * xs: 3 * xs + 8] = np.nan  # frame 3's first channels (or GLU values), reaching K frames
        p = f"dw/{i}/"
        g[p + "meta"] = np.array([T, C, K, glu, qb, xs], np.int64)
        g[p + "x"], g[p + "w"], g[p + "b"] = x, w, b
        for m in modes:
            q, d, out = O.ref_dwconv_quantize(x, xs, T, C, w, b, K, bool(glu), qb, m)
            g[p + f"q{m}"], g[p + f"d{m}"], g[p + f"o{m}"] = q, d, out
    np.savez_compressed(OUT, **g)
    print(f"{OUT}: {len(g)} arrays, {os.path.getsize(OUT) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
