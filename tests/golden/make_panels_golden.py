"""Writes tests/golden/panels_golden.npz: the reference's own pk_panels_tile
(core/passes.c:169-196, compiled from its sources into
oracle/_ref/libpkpasses.so by oracle/Makefile) on seeded float matrices, as
the encoder makes K's and P's panels for the attention (core/encoder.c:
341-351: K with its frames rounded up to 16, P with its positions rounded up
to 16 plus 16, the rest zeros):

    make -C oracle ref && python tests/golden/make_panels_golden.py

Each case stores src [n][D], (n, np, D, dk) and the panels it wrote.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "panels_golden.npz")

# n, D, dk, extra panel (P's +16)
CASES = [(37, 256, 64, 0), (45, 128, 32, 1), (16, 64, 16, 0), (1, 32, 32, 1), (129, 256, 128, 1)]


def main() -> None:
    if not O.have_passes():
        raise SystemExit("oracle/_ref/libpkpasses.so is not built: make -C oracle ref")
    rng = np.random.default_rng(77)
    g: dict[str, np.ndarray] = {}
    for i, (n, D, dk, extra) in enumerate(CASES):
        np_ = (n + 15) // 16 * 16 + 16 * extra
        src = rng.standard_normal(n * D).astype(np.float32)
        g[f"kp/{i}/meta"] = np.array([n, np_, D, dk], np.int64)
        g[f"kp/{i}/src"] = src
        g[f"kp/{i}/dst"] = O.ref_panels_kp(src, n, np_, D, dk)
    np.savez_compressed(OUT, **g)
    print(f"{OUT}: {len(g)} arrays, {os.path.getsize(OUT) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
