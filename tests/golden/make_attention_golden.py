"""Writes tests/golden/attention_golden.npz: the reference's own ref backend
(oracle/_ref/libpkref.so, compiled from its sources by oracle/Makefile) on
the attention's float work, round to nearest:

    make -C oracle ref && python tests/golden/make_attention_golden.py

* gemm_f32: k_gemm_f32 (backend/ref/kernels.c:90-105) on cases drawn as
  its tests/kcheck.c draws them (:545-556: rows, ld, the run's first k, n,
  T, xs, no bias / one bias / a bias a column, ReLU), awkward values.
* softmax: k_softmax (backend/ref/kernels.c:134-147) on rows of 1 to 700
  awkward scores (kcheck.c:511-516).
* attention: att_item (core/encoder.c:280-326) as the reference runs it
  (oracle.ref_attention: its gemm_f32 and softmax called in att_item's
  order, blocks of 16 queries, the position window from a panel boundary)
  on seeded q, K/P/V panels (their padding zeros) and position biases.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "attention_golden.npz")

# T, D, H
ATT = [(1, 64, 2), (5, 64, 1), (16, 128, 4), (17, 64, 2), (40, 256, 2), (33, 96, 2)]


def att_inputs(T: int, D: int, H: int, seed: int):
    """q rows, K/P panels (frames past T, positions past 2T-1 zero), V panels, biases."""
    g = np.random.default_rng(seed)
    dk = D // H
    Tp, R = (T + 15) // 16 * 16, 2 * T - 1
    Pp = (R + 15) // 16 * 16 + 16
    q = g.standard_normal(T * D).astype(np.float32)
    k = g.standard_normal(T * D).astype(np.float32)
    p = g.standard_normal(R * D).astype(np.float32)
    v = g.standard_normal(T * D).astype(np.float32)
    kp = O.panels_kp(k, T, Tp, D, dk)
    pp = O.panels_kp(p, R, Pp, D, dk)
    # V as 16-row panels of T frames: (t, r) at (r/16) 16 T + 16 t + r%16
    vp = np.ascontiguousarray(v.reshape(T, D // 16, 16).transpose(1, 0, 2)).reshape(-1)
    bu = (g.standard_normal(D) * 0.1).astype(np.float32)
    bv = (g.standard_normal(D) * 0.1).astype(np.float32)
    return q, kp, pp, vp, bu, bv


def gemm_f32_cases():
    """(meta, w, x, b) of the gemm_f32 cases, the same on every run: meta =
    (rows, ld, k0, n, T, xs, bias kind, relu, os)."""
    r = O.XorShift(0x51F15E)
    for _ in range(40):
        rows = 16 * (1 + r.rnd() % 12)
        ld = 1 + r.rnd() % 200
        k0 = r.rnd() % ld
        n = 1 + r.rnd() % (ld - k0)
        T = 1 + r.rnd() % 23
        xs = n + r.rnd() % 9
        bias_kind = r.rnd() % 3
        relu = r.rnd() % 2
        os_ = rows + 16 * (r.rnd() % 2)
        w = np.array([r.awkward(1.0) for _ in range(ld * rows)], np.float32)
        x = np.array([r.awkward(1.0) for _ in range(T * xs + n)], np.float32)
        b = np.array([r.awkward(2.0) for _ in range(T * os_ + rows)], np.float32)
        yield (rows, ld, k0, n, T, xs, bias_kind, relu, os_), w, x, b


def softmax_cases():
    """rows of awkward scores, the same on every run"""
    r = O.XorShift(0x50F7)
    for i in range(24):
        m = 1 + r.rnd() % 700
        yield np.array([r.awkward(20.0 if i % 3 else 400.0) for _ in range(m)], np.float32)


def run_gemm_f32(fn, meta, w, x, b) -> np.ndarray:
    """one case through fn (oracle.gemm_f32 or oracle.ref_gemm_f32): out
    starts as the bias array, so that a bias a column is out itself"""
    rows, ld, k0, n, T, xs, bias_kind, relu, os_ = meta
    out = b.copy()
    bias = (out if bias_kind == 2 else b) if bias_kind else None
    fn(out, os_, w, ld, rows, n, x, xs, T, bias, os_ if bias_kind == 2 else 0, bool(relu), w_off=16 * k0)
    return out


def main() -> None:
    if not O.have_ref():
        raise SystemExit("oracle/_ref/libpkref.so is not built: make -C oracle ref")
    g: dict[str, np.ndarray] = {}
    for i, (meta, w, x, b) in enumerate(gemm_f32_cases()):
        g[f"gf/{i}/out"] = run_gemm_f32(O.ref_gemm_f32, meta, w, x, b)
    for i, s in enumerate(softmax_cases()):
        O.ref_softmax(s, s.size, 1, s.size, 0.0883883476)
        g[f"sm/{i}/y"] = s
    for i, (T, D, H) in enumerate(ATT):
        q, kp, pp, vp, bu, bv = att_inputs(T, D, H, 300 + i)
        g[f"att/{i}/o"] = O.ref_attention(q, D, kp, pp, vp, bu, bv, T, D, H)
    np.savez_compressed(OUT, **g)
    print(f"{OUT}: {len(g)} arrays, {os.path.getsize(OUT) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
