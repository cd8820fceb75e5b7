"""Python access to the checkers: TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module. It wraps

* liboracle.so, the C restatement of the int8 path (oracle/q8_oracle.c), and
* _ref/libpkref.so, the reference's own backends compiled from its sources
  (oracle/Makefile), where it was built: ``ref_quantize``/``ref_gemm_q8``
  call its ``pk_kernels_ref`` table, the definition of correct
  (backend/ref/kernels.c);

plus the seeded generators the reference's tests use (tests/kcheck.c:40-60),
restated, so cases can be drawn the way the reference draws them.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
PKREF_SO = os.path.join(REF_DIR, "libpkref.so")

RN, RD, RU, RZ = 0, 1, 2, 3

_or = None
_ref = None


def reference_tree() -> Optional[str]:
    """The reference's source tree, where this machine has it: the
    PKTITO_REFERENCE environment variable, else the reference_path the
    checkout's BASELINE.json names; None where neither is a directory."""
    path = os.environ.get("PKTITO_REFERENCE")
    if not path:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                path = json.load(f).get("reference_path")
        except (OSError, ValueError):
            path = None
    return path if path and os.path.isdir(path) else None


def build() -> None:
    """liboracle.so always; the reference's code too where its sources are here."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    ref = reference_tree()
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref", "REF=" + ref], check=True)


def _p(a: Optional[np.ndarray]) -> int:
    return 0 if a is None else a.ctypes.data


def olib() -> ctypes.CDLL:
    global _or
    if _or is None:
        if not os.path.exists(ORACLE_SO):
            subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
        l = ctypes.CDLL(ORACLE_SO)
        vp, u32, sz = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_size_t
        l.oracle_quantize.argtypes = [vp, vp, vp, sz, u32, u32, u32, ctypes.c_int]
        l.oracle_gemm_q8.argtypes = [vp, sz, vp, vp, vp, u32, vp, vp, u32, u32, u32, ctypes.c_int, ctypes.c_int]
        l.oracle_pack_q8.argtypes = [vp, vp, u32, u32]
        l.oracle_unpack_q8.argtypes = [vp, vp, u32, u32]
        l.oracle_block_sums.argtypes = [vp, vp, u32, vp, u32, u32, u32]
        f32, i32 = ctypes.c_float, ctypes.c_int
        l.oracle_set_rint_style.argtypes = [i32]
        l.oracle_expf.argtypes = [vp, vp, sz, i32]
        l.oracle_sigmoidf.argtypes = [vp, vp, sz, i32]
        l.oracle_layernorm.argtypes = [vp, sz, vp, sz, u32, u32, vp, vp, f32, i32]
        l.oracle_layernorm_quantize.argtypes = [vp, vp, vp, sz, u32, u32, u32, vp, vp, f32, i32]
        l.oracle_silu_quantize.argtypes = [vp, vp, vp, sz, u32, u32, u32, i32]
        l.oracle_dwconv_quantize.argtypes = [vp, vp, vp, sz, vp, sz, u32, u32, vp, vp, u32, i32, u32, i32]
        l.oracle_panels_kp.argtypes = [vp, vp, u32, u32, u32, u32]
        l.oracle_panels_kp.restype = None
        l.oracle_gemm_f32.argtypes = [vp, sz, vp, u32, u32, u32, vp, sz, u32, vp, sz, i32, i32]
        l.oracle_softmax.argtypes = [vp, sz, u32, u32, f32, i32]
        l.oracle_attention.argtypes = [vp, sz, vp, sz, vp, vp, vp, vp, vp, u32, u32, u32, i32]
        for f in (l.oracle_gemm_f32, l.oracle_softmax, l.oracle_attention):
            f.restype = None
        l.oracle_tanhf.argtypes = [vp, vp, sz, i32]
        l.oracle_lstm.argtypes = [vp, vp, vp, u32, i32]
        l.oracle_tanhf.restype = l.oracle_lstm.restype = None
        l.oracle_tdt_search.argtypes = [vp, vp, vp, ctypes.c_long, vp, u32, ctypes.POINTER(_Tdt), i32]
        l.oracle_tdt_search.restype = ctypes.c_long
        for f in (l.oracle_set_rint_style, l.oracle_expf, l.oracle_sigmoidf, l.oracle_layernorm,
                  l.oracle_layernorm_quantize, l.oracle_silu_quantize, l.oracle_dwconv_quantize):
            f.restype = None
        for f in (l.oracle_quantize, l.oracle_gemm_q8, l.oracle_pack_q8, l.oracle_unpack_q8, l.oracle_block_sums):
            f.restype = None
        _or = l
    return _or


def have_ref() -> bool:
    return os.path.exists(PKREF_SO)


class _Act(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("d", ctypes.c_void_p),
                ("n", ctypes.c_uint32), ("qb", ctypes.c_uint32), ("T", ctypes.c_uint32)]


_QF = ctypes.CFUNCTYPE(None, ctypes.POINTER(_Act), ctypes.c_void_p, ctypes.c_size_t)
_GF = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                       ctypes.c_uint32, ctypes.POINTER(_Act), ctypes.c_int)


_F32F = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                         ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_void_p,
                         ctypes.c_size_t, ctypes.c_int)
_LNF = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32,
                        ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float)
_SMF = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float)
_ROWF = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_size_t)
_GLUF = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32,
                         ctypes.c_uint32)
_DWF = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32,
                        ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32)


class _Table(ctypes.Structure):
    """pk_kernels (backend/kernels.h:242-278) up to its dwconv entry."""
    _fields_ = [("id", ctypes.c_char_p), ("name", ctypes.c_char_p), ("needs", ctypes.c_void_p),
                ("competes", ctypes.c_int), ("quantize", _QF), ("gemm_q8", _GF), ("gemm_f32", _F32F),
                ("layernorm", _LNF), ("softmax", _SMF), ("silu", _ROWF), ("gelu", _ROWF), ("glu", _GLUF),
                ("dwconv", _DWF)]


def rlib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not have_ref():
            raise FileNotFoundError(PKREF_SO + " is not built (make -C oracle ref)")
        _ref = ctypes.CDLL(PKREF_SO)
    return _ref


# ---------------------------------------------------------------- restated --

def pack_q8(w_rm: np.ndarray) -> np.ndarray:
    """Plain rows [rows][n] int8 -> the PK_Q8 panel bytes (core/pkf.h:28-41)."""
    w_rm = np.ascontiguousarray(w_rm, np.int8)
    rows, n = w_rm.shape
    out = np.empty(rows * n, np.int8)
    olib().oracle_pack_q8(_p(out), _p(w_rm), rows, n)
    return out


def unpack_q8(w: np.ndarray, rows: int, n: int) -> np.ndarray:
    out = np.empty((rows, n), np.int8)
    olib().oracle_unpack_q8(_p(out), _p(np.ascontiguousarray(w, np.int8)), rows, n)
    return out


def quantize(x: np.ndarray, n: int, qb: int, T: Optional[int] = None, xs: Optional[int] = None,
             rmode: int = RN) -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    xs = n if xs is None else xs
    T = x.size // xs if T is None else T
    q = np.zeros((T, n), np.int8)
    d = np.zeros((T, n // qb), np.float32)
    olib().oracle_quantize(_p(q), _p(d), _p(x), xs, T, n, qb, rmode)
    return q, d


def gemm_q8(out: np.ndarray, os_: int, w: np.ndarray, ws: np.ndarray, bias: Optional[np.ndarray], rows: int,
            q: np.ndarray, d: np.ndarray, n: int, qb: int, T: int, add: bool, rmode: int = RN) -> None:
    assert out.dtype == np.float32 and out.flags.c_contiguous
    olib().oracle_gemm_q8(_p(out), os_, _p(w), _p(ws), _p(bias), rows, _p(q), _p(d), n, qb, T, int(add), rmode)


def block_sums(w: np.ndarray, rows: int, q: np.ndarray, n: int, qb: int, T: int) -> np.ndarray:
    s = np.empty((T, rows, n // qb), np.int32)
    olib().oracle_block_sums(_p(s), _p(w), rows, _p(q), n, qb, T)
    return s


class rint_style:
    """Within the block, the oracle's rintf rounds as gcc compiles it for
    baseline x86-64 (|x| in the mode, the sign put back: the reference's own
    ref build) instead of IEEE's rint; for holding the oracle to that build
    in the directed modes."""

    def __enter__(self):
        olib().oracle_set_rint_style(1)

    def __exit__(self, *exc):
        olib().oracle_set_rint_style(0)


def expf(x: np.ndarray, rmode: int = RN) -> np.ndarray:
    """pk_expf (core/vmath.h:134-147), elementwise."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    olib().oracle_expf(_p(y), _p(x), x.size, rmode)
    return y


def sigmoidf(x: np.ndarray, rmode: int = RN) -> np.ndarray:
    """pk_sigmoidf (core/vmath.h:149-151), elementwise."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    olib().oracle_sigmoidf(_p(y), _p(x), x.size, rmode)
    return y


def layernorm_quantize(x: np.ndarray, xs: int, T: int, n: int, qb: int, w: np.ndarray, b: np.ndarray, eps: float,
                       rmode: int = RN) -> tuple[np.ndarray, np.ndarray]:
    """normq (core/encoder.c:112-130)."""
    q = np.zeros((T, n), np.int8)
    d = np.zeros((T, n // qb), np.float32)
    olib().oracle_layernorm_quantize(_p(q), _p(d), _p(_f32(x)), xs, T, n, qb, _p(_f32(w)), _p(_f32(b)), eps, rmode)
    return q, d


def layernorm(x: np.ndarray, xs: int, T: int, n: int, w: np.ndarray, b: np.ndarray, eps: float,
              rmode: int = RN) -> np.ndarray:
    """k_layernorm (backend/ref/kernels.c:115-131)."""
    out = np.zeros((T, n), np.float32)
    olib().oracle_layernorm(_p(out), n, _p(_f32(x)), xs, T, n, _p(_f32(w)), _p(_f32(b)), eps, rmode)
    return out


def silu_quantize(u: np.ndarray, us: int, T: int, n: int, qb: int, rmode: int = RN) -> tuple[np.ndarray, np.ndarray]:
    """siluq_tile (core/encoder.c:150-158)."""
    q = np.zeros((T, n), np.int8)
    d = np.zeros((T, n // qb), np.float32)
    olib().oracle_silu_quantize(_p(q), _p(d), _p(_f32(u)), us, T, n, qb, rmode)
    return q, d


def dwconv_quantize(x: np.ndarray, xs: int, T: int, C: int, w: np.ndarray, b: np.ndarray, K: int, glu: bool, qb: int,
                    rmode: int = RN) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """glu_item + dw_item (core/encoder.c:160-183): (q, d, the convolution's floats)."""
    q = np.zeros((T, C), np.int8)
    d = np.zeros((T, C // qb), np.float32)
    out = np.zeros((T, C), np.float32)
    olib().oracle_dwconv_quantize(_p(q), _p(d), _p(out), C, _p(_f32(x)), xs, T, C, _p(_f32(w)), _p(_f32(b)), K,
                                  int(glu), qb, rmode)
    return q, d, out


def gemm_f32(out: np.ndarray, os_: int, w: np.ndarray, ld: int, rows: int, n: int, x: np.ndarray, xs: int, T: int,
             bias: Optional[np.ndarray], bs: int, relu: bool, rmode: int = RN, w_off: int = 0) -> None:
    """k_gemm_f32 (backend/ref/kernels.c:90-105) into out (written in place);
    w_off: the float of w the call's w points at (a run inside the panels)."""
    olib().oracle_gemm_f32(_p(out), os_, _p(w) + 4 * w_off, ld, rows, n, _p(x), xs, T, _p(bias), bs, int(relu),
                           rmode)


def softmax(x: np.ndarray, xs: int, T: int, n: int, scale: float, rmode: int = RN) -> None:
    """k_softmax (backend/ref/kernels.c:134-147) on T rows, in place."""
    olib().oracle_softmax(_p(x), xs, T, n, float(np.float32(scale)), rmode)


def attention(q: np.ndarray, qs: int, kp: np.ndarray, pp: np.ndarray, vp: np.ndarray, bias_u: np.ndarray,
              bias_v: np.ndarray, T: int, D: int, H: int, rmode: int = RN) -> np.ndarray:
    """att_item (core/encoder.c:280-326) over every head and query: o [T][D]."""
    o = np.zeros((T, D), np.float32)
    olib().oracle_attention(_p(o), D, _p(_f32(q)), qs, _p(_f32(kp)), _p(_f32(pp)), _p(_f32(vp)), _p(_f32(bias_u)),
                            _p(_f32(bias_v)), T, D, H, rmode)
    return o


class _Tdt(ctypes.Structure):
    """oracle_tdt (oracle/q8_oracle.c): the decoder's weights"""
    _fields_ = [(n, ctypes.c_uint32) for n in ("P", "L", "J", "V", "n_dur", "max_symbols", "n_out_pad")] + \
               [(n, ctypes.c_void_p) for n in ("dur", "embed", "wx", "wh", "wxs", "whs", "lb", "jpred", "jpreds",
                                               "jpredb", "jout", "jouts", "joutb")]


def tdt_read(path: str) -> dict:
    """A file tdt_ref wrote (oracle/tdt_ref.c): the reference's decoder
    weights (PK_Q8 bytes and scales), the frames and the reference's tokens."""
    b = open(path, "rb").read()
    P, L, J, V, nd, ms, nop, T, nt = np.frombuffer(b, np.uint32, 9).tolist()
    o = 36
    out = dict(P=P, L=L, J=J, V=V, n_dur=nd, max_symbols=ms, n_out_pad=nop, T=T)

    def take(name, dtype, count):
        nonlocal o
        a = np.frombuffer(b, dtype, count, o).copy()
        o += a.nbytes
        out[name] = a
    take("dur", np.uint32, nd)
    take("embed", np.float32, (V + 1) * P)
    wx, wxs, wh, whs, lb = [], [], [], [], []
    for _ in range(L):
        for lst, dt, cnt in ((wx, np.int8, 16 * P * P // 4), (wxs, np.float32, 4 * P), (wh, np.int8, 16 * P * P // 4),
                             (whs, np.float32, 4 * P), (lb, np.float32, 4 * P)):
            lst.append(np.frombuffer(b, dt, cnt, o).copy())
            o += lst[-1].nbytes
    out.update(wx=np.concatenate(wx), wxs=np.concatenate(wxs), wh=np.concatenate(wh), whs=np.concatenate(whs),
               lb=np.concatenate(lb))
    take("jpred", np.int8, J * P)
    take("jpreds", np.float32, J)
    take("jpredb", np.float32, J)
    take("jout", np.int8, nop * J)
    take("jouts", np.float32, nop)
    take("joutb", np.float32, nop)
    take("f", np.float32, T * J)
    take("toks", np.int32, 3 * nt)
    out["toks"] = out["toks"].reshape(nt, 3)
    assert o == len(b)
    return out


def tdt_search(m: dict, f: np.ndarray, T: int, rmode: int = RN, cap: int = 1 << 20) -> np.ndarray:
    """TDT's greedy search (core/decoder.c:125-179) as restated: tokens as
    rows of (id, frame, duration)."""
    keep = {k: np.ascontiguousarray(m[k]) for k in ("dur", "embed", "wx", "wh", "wxs", "whs", "lb", "jpred",
                                                      "jpreds", "jpredb", "jout", "jouts", "joutb")}
    t = _Tdt(m["P"], m["L"], m["J"], m["V"], m["n_dur"], m["max_symbols"], m["n_out_pad"],
             *[_p(keep[k]) for k in ("dur", "embed", "wx", "wh", "wxs", "whs", "lb", "jpred", "jpreds", "jpredb",
                                     "jout", "jouts", "joutb")])
    f = np.ascontiguousarray(f, np.float32)
    cap = min(cap, T * (m["max_symbols"] + 1) + 16)  # at most max_symbols tokens a frame
    ids, frames, durs = (np.zeros(cap, np.int32) for _ in range(3))
    n = olib().oracle_tdt_search(_p(ids), _p(frames), _p(durs), cap, _p(f), T, ctypes.byref(t), rmode)
    assert n >= 0, "more tokens than the cap"
    return np.stack([ids[:n], frames[:n], durs[:n]], axis=1)


def tanhf(x: np.ndarray, rmode: int = RN) -> np.ndarray:
    """pk_tanhf (core/vmath.h:153-165), elementwise."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    olib().oracle_tanhf(_p(y), _p(x), x.size, rmode)
    return y


TDT_REF = os.path.join(REF_DIR, "tdt_ref")


def ref_tdt(frames: int, seed: int, scale: float, path: str) -> dict:
    """The reference's own search (oracle/_ref/tdt_ref over its tiny model)."""
    subprocess.run([TDT_REF, os.path.join(REF_DIR, "tiny.pkf"), str(frames), str(seed), repr(float(scale)), path],
                   check=True)
    return tdt_read(path)


def _f32(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32).reshape(-1)
    return a


# ------------------------------------------------- the reference's own ref --

_FE = {RN: 0x000, RD: 0x400, RU: 0x800, RZ: 0xc00}  # x86-64 glibc fenv.h values


def _with_mode(rmode: int, fn):
    libm = ctypes.CDLL("libm.so.6")
    was = libm.fegetround()
    if libm.fesetround(_FE[rmode]):
        raise RuntimeError("fesetround failed")
    try:
        return fn()
    finally:
        libm.fesetround(was)


def ref_quantize(x: np.ndarray, n: int, qb: int, T: Optional[int] = None, xs: Optional[int] = None,
                 rmode: int = RN) -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    xs = n if xs is None else xs
    T = x.size // xs if T is None else T
    q = np.zeros((T, n), np.int8)
    d = np.zeros((T, n // qb), np.float32)
    act = _Act(_p(q), _p(d), n, qb, T)
    k = _Table.in_dll(rlib(), "pk_kernels_ref")
    _with_mode(rmode, lambda: k.quantize(ctypes.byref(act), _p(x), xs))
    return q, d


def ref_gemm_q8(out: np.ndarray, os_: int, w: np.ndarray, ws: np.ndarray, bias: Optional[np.ndarray], rows: int,
                q: np.ndarray, d: np.ndarray, n: int, qb: int, T: int, add: bool, rmode: int = RN) -> None:
    act = _Act(_p(q), _p(d), n, qb, T)
    k = _Table.in_dll(rlib(), "pk_kernels_ref")
    _with_mode(rmode, lambda: k.gemm_q8(_p(out), os_, _p(w), _p(ws), _p(bias), rows, ctypes.byref(act), int(add)))


def ref_gemm_f32(out: np.ndarray, os_: int, w: np.ndarray, ld: int, rows: int, n: int, x: np.ndarray, xs: int,
                 T: int, bias: Optional[np.ndarray], bs: int, relu: bool, rmode: int = RN, w_off: int = 0) -> None:
    k = _Table.in_dll(rlib(), "pk_kernels_ref")
    _with_mode(rmode, lambda: k.gemm_f32(_p(out), os_, _p(w) + 4 * w_off, ld, rows, n, _p(x), xs, T, _p(bias), bs,
                                         int(relu)))


def ref_softmax(x: np.ndarray, xs: int, T: int, n: int, scale: float, rmode: int = RN) -> None:
    k = _Table.in_dll(rlib(), "pk_kernels_ref")
    scale = float(np.float32(scale))  # a float already: ctypes' conversion would round in the mode

    def run():
        for t in range(T):
            k.softmax(_p(x) + 4 * t * xs, n, scale)
    _with_mode(rmode, run)


def ref_attention(q: np.ndarray, qs: int, kp: np.ndarray, pp: np.ndarray, vp: np.ndarray, bias_u: np.ndarray,
                  bias_v: np.ndarray, T: int, D: int, H: int, block: int = 16) -> np.ndarray:
    """att_item (core/encoder.c:280-326) as the reference runs it, under
    round-to-nearest: per head and block of `block` queries (PK_ATT_BLOCK,
    core/asr.h:16), the query rows with each position bias (numpy's float32
    adds), its ref backend's gemm_f32 for the scores over Tp keys and for the
    position products over the block's window of rows from a panel
    boundary, the scores plus their positions, its softmax row by row, and
    its gemm_f32 for the weighted values."""
    k = _Table.in_dll(rlib(), "pk_kernels_ref")
    q = _f32(q)
    kp, pp, vp, bias_u, bias_v = _f32(kp), _f32(pp), _f32(vp), _f32(bias_u), _f32(bias_v)
    dk = D // H
    Tp = (T + 15) // 16 * 16
    Pp = (2 * T - 1 + 15) // 16 * 16 + 16
    o = np.zeros((T, D), np.float32)
    scale = np.float32(1.0) / np.sqrt(np.float32(dk))
    for h in range(H):
        for i0 in range(0, T, block):
            i1 = min(i0 + block, T)
            nq = i1 - i0
            qh = q.reshape(-1)[:].view(np.float32)
            rows_q = np.stack([qh[(i0 + i) * qs + h * dk:(i0 + i) * qs + h * dk + dk] for i in range(nq)])
            qu = np.ascontiguousarray(rows_q + bias_u[h * dk:(h + 1) * dk], np.float32)
            qv = np.ascontiguousarray(rows_q + bias_v[h * dk:(h + 1) * dk], np.float32)
            sc = np.zeros(nq * Tp, np.float32)
            k.gemm_f32(_p(sc), Tp, _p(kp) + 4 * h * Tp * dk, dk, Tp, dk, _p(qu), dk, nq, 0, 0, 0)
            m_lo, m_hi = T - i1, 2 * T - 2 - i0
            m_a = m_lo & ~15
            rows = (m_hi + 1 - m_a + 15) // 16 * 16
            bd = np.zeros(nq * rows, np.float32)
            k.gemm_f32(_p(bd), rows, _p(pp) + 4 * (h * Pp * dk + (m_a // 16) * dk * 16), dk, rows, dk, _p(qv), dk,
                       nq, 0, 0, 0)
            for i in range(i0, i1):
                srow = sc[(i - i0) * Tp:(i - i0) * Tp + T]
                b0 = (i - i0) * rows + (T - 1 - i) - m_a
                srow[:] = srow + bd[b0:b0 + T]
                k.softmax(_p(sc) + 4 * (i - i0) * Tp, T, float(scale))
            out = np.zeros(nq * D, np.float32)
            k.gemm_f32(_p(out) + 4 * h * dk, D, _p(vp) + 4 * h * (dk // 16) * T * 16, T, dk, T, _p(sc), Tp, nq,
                       0, 0, 0)
            o[i0:i1, h * dk:(h + 1) * dk] = out.reshape(nq, D)[:, h * dk:(h + 1) * dk]
    return o


# ------------------------------- the reference's fastest backend, threaded --
#
# For checks at full size (the benchmark's M of 11,521 frames), where ref's
# scalar loops would take minutes: the backend the reference's own picker
# chooses on this CPU (amx-int8 on an AMX Xeon, backend/kernels.c:277-305),
# which the reference's q8check holds to ref's bits byte for byte, driven over
# all host cores the way its passes deal work (oracle/cpu_bench.c).

CPUBENCH_SO = os.path.join(REF_DIR, "libcpubench.so")
_cpub = None


def have_fast() -> bool:
    return os.path.exists(CPUBENCH_SO)


def _cpublib() -> ctypes.CDLL:
    global _cpub
    if _cpub is None:
        if not have_fast():
            raise FileNotFoundError(CPUBENCH_SO + " is not built (make -C oracle ref)")
        l = ctypes.CDLL(CPUBENCH_SO)
        vp, u32, sz = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_size_t
        l.cpub_backend.restype = ctypes.c_char_p
        l.cpub_backend.argtypes = [ctypes.c_char_p, sz]
        l.cpub_quantize.restype = None
        l.cpub_quantize.argtypes = [vp, vp, vp, sz, u32, u32, u32, ctypes.c_int]
        l.cpub_gemm.restype = None
        l.cpub_gemm.argtypes = [vp, sz, vp, vp, vp, u32, vp, vp, u32, u32, u32, ctypes.c_int, ctypes.c_int]
        l.cpub_backend(None, 0)  # the picker runs once, before any thread calls a kernel
        _cpub = l
    return _cpub


def fast_backend() -> str:
    return _cpublib().cpub_backend(None, 0).decode()


def fast_quantize(x: np.ndarray, n: int, qb: int, T: int, xs: Optional[int] = None,
                  threads: Optional[int] = None) -> tuple[np.ndarray, np.ndarray]:
    """The picked backend's quantize (round to nearest), over all cores."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    q = np.empty((T, n), np.int8)
    d = np.empty((T, n // qb), np.float32)
    _cpublib().cpub_quantize(_p(q), _p(d), _p(x), xs or n, n, qb, T, threads or os.cpu_count() or 1)
    return q, d


def fast_gemm_q8(out: np.ndarray, os_: int, w: np.ndarray, ws: np.ndarray, bias: Optional[np.ndarray], rows: int,
                 q: np.ndarray, d: np.ndarray, n: int, qb: int, T: int, add: bool,
                 threads: Optional[int] = None) -> None:
    """The picked backend's product into out (round to nearest), over all cores."""
    for a in (out, w, ws, q, d) + ((bias,) if bias is not None else ()):
        assert a.flags.c_contiguous
    _cpublib().cpub_gemm(_p(out), os_, _p(w), _p(ws), _p(bias), rows, _p(q), _p(d), n, qb, T, int(add),
                         threads or os.cpu_count() or 1)


# ------------------------------------------------ the reference's generators --

class XorShift:
    """xorshift64* as the reference's tests draw (tests/kcheck.c:40-48)."""

    def __init__(self, seed: int = 0x9E3779B97F4A7C15):
        self.s = seed & 0xFFFFFFFFFFFFFFFF

    def rnd(self) -> int:
        s = self.s
        s ^= s >> 12
        s ^= (s << 25) & 0xFFFFFFFFFFFFFFFF
        s ^= s >> 27
        self.s = s
        return ((s * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF) >> 32

    def frand(self) -> float:
        """[-1, 1), as float32"""
        return float(np.float32(np.float32(self.rnd() >> 8) / np.float32(8388608.0)) - np.float32(1.0))

    def awkward(self, scale: float) -> float:
        """the reference's awkward values (tests/kcheck.c:50-60)"""
        c = self.rnd() % 24
        s = np.float32(scale)
        if c == 0:
            return 0.0
        if c == 1:
            return -0.0
        if c == 2:
            return float(np.float32(1e-40))
        if c == 3:
            return float(-s * np.float32(30.0))
        if c == 4:
            return float(s * np.float32(0.5))
        return float(s * np.float32(self.frand()))


def seeded_normal(shape, seed: int) -> np.ndarray:
    """float32 ~N(0,1) from numpy's PCG64 generator with this seed
    (deterministic across machines for a given numpy major version)."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal(shape, dtype=np.float32)


def uniform_weights(rows: int, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(-127, 128, size=(rows, n), dtype=np.int8)


# ------------------------------- the reference's producers, as its encoder --

def _part(q: np.ndarray, d: np.ndarray, t: int, k0: int, nn: int, n: int, qb: int) -> _Act:
    """pk_quant_part's activation view (core/passes.c:114-118): nn inputs of
    column t from input k0"""
    at = t * n + k0
    return _Act(q.ctypes.data + at, d.ctypes.data + 4 * (at // qb), nn, qb, 1)


def ref_layernorm_quantize(x: np.ndarray, xs: int, T: int, n: int, qb: int, w: np.ndarray, b: np.ndarray, eps: float,
                           rmode: int = RN) -> tuple[np.ndarray, np.ndarray]:
    """normq_item (core/encoder.c:114-124) through the reference's ref table:
    k_layernorm of a frame into a row, pk_quant_part of the row."""
    x, w, b = _f32(x), _f32(w), _f32(b)
    q = np.zeros((T, n), np.int8)
    d = np.zeros((T, n // qb), np.float32)
    row = np.zeros(n, np.float32)
    k = _Table.in_dll(rlib(), "pk_kernels_ref")

    def run():
        for t in range(T):
            k.layernorm(_p(row), n, x.ctypes.data + 4 * t * xs, n, 1, n, _p(w), _p(b), eps)
            act = _part(q, d, t, 0, n, n, qb)
            k.quantize(ctypes.byref(act), _p(row), n)
    _with_mode(rmode, run)
    return q, d


def ref_silu_quantize(u: np.ndarray, us: int, T: int, n: int, qb: int, rmode: int = RN) -> tuple[np.ndarray, np.ndarray]:
    """siluq_tile (core/encoder.c:150-158) through the ref table, the whole
    row as one tile: copy, k_silu, pk_quant_part."""
    u = _f32(u)
    q = np.zeros((T, n), np.int8)
    d = np.zeros((T, n // qb), np.float32)
    k = _Table.in_dll(rlib(), "pk_kernels_ref")

    def run():
        for t in range(T):
            row = u[t * us: t * us + n].copy()
            k.silu(_p(row), n)
            act = _part(q, d, t, 0, n, n, qb)
            k.quantize(ctypes.byref(act), _p(row), n)
    _with_mode(rmode, run)
    return q, d


def ref_dwconv_quantize(x: np.ndarray, xs: int, T: int, C: int, w: np.ndarray, b: np.ndarray, K: int, glu: bool,
                        qb: int, rmode: int = RN) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """glu_item + dw_item (core/encoder.c:160-183) through the ref table:
    k_glu over the frames where glu, then per chunk of 64 channels k_dwconv
    and pk_quant_part of each frame's chunk."""
    x, w, b = _f32(x), _f32(w), _f32(b)
    q = np.zeros((T, C), np.int8)
    d = np.zeros((T, C // qb), np.float32)
    out = np.zeros((T, C), np.float32)
    k = _Table.in_dll(rlib(), "pk_kernels_ref")

    def run():
        if glu:
            h = np.zeros((T, C), np.float32)
            k.glu(_p(h), C, _p(x), xs, T, C)
            src, ss = h.reshape(-1), C
        else:
            src, ss = x, xs
        for c0 in range(0, C, 64):
            nc = min(64, C - c0)
            k.dwconv(out.ctypes.data + 4 * c0, C, src.ctypes.data + 4 * c0, ss, T, nc, w.ctypes.data + 4 * c0 * K,
                     b.ctypes.data + 4 * c0, K)
            for t in range(T):
                act = _part(q, d, t, c0, nc, C, qb)
                k.quantize(ctypes.byref(act), out.ctypes.data + 4 * (t * C + c0), nc)
    _with_mode(rmode, run)
    return q, d, out


# ------------------------------------------------- the attention's panels --

PKPASSES_SO = os.path.join(REF_DIR, "libpkpasses.so")


def panels_kp(src: np.ndarray, n: int, np_: int, D: int, dk: int) -> np.ndarray:
    """pk_panels_tile (core/passes.c:169-196) over a whole matrix: src [n][D]
    floats into K/P panels of np_ frames (the rest zeros)."""
    src = np.ascontiguousarray(src, np.float32).reshape(-1)
    dst = np.empty((D // dk) * np_ * dk, np.float32)
    olib().oracle_panels_kp(_p(dst), _p(src), n, np_, D, dk)
    return dst


def panels_v(w: np.ndarray, ws: np.ndarray, rows: int, q: np.ndarray, d: np.ndarray, n: int, qb: int, T: int,
             ps: int, rmode: int = RN) -> np.ndarray:
    """pk_gemm_panels_on (core/passes.c:119-141): the product one 16-row panel
    a call, each with os 16 into panel r/16 at (r/16) ps."""
    out = np.zeros((rows // 16 - 1) * ps + 16 * T, np.float32)
    for r in range(0, rows, 16):
        part = out[(r // 16) * ps:]
        olib().oracle_gemm_q8(_p(part), 16, _p(w[r * n:]), _p(ws[r:]), None, 16, _p(q), _p(d), n, qb, T, 0, rmode)
    return out


class _Panels(ctypes.Structure):
    """pk_panels (core/passes.h:53)"""
    _fields_ = [("dst", ctypes.c_void_p), ("src", ctypes.c_void_p), ("n", ctypes.c_uint32), ("np", ctypes.c_uint32),
                ("D", ctypes.c_uint32), ("dk", ctypes.c_uint32)]


def have_passes() -> bool:
    return os.path.exists(PKPASSES_SO)


def ref_panels_kp(src: np.ndarray, n: int, np_: int, D: int, dk: int) -> np.ndarray:
    """The reference's own pk_panels_tile (libpkpasses.so) over the whole
    matrix as one tile: rows 0..D, frames 0..n (the last, so the padding is
    written)."""
    lib = ctypes.CDLL(PKPASSES_SO)
    src = np.ascontiguousarray(src, np.float32).reshape(-1)
    dst = np.full((D // dk) * np_ * dk, np.nan, np.float32)
    arg = _Panels(_p(dst), _p(src), n, np_, D, dk)
    f = lib.pk_panels_tile
    f.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int]
    f.restype = None
    f(ctypes.addressof(arg), 0, D, 0, n, 0)
    return dst
