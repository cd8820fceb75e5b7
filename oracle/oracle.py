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


def build() -> None:
    """liboracle.so always; the reference's code too where its sources are here."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if os.path.isdir(os.environ.get("PKTITO_REFERENCE", "/root/reference")):
        subprocess.run(["make", "-s", "-C", HERE, "ref",
                        "REF=" + os.environ.get("PKTITO_REFERENCE", "/root/reference")], check=True)


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


class _Table(ctypes.Structure):
    _fields_ = [("id", ctypes.c_char_p), ("name", ctypes.c_char_p), ("needs", ctypes.c_void_p),
                ("competes", ctypes.c_int), ("quantize", _QF), ("gemm_q8", _GF)]


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
