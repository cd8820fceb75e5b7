"""libpktito_b200: libpktito's int8 path (quantize + gemm_q8) on B200, from Python.

A thin ctypes layer over the C ABI of include/pktito_b200.h, for tests,
benchmarks and Python callers. The arithmetic lives in the CUDA library
(libpktito_b200.so, built in place by libpktito_b200.build); nothing here
computes a result, and every call fails loudly (PkbError) when the library
or a GPU is missing.

Two call styles, as the C ABI has them:

* host arrays (numpy), synchronous: ``quantize_host`` / ``gemm_q8_host`` and
  the reference-facing table ``Table`` (the ``pk_kernels_cuda_b200`` entry of
  libpktito's backend table, backend/kernels.h:242-278);
* device buffers (torch CUDA tensors), enqueued on the current stream:
  ``quantize_dev`` / ``repack_q8_dev`` / ``gemm_q8_dev``.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpktito_b200.so")

RN, RD, RU, RZ = 0, 1, 2, 3
MAX_N = 16384

_STATUS = {1: "EINVAL", 2: "ECUDA", 3: "ENOMEM", 4: "ETIMEOUT", 5: "ENODEV"}


class PkbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"pkb {_STATUS.get(code, code)}: {msg}")
        self.code = code


class PkAct(ctypes.Structure):
    """pk_act (backend/kernels.h:41-45)."""
    _fields_ = [("q", ctypes.c_void_p), ("d", ctypes.c_void_p),
                ("n", ctypes.c_uint32), ("qb", ctypes.c_uint32), ("T", ctypes.c_uint32)]


_QUANT_FN = ctypes.CFUNCTYPE(None, ctypes.POINTER(PkAct), ctypes.c_void_p, ctypes.c_size_t)
_GEMM_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p,
                            ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(PkAct), ctypes.c_int)


class PkKernels(ctypes.Structure):
    """pk_kernels (backend/kernels.h:242-278); the members past gemm_q8 as
    plain pointers, since Python calls only the int8 path."""
    _fields_ = [("id", ctypes.c_char_p), ("name", ctypes.c_char_p), ("needs", ctypes.c_void_p),
                ("competes", ctypes.c_int), ("quantize", _QUANT_FN), ("gemm_q8", _GEMM_FN)] + \
               [(f, ctypes.c_void_p) for f in ("gemm_f32", "layernorm", "softmax", "silu", "gelu", "glu",
                                               "dwconv", "conv3x3s2", "lstm", "stft", "resample")]


_lib: Optional[ctypes.CDLL] = None

# the symbols include/pktito_b200.h declares, with their C signatures
_SIGS = {
    "pkb_last_error": (ctypes.c_char_p, []),
    "pkb_device_count": (ctypes.c_int, []),
    "pkb_set_thread_device": (ctypes.c_int, [ctypes.c_int]),
    "pkb_device_errors": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)]),
    "pkb_wait_selftest": (ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_int)]),
    "pkb_rcp_selftest": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint32, ctypes.c_uint32,
                                        ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint32)]),
    "pkb_quantize_host": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                         ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]),
    "pkb_gemm_q8_host": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int,
                                        ctypes.c_int]),
    "pkb_forget": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t]),
    "pkb_wpack_bytes": (ctypes.c_size_t, [ctypes.c_uint32, ctypes.c_uint32]),
    "pkb_repack_q8_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                         ctypes.c_uint32]),
    "pkb_quantize_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                        ctypes.c_int]),
    "pkb_gemm_q8_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                       ctypes.c_int, ctypes.c_int]),
    "pkb_layernorm_quantize_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                  ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int]),
    "pkb_silu_quantize_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                             ctypes.c_int]),
    "pkb_dwconv_quantize_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32,
                                               ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                               ctypes.c_int, ctypes.c_uint32, ctypes.c_int]),
    "pkb_gemm_q8_panels_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t,
                                              ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                              ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int]),
    "pkb_gemm_f32_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                        ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                        ctypes.c_size_t, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
                                        ctypes.c_int, ctypes.c_int]),
    "pkb_softmax_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32,
                                       ctypes.c_uint32, ctypes.c_float, ctypes.c_int]),
    "pkb_attention_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                         ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                         ctypes.c_uint32, ctypes.c_int]),
    "pkb_attention_rows_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                              ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                              ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                              ctypes.c_uint32, ctypes.c_int]),
    "pkb_gemm_f32_host": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_uint32,
                                         ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
                                         ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                         ctypes.c_int]),
    "pkb_softmax_host": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float, ctypes.c_int]),
    "pkb_tdt_work_bytes": (ctypes.c_size_t, [ctypes.c_void_p, ctypes.c_uint32]),
    "pkb_tdt_search_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]),
    "pkb_layernorm_dev": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                         ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_float, ctypes.c_int]),
    "pkb_launch_count": (ctypes.c_uint64, []),
    "pkb_tdt_last_rounds": (ctypes.c_uint64, []),
    "pkb_host_bytes": (None, [ctypes.c_void_p, ctypes.c_void_p]),
    "pkb_quantize_host_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                                 ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]),
}


def lib() -> ctypes.CDLL:
    """The in-tree libpktito_b200.so, loaded once; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise PkbError(5, f"{LIB_PATH} is not built (python -m libpktito_b200.build)")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def _check(rc: int) -> None:
    if rc:
        raise PkbError(rc, lib().pkb_last_error().decode(errors="replace"))


def device_count() -> int:
    return lib().pkb_device_count()


def set_thread_device(dev: int) -> None:
    _check(lib().pkb_set_thread_device(dev))


def wait_selftest(limit_cycles: int = 2_000_000) -> bool:
    """Runs the bounded-wait self-test on the current device (a wait that
    nothing completes gives up, sets the error word's timeout bit); True if
    the wait gave up as it should."""
    g = ctypes.c_int(0)
    _check(lib().pkb_wait_selftest(limit_cycles, ctypes.byref(g)))
    return bool(g.value)


def rcp_selftest(rmode: int, lo_bits: int = 0x3F800000, hi_bits: int = 0x7F800000) -> tuple[int, int]:
    """(mismatches, smallest mismatching bits) of the sigmoid's reciprocal
    against the correctly rounded one over floats with bits in [lo, hi)."""
    m, f = ctypes.c_uint64(0), ctypes.c_uint32(0)
    _check(lib().pkb_rcp_selftest(rmode, lo_bits, hi_bits, ctypes.byref(m), ctypes.byref(f)))
    return m.value, f.value


def device_errors(dev: int = 0) -> int:
    w = ctypes.c_uint32()
    _check(lib().pkb_device_errors(dev, ctypes.byref(w)))
    return w.value


def launch_count() -> int:
    return int(lib().pkb_launch_count())


def host_bytes() -> tuple[int, int]:
    """(host to device, device to host) bytes the host-pointer calls copied."""
    up, down = ctypes.c_uint64(), ctypes.c_uint64()
    lib().pkb_host_bytes(ctypes.byref(up), ctypes.byref(down))
    return int(up.value), int(down.value)


def _ptr(a) -> int:
    if a is None:
        return 0
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()  # torch tensor


# ------------------------------------------------------------ host arrays --

def quantize_host(x: np.ndarray, n: int, qb: int, T: Optional[int] = None, xs: Optional[int] = None,
                  rmode: int = RN) -> tuple[np.ndarray, np.ndarray]:
    """Columns of x (float32; column t at x[t*xs:]) to (q [T][n] int8, d [T][n/qb] float32)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if xs is None:
        xs = n
    if T is None:
        T = x.size // xs if xs else 0
    q = np.zeros((T, n), np.int8)
    d = np.zeros((T, n // qb), np.float32)
    _check(lib().pkb_quantize_host(_ptr(q), _ptr(d), n, qb, T, _ptr(x), xs, rmode))
    return q, d


def gemm_q8_host(out: np.ndarray, os_: int, w: np.ndarray, ws: np.ndarray, bias: Optional[np.ndarray],
                 rows: int, q: np.ndarray, d: np.ndarray, n: int, qb: int, T: int, add: bool,
                 rmode: int = RN) -> None:
    """pk_k_gemm_q8 into out (float32, in place), w the PK_Q8 bytes at its first row."""
    assert out.dtype == np.float32 and out.flags.c_contiguous
    _check(lib().pkb_gemm_q8_host(_ptr(out), os_, _ptr(w), _ptr(ws), _ptr(bias), rows, _ptr(q), _ptr(d),
                                  n, qb, T, int(add), rmode))


def forget(p: np.ndarray) -> None:
    _check(lib().pkb_forget(_ptr(p), p.nbytes))


class Table:
    """The cuda-b200 entry of libpktito's backend table, called as the
    reference's passes call any backend (host pointers, void functions that
    abort on failure)."""

    def __init__(self):
        self.k = PkKernels.in_dll(lib(), "pk_kernels_cuda_b200")

    @property
    def id(self) -> str:
        return self.k.id.decode()

    def quantize(self, act: PkAct, x: np.ndarray, xs: int) -> None:
        self.k.quantize(ctypes.byref(act), _ptr(x), xs)

    def gemm_q8(self, out: np.ndarray, os_: int, w: np.ndarray, ws: np.ndarray, bias: Optional[np.ndarray],
                rows: int, act: PkAct, add: bool) -> None:
        self.k.gemm_q8(_ptr(out), os_, _ptr(w), _ptr(ws), _ptr(bias), rows, ctypes.byref(act), int(add))


# ---------------------------------------------------------- device buffers --

def _stream(stream=None) -> int:
    if stream is not None:
        return int(stream)
    import torch
    return torch.cuda.current_stream().cuda_stream


def quantize_dev(q, d, x, xs: int, T: int, n: int, qb: int, rmode: int = RN, stream=None) -> None:
    _check(lib().pkb_quantize_dev(_stream(stream), _ptr(q), _ptr(d), _ptr(x), xs, T, n, qb, rmode))


def layernorm_quantize_dev(q, d, x, xs: int, T: int, n: int, qb: int, w, b, eps: float, rmode: int = RN,
                           stream=None) -> None:
    """normq (core/encoder.c:112-130) on device buffers: rows layer-normalized
    and quantized in one kernel."""
    _check(lib().pkb_layernorm_quantize_dev(_stream(stream), _ptr(q), _ptr(d), _ptr(x), xs, T, n, qb, _ptr(w), _ptr(b),
                                            eps, rmode))


def layernorm_dev(out, os_: int, x, xs: int, T: int, n: int, w, b, eps: float, rmode: int = RN,
                  stream=None) -> None:
    """k_layernorm (backend/ref/kernels.c:115-131) on device rows; out may be x."""
    _check(lib().pkb_layernorm_dev(_stream(stream), _ptr(out), os_, _ptr(x), xs, T, n, _ptr(w), _ptr(b), eps, rmode))


def silu_quantize_dev(q, d, u, us: int, T: int, n: int, qb: int, rmode: int = RN, stream=None) -> None:
    """siluq_tile (core/encoder.c:150-158) on device buffers."""
    _check(lib().pkb_silu_quantize_dev(_stream(stream), _ptr(q), _ptr(d), _ptr(u), us, T, n, qb, rmode))


def dwconv_quantize_dev(q, d, out, os_: int, x, xs: int, T: int, C: int, w, b, K: int, glu: bool, qb: int,
                        rmode: int = RN, stream=None) -> None:
    """glu_item + dw_item (core/encoder.c:160-183) on device buffers; out may be None."""
    _check(lib().pkb_dwconv_quantize_dev(_stream(stream), _ptr(q), _ptr(d), _ptr(out), os_, _ptr(x), xs, T, C, _ptr(w),
                                         _ptr(b), K, int(glu), qb, rmode))


PANELS_V, PANELS_KP = 1, 2


def gemm_q8_panels_dev(panels, kind: int, ps: int, dk: int, tpad: int, wpack, ws, rows: int, q, d, n: int, qb: int,
                       T: int, rmode: int = RN, stream=None) -> None:
    """The product into the attention's V or K/P panels (core/passes.c:119-196)."""
    _check(lib().pkb_gemm_q8_panels_dev(_stream(stream), _ptr(panels), kind, ps, dk, tpad, _ptr(wpack), _ptr(ws), rows,
                                        _ptr(q), _ptr(d), n, qb, T, rmode))


def gemm_f32_dev(out, os_: int, w, ld: int, rows: int, n: int, x, xs: int, T: int, bias, bs: int, relu: bool,
                 rmode: int = RN, stream=None, w_off: int = 0) -> None:
    """pk_k_gemm_f32 (backend/ref/kernels.c:90-105) on device buffers; w_off:
    the float of w the call's run of panels starts at."""
    _check(lib().pkb_gemm_f32_dev(_stream(stream), _ptr(out), os_, _ptr(w) + 4 * w_off, ld, rows, n, _ptr(x), xs, T,
                                  _ptr(bias), bs, int(relu), rmode))


def softmax_dev(x, xs: int, T: int, n: int, scale: float, rmode: int = RN, stream=None) -> None:
    """pk_k_softmax (backend/ref/kernels.c:134-147) on T rows in place."""
    _check(lib().pkb_softmax_dev(_stream(stream), _ptr(x), xs, T, n, float(np.float32(scale)), rmode))


def attention_dev(o, os_: int, q, qs: int, kp, pp, vp, bias_u, bias_v, T: int, D: int, H: int, rmode: int = RN,
                  stream=None) -> None:
    """att_item (core/encoder.c:280-326) over one segment's heads and queries,
    K, P and V in the reference's panel layouts."""
    _check(lib().pkb_attention_dev(_stream(stream), _ptr(o), os_, _ptr(q), qs, _ptr(kp), _ptr(pp), _ptr(vp),
                                   _ptr(bias_u), _ptr(bias_v), T, D, H, rmode))


class AttSegment(ctypes.Structure):
    _fields_ = [("T", ctypes.c_uint32), ("f", ctypes.c_uint32), ("p", ctypes.c_uint32)]


def attention_rows_dev(o, os_: int, q, qs: int, k, ks: int, v, vs: int, p, ps: int, bias_u, bias_v, D: int, H: int,
                       segs, rmode: int = RN, stream=None) -> None:
    """The attention over a batch of segments, q, K, V and P as rows; segs:
    (T, first frame, first position row) a segment."""
    arr = (AttSegment * max(1, len(segs)))(*[AttSegment(*s) for s in segs])
    _check(lib().pkb_attention_rows_dev(_stream(stream), _ptr(o), os_, _ptr(q), qs, _ptr(k), ks, _ptr(v), vs,
                                        _ptr(p), ps, _ptr(bias_u), _ptr(bias_v), D, H, ctypes.addressof(arr),
                                        len(segs), rmode))


class TdtModel(ctypes.Structure):
    """pkb_tdt_model (include/pktito_b200.h): the TDT decoder's device weights."""
    _fields_ = [(n, ctypes.c_uint32) for n in ("P", "L", "J", "V", "n_dur", "max_symbols", "n_out_pad")] + \
               [("dur", ctypes.c_uint32 * 16), ("embed", ctypes.c_void_p)] + \
               [(n, ctypes.c_void_p * 4) for n in ("wx", "wh", "wxs", "whs", "lb")] + \
               [(n, ctypes.c_void_p) for n in ("jpred", "jpreds", "jpredb", "jout", "jouts", "joutb")]


def tdt_last_rounds() -> int:
    """Rounds this thread's last tdt_search_dev ran (its longest segment's joint steps)."""
    return int(lib().pkb_tdt_last_rounds())


def tdt_work_bytes(m: TdtModel, S: int) -> int:
    return int(lib().pkb_tdt_work_bytes(ctypes.byref(m), S))


def tdt_search_dev(m: TdtModel, f, f0: np.ndarray, T: np.ndarray, toks, ntok, cap: int, work, rmode: int = RN,
                   stream=None) -> None:
    """TDT's greedy search (core/decoder.c:125-179) over len(T) segments in
    lockstep: f device rows of J, f0/T host arrays, toks/ntok/work device."""
    f0 = np.ascontiguousarray(f0, np.uint32)
    T = np.ascontiguousarray(T, np.uint32)
    nbytes = work.numel() * work.element_size()
    _check(lib().pkb_tdt_search_dev(_stream(stream), ctypes.byref(m), _ptr(f), f0.ctypes.data, T.ctypes.data, T.size,
                                    _ptr(toks), _ptr(ntok), cap, _ptr(work), nbytes, rmode))


def repack_q8_dev(wpack, w_pk, rows: int, n: int, stream=None) -> None:
    _check(lib().pkb_repack_q8_dev(_stream(stream), _ptr(wpack), _ptr(w_pk), rows, n))


def gemm_q8_dev(out, os_: int, wpack, ws, bias, rows: int, q, d, n: int, qb: int, T: int, add: bool,
                rmode: int = RN, stream=None) -> None:
    _check(lib().pkb_gemm_q8_dev(_stream(stream), _ptr(out), os_, _ptr(wpack), _ptr(ws), _ptr(bias), rows,
                                 _ptr(q), _ptr(d), n, qb, T, int(add), rmode))
