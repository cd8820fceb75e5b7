"""The fused producers' entry points refuse bad arguments before touching a
device (CPU only: every check here fails before any CUDA call), and T = 0
does nothing, as the reference's kernels read and write nothing then."""
import ctypes

import numpy as np
import pytest

import libpktito_b200 as P

EINVAL = 1
B = np.zeros(64, np.float32)  # a host pointer: never dereferenced by a call refused up front


def p(a):
    return a.ctypes.data


def ln(**kw):
    a = dict(q=p(B), d=p(B), x=p(B), xs=64, T=2, n=64, qb=32, w=p(B), b=p(B), eps=1e-5, rmode=0)
    a.update(kw)
    return P.lib().pkb_layernorm_quantize_dev(0, a["q"], a["d"], a["x"], a["xs"], a["T"], a["n"], a["qb"], a["w"],
                                              a["b"], a["eps"], a["rmode"])


def si(**kw):
    a = dict(q=p(B), d=p(B), u=p(B), us=64, T=2, n=64, qb=32, rmode=0)
    a.update(kw)
    return P.lib().pkb_silu_quantize_dev(0, a["q"], a["d"], a["u"], a["us"], a["T"], a["n"], a["qb"], a["rmode"])


def dw(**kw):
    a = dict(q=p(B), d=p(B), out=None, os=64, x=p(B), xs=128, T=2, C=64, w=p(B), b=p(B), K=9, glu=1, qb=32, rmode=0)
    a.update(kw)
    return P.lib().pkb_dwconv_quantize_dev(0, a["q"], a["d"], a["out"], a["os"], a["x"], a["xs"], a["T"], a["C"],
                                           a["w"], a["b"], a["K"], a["glu"], a["qb"], a["rmode"])


@pytest.mark.parametrize("kw", [dict(qb=128), dict(qb=16), dict(n=48), dict(n=0), dict(n=8192 + 64, xs=8192 + 64),
                                dict(xs=32), dict(rmode=4), dict(x=None), dict(w=None), dict(b=None),
                                dict(q=p(B) + 1), dict(x=p(B) + 2)])
def test_layernorm_quantize_refuses(kw):
    assert ln(**kw) == EINVAL
    assert P.lib().pkb_last_error()


@pytest.mark.parametrize("kw", [dict(qb=128), dict(n=48), dict(us=32), dict(rmode=-1), dict(u=None),
                                dict(d=p(B) + 1)])
def test_silu_quantize_refuses(kw):
    assert si(**kw) == EINVAL


@pytest.mark.parametrize("kw", [dict(qb=96), dict(C=48), dict(C=0), dict(K=8), dict(K=65), dict(xs=100),
                                dict(glu=0, xs=63), dict(x=None), dict(w=None), dict(out=p(B), os=32),
                                dict(out=p(B) + 64, os=64, glu=0, xs=64), dict(rmode=9)])
def test_dwconv_quantize_refuses(kw):
    assert dw(**kw) == EINVAL


def test_out_overlapping_x_is_refused():
    x = np.zeros(1024, np.float32)
    assert dw(x=p(x), xs=128, out=p(x) + 4 * 200, os=64) == EINVAL
    assert "overlap" in P.lib().pkb_last_error().decode()


def test_no_frames_is_a_no_op():
    assert ln(T=0, x=None) == 0
    assert si(T=0, u=None) == 0
    assert dw(T=0, x=None) == 0


def test_exported():
    for name in ("pkb_layernorm_quantize_dev", "pkb_silu_quantize_dev", "pkb_dwconv_quantize_dev"):
        assert isinstance(getattr(P.lib(), name), ctypes._CFuncPtr)


@pytest.mark.parametrize("args", [(4, 0x3F800000, 0x40000000), (0, 0x3F000000, 0x40000000),
                                  (0, 0x3F800000, 0x7F800001), (0, 0x40000000, 0x40000000)])
def test_rcp_selftest_refuses(args):
    m, f = ctypes.c_uint64(), ctypes.c_uint32()
    assert P.lib().pkb_rcp_selftest(*args, ctypes.byref(m), ctypes.byref(f)) == EINVAL
