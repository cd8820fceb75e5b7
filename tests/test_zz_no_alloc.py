"""pkb_quantize_host_noalloc, through the C ABI, against pkb_quantize_host.

The entry point is for callers that cannot allocate memory when they
quantize: an application whose own pool already holds all of a GPU's memory,
or a real-time audio callback in which an allocation (which can synchronize
the whole device) is not allowed. It works in a fixed array compiled into the
library instead. Two calls in a row, on different columns, must each give
exactly the bytes and scales the allocating entry point gives (the tests'
tolerance for this path is none: bit for bit), and a call too large for the
array must be refused without work.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(lib, x, n, qb, T, xs):
    q = np.zeros(T * n, np.int8)
    d = np.zeros(T * n // qb, np.float32)
    rc = lib.pkb_quantize_host_noalloc(q.ctypes.data, d.ctypes.data, n, qb, T, x.ctypes.data, xs, 0)
    return rc, q.reshape(T, n), d.reshape(T, n // qb)


def test_noalloc_matches_the_allocating_entry_on_two_calls(pkb, cuda_device):
    lib = pkb.lib()
    cases = [(750, 1024, 32, 1024), (37, 4096, 64, 4128)]
    for i, (T, n, qb, xs) in enumerate(cases):
        rng = np.random.default_rng(4242 + i)
        x = (rng.standard_normal(T * xs + n) * rng.choice([1.0, 1e4, 1e-38], T * xs + n)).astype(np.float32)
        x[5] = np.nan                 # a block with a NaN: zeros, scale 0
        x[xs: xs + qb] = 0.0          # a block of zeros: scale 0
        rc, q1, d1 = _noalloc(lib, x, n, qb, T, xs)
        assert rc == 0, lib.pkb_last_error()
        q2, d2 = pkb.quantize_host(x, n, qb, T=T, xs=xs)
        assert np.array_equal(q1, q2), f"call {i + 1}: bytes differ"
        assert d1.tobytes() == d2.tobytes(), f"call {i + 1}: scales differ"


def test_noalloc_refuses_what_its_array_cannot_hold(pkb, cuda_device):
    lib = pkb.lib()
    T, n, qb = 2048, 4096, 32           # 43 MB of staging, past the 8 MiB array
    x = np.ones(T * n, np.float32)
    q = np.full(T * n, 7, np.int8)
    d = np.full(T * n // qb, 7.0, np.float32)
    rc = lib.pkb_quantize_host_noalloc(q.ctypes.data, d.ctypes.data, n, qb, T, x.ctypes.data, n, 0)
    assert rc == 1 and b"fixed staging" in lib.pkb_last_error()
    assert (q == 7).all() and (d == 7.0).all()  # nothing written
