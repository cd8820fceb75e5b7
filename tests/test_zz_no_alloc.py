"""pkb_quantize_host_noalloc, through the C ABI, against pkb_quantize_host
and against the oracle.

The entry point is for callers that cannot allocate memory when they
quantize: an application whose own pool already holds all of a GPU's memory,
or a real-time audio callback in which an allocation (which can synchronize
the whole device) is not allowed. It works in a fixed array compiled into the
library instead. Two calls in a row, on different columns, must each give
exactly the bytes and scales the allocating entry point gives and the
oracle's (the tests' tolerance for this path is none: bit for bit), in the
rounding modes the reference's checks use; a call too large for the array
must be refused without work; and a call runs on the device its thread was
bound to.
"""
import threading

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _noalloc(lib, x, n, qb, T, xs, rmode=O.RN):
    q = np.zeros(T * n, np.int8)
    d = np.zeros(T * n // qb, np.float32)
    rc = lib.pkb_quantize_host_noalloc(q.ctypes.data, d.ctypes.data, n, qb, T, x.ctypes.data, xs, rmode)
    return rc, q.reshape(T, n), d.reshape(T, n // qb)


def _columns(i, T, n, qb, xs):
    rng = np.random.default_rng(4242 + i)
    x = (rng.standard_normal(T * xs + n) * rng.choice([1.0, 1e4, 1e-38], T * xs + n)).astype(np.float32)
    x[5] = np.nan                 # a block with a NaN: zeros, scale 0
    x[xs: xs + qb] = 0.0          # a block of zeros: scale 0
    return x


@pytest.mark.parametrize("rmode", [O.RN, O.RD, O.RZ])
def test_noalloc_matches_the_allocating_entry_and_the_oracle_on_two_calls(pkb, cuda_device, rmode):
    lib = pkb.lib()
    cases = [(750, 1024, 32, 1024), (37, 4096, 64, 4128)]
    for i, (T, n, qb, xs) in enumerate(cases):
        x = _columns(i, T, n, qb, xs)
        rc, q1, d1 = _noalloc(lib, x, n, qb, T, xs, rmode)
        assert rc == 0, lib.pkb_last_error()
        q2, d2 = pkb.quantize_host(x, n, qb, T=T, xs=xs, rmode=rmode)
        assert np.array_equal(q1, q2), f"call {i + 1}: bytes differ from pkb_quantize_host"
        assert d1.tobytes() == d2.tobytes(), f"call {i + 1}: scales differ from pkb_quantize_host"
        qo, do = O.quantize(x, n, qb, T=T, xs=xs, rmode=rmode)
        assert np.array_equal(q1, qo), f"call {i + 1}: bytes differ from the oracle"
        assert d1.tobytes() == do.tobytes(), f"call {i + 1}: scales differ from the oracle"


def test_noalloc_refuses_what_its_array_cannot_hold(pkb, cuda_device):
    lib = pkb.lib()
    T, n, qb = 2048, 4096, 32           # 43 MB of staging, past the 8 MiB array
    x = np.ones(T * n, np.float32)
    q = np.full(T * n, 7, np.int8)
    d = np.full(T * n // qb, 7.0, np.float32)
    rc = lib.pkb_quantize_host_noalloc(q.ctypes.data, d.ctypes.data, n, qb, T, x.ctypes.data, n, 0)
    assert rc == 1 and b"fixed staging" in lib.pkb_last_error()
    assert (q == 7).all() and (d == 7.0).all()  # nothing written


def test_noalloc_runs_on_the_threads_device(pkb, cuda_device):
    """A thread bound by pkb_set_thread_device quantizes on that device (the
    last one visible), made current as every host-pointer call makes it."""
    import torch
    lib = pkb.lib()
    dev = torch.cuda.device_count() - 1
    T, n, qb = 64, 1024, 32
    x = _columns(9, T, n, qb, n)
    seen = {}

    def bound():
        pkb.set_thread_device(dev)
        rc, q, d = _noalloc(lib, x, n, qb, T, n)
        seen.update(rc=rc, q=q, d=d, device=torch.cuda.current_device(),
                    err=lib.pkb_last_error() if rc else b"")

    th = threading.Thread(target=bound)
    th.start()
    th.join()
    assert seen["rc"] == 0, seen["err"]
    assert seen["device"] == dev
    qo, do = O.quantize(x, n, qb, T=T)
    assert np.array_equal(seen["q"], qo) and seen["d"].tobytes() == do.tobytes()
