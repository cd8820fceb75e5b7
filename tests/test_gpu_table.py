"""The cuda-b200 table under the reference engine's call pattern, and the
benchmark's own device path at its full size, bit for bit against the
reference.

The reference's passes call a backend from every thread of its pool at once
(core/pool.c:115-122): the activations in items of 16 columns
(pk_quantize_on, core/passes.c:39-46), then each product in slices of 64 or
256 rows of its matrix (w + r0 * cols, a run of panels from inside the
matrix) and chunks of columns (pk_gemm_on, core/passes.c:60-109), every
output written by exactly one call. The weights' device copies are shared by
all those calls and absorb the slices as they arrive.
"""
import threading

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def gemm_items(rows: int, T: int, nth: int) -> list[tuple[int, int, int, int]]:
    """(r0, nr, c0, nc) of every item pk_gemm_on deals (core/passes.c:90-109):
    rows in steps of 256 where rows/256 >= 2 threads, else 64; the columns
    in the chunk count (1..8, chunks of at least 48 columns) that leaves the
    pool's last round least idle, chunks whole multiples of 12."""
    step = 256 if rows // 256 >= 2 * nth else 64
    rb = (rows + step - 1) // step
    best, best_idle, best_all = 1, 2 ** 32 - 1, 1
    cc = 1
    while cc <= 8 and (cc == 1 or T // cc >= 48):
        items = rb * cc
        all_ = (items + nth - 1) // nth * nth
        if (all_ - items) * best_all < best_idle * all_:
            best, best_idle, best_all = cc, all_ - items, all_
        cc += 1
    cstep = (T + best - 1) // best
    cstep = (cstep + 11) // 12 * 12 if best > 1 else T
    cc = (T + cstep - 1) // cstep
    out = []
    for i in range(rb * cc):
        r0, c0 = (i % rb) * step, (i // rb) * cstep
        out.append((r0, min(step, rows - r0), c0, min(cstep, T - c0)))
    return out


def pool_run(nth: int, items: list, fn) -> None:
    """items dealt to nth threads from a shared counter, as core/pool.c does"""
    nxt = [0]
    lock = threading.Lock()
    errors = []

    def worker():
        while True:
            with lock:
                i = nxt[0]
                nxt[0] += 1
            if i >= len(items):
                return
            try:
                fn(items[i])
            except Exception as e:  # noqa: BLE001
                errors.append(e)
                return

    ts = [threading.Thread(target=worker) for _ in range(nth)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors[0]


def _sub_act(pkb, q, d, n, qb, c0, nc):
    return pkb.PkAct(q[c0 * n:].ctypes.data, d[c0 * (n // qb):].ctypes.data, n, qb, nc)


@pytest.mark.parametrize("nth", [8, 9])
def test_table_called_from_a_pool_as_the_engine_calls_it(pkb, cuda_device, nth):
    """Eight (nine) threads at once: quantize in items of 16 columns, then
    three products sliced as pk_gemm_on slices them (a 4096-row matrix in
    steps of 256 at 8 threads and of 64 at 9, so the two runs slice the same
    weights differently; a bias; one product adding), each output checked
    against the oracle."""
    tab = pkb.Table()
    T, n, qb = 301, 1024, 32
    x = O.seeded_normal(T * n, 5 + nth)
    q = np.zeros(T * n, np.int8)
    d = np.zeros(T * n // qb, np.float32)
    pool_run(nth, [t0 for t0 in range(0, T, 16)],
             lambda t0: tab.quantize(_sub_act(pkb, q, d, n, qb, t0, min(16, T - t0)), x[t0 * n:], n))
    qo, do = O.quantize(x, n, qb)
    assert np.array_equal(q.reshape(T, n), qo) and d.tobytes() == do.tobytes()
    mats = [(4096, False, False), (1024, True, False), (2048, False, True)]
    for k, (rows, bias_on, add) in enumerate(mats):
        w = O.pack_q8(O.uniform_weights(rows, n, 100 + k))
        ws = (1e-3 + 9e-3 * np.random.default_rng(k).random(rows)).astype(np.float32)
        b = np.random.default_rng(50 + k).standard_normal(rows).astype(np.float32) if bias_on else None
        os_ = rows + (8 if k == 1 else 0)
        out0 = np.random.default_rng(7 + k).standard_normal(T * os_).astype(np.float32)
        for rnd in range(2):  # the second round finds the weights' device copy
            out = out0.copy()
            pool_run(nth, gemm_items(rows, T, nth),
                     lambda it: tab.gemm_q8(out[it[2] * os_ + it[0]:], os_, w[it[0] * n:], ws[it[0]:],
                                            None if b is None else b[it[0]:], it[1],
                                            _sub_act(pkb, q, d, n, qb, it[2], it[3]), add))
            want = out0.copy()
            O.gemm_q8(want, os_, w, ws, b, rows, qo, do, n, qb, T, add)
            assert out.tobytes() == want.tobytes(), f"matrix {k} round {rnd}"


def test_weight_slices_in_any_order_then_the_whole_matrix(pkb, cuda_device):
    """Slices of one matrix arriving out of order, of two sizes, then the
    whole matrix in one call, then the matrix rewritten after pkb_forget:
    every call the oracle's bits."""
    T, n, qb, rows = 40, 512, 32, 1024
    x = O.seeded_normal(T * n, 77)
    q, d = O.quantize(x, n, qb)
    w = O.pack_q8(O.uniform_weights(rows, n, 8))
    ws = np.linspace(1e-3, 1e-2, rows).astype(np.float32)
    want = np.zeros(T * rows, np.float32)
    O.gemm_q8(want, rows, w, ws, None, rows, q, d, n, qb, T, False)
    for step, order in ((64, [5, 1, 0, 3, 2, 15, 4]), (256, [3, 0, 2, 1])):
        got = np.zeros(T * rows, np.float32)
        order = order + [i for i in range(rows // step) if i not in order]
        for i in order:
            r0 = i * step
            pkb.gemm_q8_host(got[r0:], rows, w[r0 * n:], ws[r0:], None, step, q, d, n, qb, T, False)
        assert got.tobytes() == want.tobytes(), f"slices of {step}"
    got = np.zeros(T * rows, np.float32)
    pkb.gemm_q8_host(got, rows, w, ws, None, rows, q, d, n, qb, T, False)
    assert got.tobytes() == want.tobytes()
    pkb.forget(w)
    w[:] = O.pack_q8(O.uniform_weights(rows, n, 9))
    got = np.zeros(T * rows, np.float32)
    pkb.gemm_q8_host(got, rows, w, ws, None, rows, q, d, n, qb, T, False)
    want = np.zeros(T * rows, np.float32)
    O.gemm_q8(want, rows, w, ws, None, rows, q, d, n, qb, T, False)
    assert got.tobytes() == want.tobytes()
    pkb.forget(w)


@pytest.mark.skipif(not O.have_fast(), reason="the reference's backends are not built (make -C oracle ref)")
def test_benchmark_path_at_full_size(pkb, cuda_device):
    """The benchmark's own path at its full size: the batch's 11,521 frames
    (about 20 tiles a CTA), FF-up, FF-down (adding) and the position product
    (22,978 positions, on a side stream), quantized and multiplied inside one
    CUDA graph whose kernels launch with programmatic dependent launch, each
    result compared byte for byte with the reference's own kernels (its
    picked backend, threaded) on the same inputs."""
    import torch
    T, R, D, F, qb = 11521, 22978, 1024, 4096, 32
    g = torch.Generator(device="cuda").manual_seed(31)
    dev = torch.device("cuda")
    x_att = torch.randn(T * D, device=dev, generator=g)
    x_ff = torch.randn(T * F, device=dev, generator=g) * 3
    x_pos = torch.randn(R * D, device=dev, generator=g)
    mats = {}
    for name, rows, n in (("up", F, D), ("down", D, F), ("pos", D, D)):
        w_pk = torch.randint(-127, 128, (rows * n,), dtype=torch.int8, device=dev, generator=g)
        wp = torch.empty_like(w_pk)
        pkb.repack_q8_dev(wp, w_pk, rows, n)
        ws = 1e-3 + 9e-3 * torch.rand(rows, device=dev, generator=g)
        mats[name] = (w_pk, wp, ws, rows, n)
    qa, da = torch.empty(T * D, dtype=torch.int8, device=dev), torch.empty(T * D // qb, device=dev)
    qf, df = torch.empty(T * F, dtype=torch.int8, device=dev), torch.empty(T * F // qb, device=dev)
    qp, dp = torch.empty(R * D, dtype=torch.int8, device=dev), torch.empty(R * D // qb, device=dev)
    out_up = torch.zeros(T * F, device=dev)
    out_down0 = torch.randn(T * D, device=dev, generator=g)
    out_down = out_down0.clone()
    out_pos = torch.zeros(R * D, device=dev)
    side = torch.cuda.Stream()

    def step():
        s0 = torch.cuda.current_stream()
        side.wait_stream(s0)
        pkb.quantize_dev(qp, dp, x_pos, D, R, D, qb, stream=side.cuda_stream)
        w = mats["pos"]
        pkb.gemm_q8_dev(out_pos, D, w[1], w[2], None, D, qp, dp, D, qb, R, False, stream=side.cuda_stream)
        pkb.quantize_dev(qa, da, x_att, D, T, D, qb)
        w = mats["up"]
        pkb.gemm_q8_dev(out_up, F, w[1], w[2], None, F, qa, da, D, qb, T, False)
        pkb.quantize_dev(qf, df, x_ff, F, T, F, qb)
        w = mats["down"]
        pkb.gemm_q8_dev(out_down, D, w[1], w[2], None, D, qf, df, F, qb, T, True)
        s0.wait_stream(side)

    step()  # the device's set-up comes before the capture
    torch.cuda.synchronize()
    out_down.copy_(out_down0)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    torch.cuda.synchronize()
    assert pkb.device_errors(0) == 0
    checks = (("up", x_att, T, out_up, None), ("down", x_ff, T, out_down, out_down0), ("pos", x_pos, R, out_pos, None))
    for name, x, M, out, before in checks:
        w_pk, _, ws, rows, n = mats[name]
        q, dd = O.fast_quantize(x.cpu().numpy(), n, qb, M)
        want = before.cpu().numpy() if before is not None else np.empty(M * rows, np.float32)
        O.fast_gemm_q8(want, rows, w_pk.cpu().numpy(), ws.cpu().numpy(), None, rows, q, dd, n, qb, M,
                       before is not None)
        got = out.cpu().numpy()
        assert got.tobytes() == want.tobytes(), f"{name}: {int((got.view(np.uint32) != want.view(np.uint32)).sum())} differ"
    del graph


@pytest.mark.parametrize("pinned", [False, True])
def test_quantized_activations_reused_only_while_unchanged(pkb, cuda_device, pinned):
    """A product reads the device copy of activations this library quantized
    only while the caller's bytes and scales are still the ones written:
    unchanged (whole range and a run of frames from inside it), one byte
    changed, one scale changed, and the buffer quantized again - every call
    the oracle's bits for the bytes the caller holds at that moment."""
    import torch
    T, n, qb, rows = 300, 1024, 32, 256
    x = O.seeded_normal(T * n, 91)

    def buf(a):
        if not pinned:
            return a.copy(), None
        t = torch.empty(a.size, dtype={np.dtype(np.float32): torch.float32, np.dtype(np.int8): torch.int8}[a.dtype],
                        pin_memory=True)
        v = t.numpy()
        v[:] = a
        return v, t

    q, tq = buf(np.zeros(T * n, np.int8))
    d, td = buf(np.zeros(T * n // qb, np.float32))
    out, to = buf(np.zeros(T * rows, np.float32))
    w = O.pack_q8(O.uniform_weights(rows, n, 92))
    ws = np.linspace(1e-3, 1e-2, rows).astype(np.float32)
    tab = pkb.Table()
    pkb.forget(w)  # an earlier matrix may have had this address
    up0, down0 = pkb.host_bytes()
    tab.quantize(pkb.PkAct(q.ctypes.data, d.ctypes.data, n, qb, T), x, n)
    up1, down1 = pkb.host_bytes()
    assert (up1 - up0, down1 - down0) == (T * n * 4, T * (n + 4 * (n // qb)) + 4)

    def check(label, t0=0, tn=T, reused=True, weights=False):
        out[:] = 0
        act = pkb.PkAct(q[t0 * n:].ctypes.data, d[t0 * (n // qb):].ctypes.data, n, qb, tn)
        up0, down0 = pkb.host_bytes()
        tab.gemm_q8(out, rows, w, ws, None, rows, act, False)
        up1, down1 = pkb.host_bytes()
        want = np.zeros(tn * rows, np.float32)
        O.gemm_q8(want, rows, w, ws, None, rows, q[t0 * n:(t0 + tn) * n].copy(),
                  d[t0 * (n // qb):(t0 + tn) * (n // qb)].copy(), n, qb, tn, False)
        assert out[:tn * rows].tobytes() == want.tobytes(), label
        # the copies the call counted: row scales (and the biases' slot),
        # the activations unless their device copy was read, the weights
        # when uploaded; the results and the error word back
        up = 2 * rows * 4 + (0 if reused else tn * (n + 4 * (n // qb))) + (rows * n if weights else 0)
        assert (up1 - up0, down1 - down0) == (up, tn * rows * 4 + 4), label

    check("unchanged", weights=True)
    check("frames 37..236 from inside", 37, 200)
    q[5 * n + 17] = np.int8(-q[5 * n + 17] - 1)
    check("one byte changed", reused=False)
    d[3] = np.float32(d[3] * 2)
    check("one scale changed", reused=False)
    x2 = O.seeded_normal(T * n, 93)
    tab.quantize(pkb.PkAct(q.ctypes.data, d.ctypes.data, n, qb, T), x2, n)
    check("quantized again")
    pkb.forget(q)
    pkb.forget(w)
    del tq, td, to
