#!/usr/bin/env python3
"""libpktito's int8 path on B200: the batched encoder benchmark.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the benchmark configuration "batched encoder"): 64 independent
segments of seeded lengths uniform in 2-30 s (25-375 encoder frames each),
through the int8 GEMM path of a 24-layer, d_model 1024 Parakeet-shaped
encoder with random int8 weights: per layer its eleven products (feed-forward
up/down twice, q/k/v, the position projection over 2T-1 rows, attention out,
pointwise convolutions 1024->2048 and 1024->1024, core/encoder.c:329-368),
plus the subsampling's three (core/encoder.c:218-251, 463-465); every
product's float32 input quantized (blocks of 32) and multiplied, each input
once as the reference does (q, k and v share the layer's normed input; the
position input is quantized once a forward pass). The
segments' frames are concatenated into one M per product, which is
bit-identical per frame to running them one by one (a product's columns are
independent). The float parts between products (norms, attention, GLU,
depthwise convolution) are outside the int8 path and not timed; each
product's input is a resident float32 activation ~N(0,1).

A step is one pass over the batch: 267 products and 196 quantizations. value
is whole-job int8 TOPS (2*M*N*K summed over the products, over every rank);
audio-seconds per second is reported beside it. Multi-GPU: one process per
GPU (torchrun), segments partitioned across the GPUs with no collective on
the data path; the time is the max over ranks, the work the sum. Weak
scaling (the default): every GPU takes configs[3]'s batch of 64 segments
(the same seeded lengths on each), so the work per GPU is fixed as the GPUs
are added. `--scaling strong`: the one batch of 64
segments is dealt across the GPUs longest first, so each GPU's share shrinks
as 1/N (at 8 GPUs about 1,440 frames a GPU, where an N = 1024 product has 96
tiles of 128 x 128 for 148 SMs). The long-form workload always
splits its one hour across the GPUs.

`--impl reference` times the reference's own CPU backend (the one its picker
chooses on this host, built from its sources into oracle/_ref) on a bounded
sample of the same products, on all host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# Each host thread that calls the reference-facing table drives three CUDA
# streams of its own (uploads, kernels, downloads). With the runtime's
# default of 8 hardware queues a device, the e2e legs' streams (and torch's)
# share queues and one lane's copies wait behind another's; measured on B200
# in one call, the 2-lane e2e leg ran at 10.9 TOPS with the default and 14.2
# with 32 queues. Read when CUDA starts, so set before anything starts it.
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

METRIC = "int8 GEMM TOPS (% of B200 int8 peak); encoder audio-s/s at 1/2/4/8 GPUs"
SEGMENTS = 64
LAYERS = 24
D, F, C = 1024, 4096, 256
HEADS = 8  # the FastConformer's attention heads (dk 128)
QB = 32
SEED = 20261201
CONCURRENT = ("q", "k", "v", "pos")  # a layer's products that read no other's results
CHECK_LAYERS = (-1, 0, LAYERS - 1)  # the subsampling (-1) and the layers whose results are checked
WORKLOAD = "batched"  # configs[3]; "longform": configs[4]
J, VOCAB_OUT = 640, 8208  # the TDT joint: hidden width, outputs (8192 + 1 + 5 durations, padded to 16)


# ---------------------------------------------------------------- workload --

def draw_segments(seed: int) -> list[tuple[float, int, int, int]]:
    """(seconds, T0, T2, T3) of 64 segments of seeded lengths: mel frames at
    100/s, each 2x subsampling stage ceil-halving (core/encoder.c:430)."""
    rng = np.random.default_rng(seed)
    out = []
    for sec in rng.uniform(2.0, 30.0, SEGMENTS):
        t0 = int(sec * 100)
        t1 = (t0 + 1) // 2
        t2 = (t1 + 1) // 2
        t3 = (t2 + 1) // 2
        out.append((float(sec), t0, t2, t3))
    return out


def longform_chunks() -> list[tuple[float, int, int, int]]:
    """(seconds, T0, T2, T3) of the long-form workload's chunks:
    the hour cut by the reference's own segmenter and chunker
    (tests/golden/longform_chunks.json, written by
    tests/golden/make_longform.py); mel frames = samples / hop 160
    (pk_mel_frames, core/mel.c:32), each 2x subsampling stage ceil-halving."""
    with open(os.path.join(ROOT, "tests", "golden", "longform_chunks.json")) as f:
        doc = json.load(f)
    out = []
    for a, b in doc["chunks"]:
        t0 = (b - a) // 160
        t1 = (t0 + 1) // 2
        t2 = (t1 + 1) // 2
        t3 = (t2 + 1) // 2
        out.append(((b - a) / doc["rate"], t0, t2, t3))
    return out


def partition(segs, world: int) -> list[list[int]]:
    """The segments dealt to `world` GPUs longest first, each to the GPU with
    the fewest encoder frames so far (ties to the lower rank), as the
    reference deals chunks to lanes (core/asr.c:373-398)."""
    order = sorted(range(len(segs)), key=lambda i: (-segs[i][3], i))
    load = [0] * world
    share: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        share[r].append(i)
        load[r] += segs[i][3]
    return [sorted(s) for s in share]


def segments(rank: int, world: int = 1, scaling: str = "weak") -> list[tuple[float, int, int, int]]:
    """The rank's segments. Weak scaling: configs[3]'s batch of 64 segments
    on every GPU (the same seeded lengths, so each GPU's work is the same and
    fixed as GPUs are added; per-rank draws would make the job's time the
    largest draw's, up to 6 % more work than the mean at 8 GPUs). Strong
    scaling: the rank's share of the one batch, partitioned across the GPUs."""
    if WORKLOAD == "longform":
        segs = longform_chunks()
        return [segs[i] for i in partition(segs, world)[rank]]
    if scaling == "weak":
        return draw_segments(SEED)
    segs = draw_segments(SEED)
    return [segs[i] for i in partition(segs, world)[rank]]


def products(segs) -> list[dict]:
    """The step's products: name, rows (N), n (K), M, add, bias, layer, and
    inp, the quantized activation the product reads: q, k and v read one
    (the layer's normed input, core/encoder.c:345-350), every layer's
    position product reads the one quantized once a forward pass
    (core/encoder.c:469); every other product has its own."""
    t3 = sum(s[3] for s in segs)
    r = sum(2 * s[3] - 1 for s in segs)
    t2 = sum(s[2] for s in segs)
    prods = [dict(name="sub_pw1", rows=C, n=C, M=t2 * 32, add=0, bias=1, layer=-1),
             dict(name="sub_pw2", rows=C, n=C, M=t3 * 16, add=0, bias=1, layer=-1),
             dict(name="sub_out", rows=D, n=F, M=t3, add=0, bias=1, layer=-1)]
    for l in range(LAYERS):
        prods += [dict(name="ff1_up", rows=F, n=D, M=t3, add=0, bias=0, layer=l),
                  dict(name="ff1_down", rows=D, n=F, M=t3, add=1, bias=0, layer=l),
                  dict(name="q", rows=D, n=D, M=t3, add=0, bias=0, layer=l),
                  dict(name="k", rows=D, n=D, M=t3, add=0, bias=0, layer=l),
                  dict(name="v", rows=D, n=D, M=t3, add=0, bias=0, layer=l),
                  dict(name="pos", rows=D, n=D, M=r, add=0, bias=0, layer=l),
                  dict(name="o", rows=D, n=D, M=t3, add=1, bias=0, layer=l),
                  dict(name="pw1", rows=2 * D, n=D, M=t3, add=0, bias=0, layer=l),
                  dict(name="pw2", rows=D, n=D, M=t3, add=1, bias=0, layer=l),
                  dict(name="ff2_up", rows=F, n=D, M=t3, add=0, bias=0, layer=l),
                  dict(name="ff2_down", rows=D, n=F, M=t3, add=1, bias=0, layer=l)]
    for p in prods:
        p["inp"] = ("ape" if p["name"] == "pos" else f"{p['layer']}:att" if p["name"] in ("q", "k", "v")
                    else f"{p['layer']}:{p['name']}")
    return prods


def joint_steps(segs) -> list[int]:
    """The long-form workload's TDT joint in lockstep over the rank's chunks
    (core/decoder.c:121-147, one joint output a frame): at step i the chunks
    still longer than i frames."""
    if WORKLOAD != "longform" or not segs:
        return []
    return [sum(1 for sg in segs if sg[3] > i) for i in range(max(sg[3] for sg in segs))]


def step_ops(prods, segs=None) -> float:
    ops = float(sum(2.0 * p["M"] * p["rows"] * p["n"] for p in prods))
    if segs is not None and WORKLOAD == "longform":
        # jenc over every frame (pk_joint_frames, core/decoder.c:149-156), jout at each lockstep step
        ops += 2.0 * sum(sg[3] for sg in segs) * J * D + sum(2.0 * m * VOCAB_OUT * J for m in joint_steps(segs))
    return ops


def audio_seconds(segs) -> float:
    return float(sum(s[0] for s in segs))


# ------------------------------------------------------------------ clocks --

class ClockSampler:
    """nvidia-smi's clocks and throttle reasons, sampled every 200 ms while
    the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU baseline --



def cpu_baseline(prods, min_s: float = 10.0) -> dict:
    """The reference's own CPU backend (its picker's choice, oracle/_ref) on a
    bounded sample: the subsampling's three products and one layer's eleven,
    each at the batch's M, on every host core. Passes over the sample repeat
    until at least `min_s` seconds of CPU work have run (at most 8); the rate
    is the median pass's."""
    import ctypes
    so = os.path.join(ROOT, "oracle", "_ref", "libcpubench.so")
    if not os.path.exists(so):
        return {"value": None, "unit": "TOPS", "cores": None, "kind": "reference",
                "sample": "unavailable: oracle/_ref/libcpubench.so not built"}
    lib = ctypes.CDLL(so)
    lib.cpub_backend.restype = ctypes.c_char_p
    lib.cpub_backend.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    lib.cpub_time.restype = ctypes.c_double
    lib.cpub_time.argtypes = [ctypes.c_uint32] * 5 + [ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                                      ctypes.POINTER(ctypes.c_double)]
    picks = ctypes.create_string_buffer(512)
    backend = lib.cpub_backend(picks, 512).decode()
    cores = os.cpu_count() or 1
    sample = [p for p in prods if p["layer"] in (-1, 0)]
    qs = ctypes.c_double()
    t_start = time.time()
    reps = max(1, int(os.environ.get("PKB_CPU_REPS", "3")))
    rates = []
    while len(rates) < 8 and (not rates or time.time() - t_start < min_s):
        ops = t = 0.0
        for p in sample:
            sec = lib.cpub_time(p["rows"], p["n"], p["M"], QB, p["add"], cores, reps, 1, ctypes.byref(qs))
            if sec > 0:
                ops += 2.0 * p["M"] * p["rows"] * p["n"]
                t += sec
        if t > 0:
            rates.append(ops / t / 1e12)
        else:
            break
    value = float(np.median(rates)) if rates else None
    return {"value": value, "unit": "TOPS", "cores": cores, "kind": "reference",
            "backend": backend, "picks": picks.value.decode(),
            "sample": f"{len(sample)} products (subsampling + layer 0) at the batch's M, quantize + product, "
                      f"best of {reps} timed runs after a warm one each; {len(rates)} passes, median pass rate; "
                      f"{time.time() - t_start:.1f} s of CPU work"}


# ------------------------------------------------------------ our GPU arm --

class Model:
    """Device-resident weights (PK_Q8 bytes repacked once, as at load time),
    activations and outputs for one rank's workload. Every product has an
    output buffer of its own, so that after a step each product's results
    are still there to be checked."""

    def __init__(self, prods, dev, seed, segs=None):
        import torch
        import libpktito_b200 as P
        self.P, self.torch = P, torch
        g = torch.Generator(device=dev).manual_seed(seed)
        self.w, self.ws, self.bias, self.w_pk = {}, {}, {}, {}
        for p in prods:
            key = (p["layer"], p["name"])
            if key in self.w:
                continue
            rows, n = p["rows"], p["n"]
            # random weights uniform in [-127, 127]: in the model file's PK_Q8
            # panel order they are random bytes too; repacked on the device
            # as at load time
            w_pk = torch.randint(-127, 128, (rows * n,), dtype=torch.int8, device=dev, generator=g)
            wpack = torch.empty(rows * n, dtype=torch.int8, device=dev)
            P.repack_q8_dev(wpack, w_pk, rows, n)
            self.w[key] = wpack
            if p["layer"] in CHECK_LAYERS:
                self.w_pk[key] = w_pk  # the model file's bytes, for the parity check
            self.ws[key] = (1e-3 + 9e-3 * torch.rand(rows, device=dev, generator=g)).float()
            self.bias[key] = torch.randn(rows, device=dev, generator=g) if p["bias"] else None
        self.x, self.q, self.d = {}, {}, {}
        for p in prods:
            xk = (p["M"], p["n"])
            if xk not in self.x:
                self.x[xk] = torch.randn(p["M"] * p["n"], device=dev, generator=g)
                self.q[xk] = torch.empty(p["M"] * p["n"], dtype=torch.int8, device=dev)
                self.d[xk] = torch.empty(p["M"] * p["n"] // QB, dtype=torch.float32, device=dev)
        self.out = [torch.zeros(p["M"] * p["rows"], device=dev) for p in prods]
        self.prods = prods
        self.joint = None
        if segs is not None and WORKLOAD == "longform":
            # the TDT joint: jenc over the rank's frames, then jout
            # in lockstep over its chunks, every input a whole row a block
            T3, steps = sum(sg[3] for sg in segs), joint_steps(segs)
            mmax = max(steps)

            def mat(rows, n):
                w_pk = torch.randint(-127, 128, (rows * n,), dtype=torch.int8, device=dev, generator=g)
                wp = torch.empty_like(w_pk)
                P.repack_q8_dev(wp, w_pk, rows, n)
                return (w_pk, wp, (1e-3 + 9e-3 * torch.rand(rows, device=dev, generator=g)).float(),
                        torch.randn(rows, device=dev, generator=g))

            self.joint = {"T3": T3, "steps": steps, "jenc": mat(J, D), "jout": mat(VOCAB_OUT, J),
                          "xe": torch.randn(T3 * D, device=dev, generator=g),
                          "qe": torch.empty(T3 * D, dtype=torch.int8, device=dev), "de": torch.empty(T3, device=dev),
                          "f": torch.empty(T3 * J, device=dev),
                          "z": torch.randn(mmax * J, device=dev, generator=g),
                          "qz": torch.empty(mmax * J, dtype=torch.int8, device=dev),
                          "dz": torch.empty(mmax, device=dev), "logits": torch.empty(mmax * VOCAB_OUT, device=dev)}
        # q, k, v and the position product of a layer depend on no one of
        # them (core/encoder.c:347-352): they run side by side on streams of
        # their own
        self.side = [torch.cuda.Stream(dev) for _ in range(len(CONCURRENT))]
        torch.cuda.synchronize()

    def step(self):
        P, torch = self.P, self.torch
        s0 = torch.cuda.current_stream()
        held = {}  # the input each activation buffer holds, quantized

        def quantize(p, s):
            xk = (p["M"], p["n"])
            if held.get(xk) != p["inp"]:
                P.quantize_dev(self.q[xk], self.d[xk], self.x[xk], p["n"], p["M"], p["n"], QB, stream=s.cuda_stream)
                held[xk] = p["inp"]

        def gemm(i, s):
            p = self.prods[i]
            key, xk = (p["layer"], p["name"]), (p["M"], p["n"])
            P.gemm_q8_dev(self.out[i], p["rows"], self.w[key], self.ws[key], self.bias[key], p["rows"],
                          self.q[xk], self.d[xk], p["n"], QB, p["M"], bool(p["add"]), stream=s.cuda_stream)

        prods = self.prods
        i = 0
        while i < len(prods):
            p = prods[i]
            if p["name"] != CONCURRENT[0]:
                quantize(p, s0)
                gemm(i, s0)
                i += 1
                continue
            group = list(range(i, i + len(CONCURRENT)))
            assert [prods[j]["name"] for j in group] == list(CONCURRENT)
            for j in group:  # their inputs, once, before the fork
                quantize(prods[j], s0)
            for j, s in zip(group, self.side):
                s.wait_stream(s0)
                gemm(j, s)
            for s in self.side:
                s0.wait_stream(s)
            i += len(CONCURRENT)
        jt = self.joint
        if jt:
            st = s0.cuda_stream
            _, wp, ws, b = jt["jenc"]
            P.quantize_dev(jt["qe"], jt["de"], jt["xe"], D, jt["T3"], D, D, stream=st)
            P.gemm_q8_dev(jt["f"], J, wp, ws, b, J, jt["qe"], jt["de"], D, D, jt["T3"], False, stream=st)
            _, wp, ws, b = jt["jout"]
            for m in jt["steps"]:
                P.quantize_dev(jt["qz"], jt["dz"], jt["z"], J, m, J, J, stream=st)
                P.gemm_q8_dev(jt["logits"], VOCAB_OUT, wp, ws, b, VOCAB_OUT, jt["qz"], jt["dz"], J, J, m, False,
                              stream=st)


def parity_check(model, graph, world: int) -> dict:
    """Ties the timed step's results to the reference's bits. After the timed
    region, the step runs once more exactly as it was timed (the same CUDA
    graph: programmatic dependent launch, q/k/v/pos on side streams, about
    20 tiles a CTA at the batch's M), and every product of the subsampling
    and of layers CHECK_LAYERS is compared byte for byte with the
    reference's own kernels on the same inputs: each product's float input
    quantized by the reference, its results computed by the reference from
    those bytes (for the products that add, onto the results the replay
    found). The checker is the backend the reference's picker chooses on
    this host (amx-int8 on an AMX Xeon; the reference's q8check holds it to
    ref's bits), built from its sources into oracle/_ref and run on the
    host's cores; nothing timed runs through it."""
    torch = model.torch
    try:
        from oracle import oracle as O
        if not O.have_fast():
            raise FileNotFoundError("oracle/_ref/libcpubench.so is not built")
        backend = O.fast_backend()
    except Exception as e:  # noqa: BLE001
        return {"checked": 0, "equal": 0, "unavailable": str(e)}
    prods = model.prods
    idx = [i for i, p in enumerate(prods) if p["layer"] in CHECK_LAYERS]
    before = {i: model.out[i].cpu().numpy() for i in idx if prods[i]["add"]}
    if graph is not None:
        graph.replay()
    else:
        model.step()
    torch.cuda.synchronize()
    threads = max(1, (os.cpu_count() or 1) // max(1, world))
    checked = equal = 0
    bad = []
    qd = {}
    for xk in sorted({(prods[i]["M"], prods[i]["n"]) for i in idx}):
        M, n = xk
        q, d = O.fast_quantize(model.x[xk].cpu().numpy(), n, QB, M, threads=threads)
        same = (np.array_equal(model.q[xk].cpu().numpy().reshape(M, n), q) and
                model.d[xk].cpu().numpy().tobytes() == d.tobytes())
        checked += 1
        equal += int(same)
        if not same:
            bad.append(f"quantize M {M} x n {n}")
        qd[xk] = (q, d)
    for i in idx:
        p = prods[i]
        key, xk = (p["layer"], p["name"]), (p["M"], p["n"])
        want = before[i].copy() if p["add"] else np.empty(p["M"] * p["rows"], np.float32)
        b = model.bias[key].cpu().numpy() if model.bias[key] is not None else None
        O.fast_gemm_q8(want, p["rows"], model.w_pk[key].cpu().numpy(), model.ws[key].cpu().numpy(), b, p["rows"],
                       qd[xk][0], qd[xk][1], p["n"], QB, p["M"], bool(p["add"]), threads=threads)
        same = model.out[i].cpu().numpy().tobytes() == want.tobytes()
        checked += 1
        equal += int(same)
        if not same:
            bad.append(f"{p['name']} layer {p['layer']}")
    jt = model.joint
    if jt:
        # jenc over the frames, and jout at the last lockstep step
        for name, x, M, n, rows, out in (("jenc", jt["xe"], jt["T3"], D, J, jt["f"]),
                                         ("jout", jt["z"], jt["steps"][-1], J, VOCAB_OUT, jt["logits"])):
            w_pk, _, ws, b = jt[name]
            q, d = O.fast_quantize(x.cpu().numpy()[:M * n], n, n, M, threads=threads)
            want = np.empty(M * rows, np.float32)
            O.fast_gemm_q8(want, rows, w_pk.cpu().numpy(), ws.cpu().numpy(), b.cpu().numpy(), rows, q, d, n, n, M,
                           False, threads=threads)
            same = out.cpu().numpy()[:M * rows].tobytes() == want.tobytes()
            checked += 1
            equal += int(same)
            if not same:
                bad.append(name)
    return {"checked": checked, "equal": equal, "products": len(idx) + (2 if jt else 0),
            "quantized_inputs": checked - len(idx) - (2 if jt else 0),
            "layers": [l for l in CHECK_LAYERS if l >= 0], "subsampling": -1 in CHECK_LAYERS,
            "path": "the timed CUDA graph replayed once more (PDL, q/k/v/pos on side streams, the batch's M)",
            "checker": f"the reference's {backend} backend (its picker's choice; held to ref's bits by its own "
                       "q8check), built from its sources into oracle/_ref, on the host's cores",
            "mismatches": bad[:8]}


def kernel_roofline(model, prods, sm_mhz: float | None) -> dict:
    """The dominant kernel (the product) timed alone on its most frequent
    shape, with CUDA events on its stream: achieved int8 TOPS over the
    measured peak; beside it the fraction of the fp32 bound its epilogue
    chain has at this qb, and the quantizer's HBM rate on the same input."""
    torch, P = model.torch, model.P
    ok = next(i for i, x in enumerate(prods) if x["name"] == "ff1_up")
    p = prods[ok]
    key, xk = (p["layer"], p["name"]), (p["M"], p["n"])
    s = torch.cuda.current_stream()
    for _ in range(3):
        P.gemm_q8_dev(model.out[ok], p["rows"], model.w[key], model.ws[key], None, p["rows"], model.q[xk],
                      model.d[xk], p["n"], QB, p["M"], False)
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.synchronize()
    e0.record(s)
    for _ in range(reps):
        P.gemm_q8_dev(model.out[ok], p["rows"], model.w[key], model.ws[key], None, p["rows"], model.q[xk],
                      model.d[xk], p["n"], QB, p["M"], False)
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    achieved = 2.0 * p["M"] * p["rows"] * p["n"] / (ms * 1e-3) / 1e12
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        peaks = json.load(open(peaks_path))
        peak, src = 2.0 * float(peaks["bf16_tflops"]), "of measured: 2 x bf16_tflops (burst) of MEASURED_PEAKS.json"
    except (OSError, KeyError, ValueError):
        peak, src = 2.0 * 1590.0, "of fallback: 2 x 1.59 PFLOP/s bf16"
    traffic = None
    prof = os.path.join(ROOT, "profiles", "gemm_q8_traffic.json")
    if os.path.exists(prof):
        try:
            t = json.load(open(prof))
            if (t.get("M"), t.get("rows"), t.get("n")) == (p["M"], p["rows"], p["n"]):
                traffic = t.get("bytes_per_launch")
        except (OSError, ValueError):
            traffic = None
    # the epilogue's own bound: per output and block one exact subtract and
    # one FMA, two fp32 lane-operations, on 128 FP32 lanes a cycle per SM
    mhz = sm_mhz or 1965.0
    lane_ops = 2.0 * p["M"] * p["rows"] * (p["n"] // QB)
    fp32_peak = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count * 128 * mhz * 1e6
    epi = {"lane_ops_per_launch": lane_ops, "achieved_lane_ops_per_s": lane_ops / (ms * 1e-3),
           "peak_lane_ops_per_s": fp32_peak, "frac": lane_ops / (ms * 1e-3) / fp32_peak,
           "note": f"one subtract + one FMA per output per block of {QB}; 128 fp32 lanes/clk/SM at {mhz:.0f} MHz"}
    # the quantizer on the same product's input
    qd = model.q[xk]
    x = model.x[xk]
    for _ in range(3):
        P.quantize_dev(qd, model.d[xk], x, p["n"], p["M"], p["n"], QB)
    s.synchronize()
    e0.record(s)
    for _ in range(reps):
        P.quantize_dev(qd, model.d[xk], x, p["n"], p["M"], p["n"], QB)
    e1.record(s)
    e1.synchronize()
    qms = e0.elapsed_time(e1) / reps
    qbytes = p["M"] * p["n"] * (4 + 1 + 4.0 / QB)
    try:
        hbm = float(json.load(open(peaks_path))["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        hbm = 6650.0
    quant = {"ms_per_launch": qms, "gbs": qbytes / (qms * 1e-3) / 1e9, "peak_gbs": hbm,
             "frac": qbytes / (qms * 1e-3) / 1e9 / hbm, "bytes_per_launch": qbytes,
             "shape": f"T {p['M']} x n {p['n']}, qb {QB}"}
    # fast mode (the reference's qb 64, core/encoder.c:56, core/asr.c:151) on
    # the same shape: half the epilogue's chain per output
    fast = None
    if QB == 32 and p["n"] % 64 == 0:
        q64 = torch.empty_like(model.q[xk])
        d64 = torch.empty(p["M"] * p["n"] // 64, device=q64.device)
        P.quantize_dev(q64, d64, x, p["n"], p["M"], p["n"], 64)
        run64 = lambda: P.gemm_q8_dev(model.out[ok], p["rows"], model.w[key], model.ws[key], None, p["rows"], q64,
                                      d64, p["n"], 64, p["M"], False)
        for _ in range(3):
            run64()
        s.synchronize()
        e0.record(s)
        for _ in range(reps):
            run64()
        e1.record(s)
        e1.synchronize()
        ms64 = e0.elapsed_time(e1) / reps
        a64 = 2.0 * p["M"] * p["rows"] * p["n"] / (ms64 * 1e-3) / 1e12
        lane64 = 2.0 * p["M"] * p["rows"] * (p["n"] // 64)
        fast = {"qb": 64, "ms_per_launch": ms64, "achieved": a64, "frac": a64 / peak,
                "epilogue_fp32_frac": lane64 / (ms64 * 1e-3) / fp32_peak,
                "note": "the same product in fast mode (blocks of 64), timed alone with CUDA events"}
        del q64, d64
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "fast_mode_qb64": fast,
            "traffic": traffic, "kernel": "pkb::gemm::gemm_q8_kernel",
            "shape": f"M {p['M']} x N {p['rows']} x K {p['n']}, qb {QB}", "ms_per_launch": ms,
            "peak_note": src + "; int8 dense is twice bf16 dense on B200 (4.5 vs 2.25 PFLOP/s nominal)",
            "algorithmic_ops_per_launch": 2.0 * p["M"] * p["rows"] * p["n"],
            "epilogue_fp32": epi, "quantize": quant}


def producers_roofline(model, T: int) -> dict:
    """The fused producers of the product's inputs (the reference's normq,
    siluq_tile and glu_item + dw_item, core/encoder.c:112-183) at this rank's
    frame count, each timed alone with CUDA events on its stream, its inputs
    rotated over buffers that together exceed the 126 MB L2: achieved bytes
    (the input read once, q and d written, the small per-column operands)
    over the measured HBM copy rate."""
    torch, P = model.torch, model.P
    s = torch.cuda.current_stream()
    try:
        hbm = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"])
        src = "of measured: hbm_gbs of MEASURED_PEAKS.json"
    except (OSError, KeyError, ValueError):
        hbm, src = 6650.0, "of fallback: 6.65 TB/s"
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 99)
    K = 9  # the FastConformer's depthwise kernel

    def timed(fn, nbuf: int) -> float:
        for i in range(3):
            fn(i % nbuf)
        s.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 12 * nbuf
        e0.record(s)
        for i in range(reps):
            fn(i % nbuf)
        e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    out = {}
    q = torch.empty(T * F, dtype=torch.int8, device="cuda")
    d = torch.empty(T * F // QB, dtype=torch.float32, device="cuda")
    # LayerNorm -> quantize: 47 MB an input at T = 11521, three of them
    xs = [torch.randn(T * D, device="cuda", generator=g) for _ in range(3)]
    w, b = torch.randn(D, device="cuda", generator=g), torch.randn(D, device="cuda", generator=g)
    ms = timed(lambda i: P.layernorm_quantize_dev(q, d, xs[i], D, T, D, QB, w, b, 1e-5), 3)
    byt = T * D * (4 + 1 + 4.0 / QB) + 2 * D * 4
    out["layernorm_quantize"] = {"us": ms * 1e3, "gbs": byt / (ms * 1e-3) / 1e9, "frac": byt / (ms * 1e-3) / 1e9 / hbm,
                                 "bytes_per_launch": byt, "shape": f"T {T} x n {D}, qb {QB}",
                                 "launches_per_step": 4 * LAYERS}
    del xs
    # SiLU -> quantize: the FF-up output, 189 MB
    u = torch.randn(T * F, device="cuda", generator=g) * 4
    ms = timed(lambda i: P.silu_quantize_dev(q, d, u, F, T, F, QB), 1)
    byt = T * F * (4 + 1 + 4.0 / QB)
    out["silu_quantize"] = {"us": ms * 1e3, "gbs": byt / (ms * 1e-3) / 1e9, "frac": byt / (ms * 1e-3) / 1e9 / hbm,
                            "bytes_per_launch": byt, "shape": f"T {T} x n {F}, qb {QB}",
                            "launches_per_step": 2 * LAYERS}
    del u
    # GLU + depthwise conv -> quantize from pw1's output: 94 MB, two of them
    xg = [torch.randn(T * 2 * D, device="cuda", generator=g) for _ in range(2)]
    wd, bd = torch.randn(D * K, device="cuda", generator=g) * 0.3, torch.randn(D, device="cuda", generator=g)
    ms = timed(lambda i: P.dwconv_quantize_dev(q, d, None, D, xg[i], 2 * D, T, D, wd, bd, K, True, QB), 2)
    byt = T * D * (8 + 1 + 4.0 / QB) + D * (K + 1) * 4
    out["glu_dwconv_quantize"] = {"us": ms * 1e3, "gbs": byt / (ms * 1e-3) / 1e9,
                                  "frac": byt / (ms * 1e-3) / 1e9 / hbm, "bytes_per_launch": byt,
                                  "shape": f"T {T} x C {D}, K {K}, qb {QB}", "launches_per_step": LAYERS}
    del xg
    out["bound"] = "hbm"
    out["peak_gbs"] = hbm
    out["peak_note"] = src
    out["note"] = ("bytes: the input read once, q and d written, w/b or taps; inputs rotated over buffers "
                   "larger than L2; each producer bit-exact to the reference's float step + quantize")
    return out


def attention_inputs(torch, Ts: list[int], seed: int):
    """Seeded q, K, V and P rows of a batch of segments (the products'
    outputs: frames one segment after another, P's 2T - 1 rows a segment
    likewise), the position biases and the segment table."""
    M, Rs = sum(Ts), sum(2 * t - 1 for t in Ts)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q, k, v = (torch.randn(M * D, device="cuda", generator=g) for _ in range(3))
    p = torch.randn(Rs * D, device="cuda", generator=g)
    bu, bv = (0.1 * torch.randn(D, device="cuda", generator=g) for _ in range(2))
    segs, f, r = [], 0, 0
    for t in Ts:
        segs.append((t, f, r))
        f += t
        r += 2 * t - 1
    return q, k, v, p, bu, bv, segs


def attention_check(torch, o, q, k, v, p, bu, bv, segs, picks) -> dict:
    """The attention's outputs of the picked segments against the oracle's
    att_item (core/encoder.c:280-326), K, P and V laid out as its panels."""
    from oracle import oracle as O
    dk = D // HEADS
    qh, kh, vh, ph, oh = (t.view(-1, D).cpu().numpy() for t in (q, k, v, p, o))
    bu_h, bv_h = bu.cpu().numpy(), bv.cpu().numpy()
    bad = []
    for i in picks:
        T, f, r = segs[i]
        R = 2 * T - 1
        Tp, Pp = (T + 15) // 16 * 16, (R + 15) // 16 * 16 + 16
        kp = O.panels_kp(np.ascontiguousarray(kh[f:f + T]).reshape(-1), T, Tp, D, dk)
        pp = O.panels_kp(np.ascontiguousarray(ph[r:r + R]).reshape(-1), R, Pp, D, dk)
        vp = np.ascontiguousarray(vh[f:f + T].reshape(T, D // 16, 16).transpose(1, 0, 2)).reshape(-1)
        want = O.attention(np.ascontiguousarray(qh[f:f + T]), D, kp, pp, vp, bu_h, bv_h, T, D, HEADS)
        if oh[f:f + T].tobytes() != want.tobytes():
            bad.append(int(T))
    return {"checked_segments": [int(segs[i][0]) for i in picks], "equal": len(picks) - len(bad), "mismatches": bad,
            "checker": "the oracle's att_item (oracle/q8_oracle.c), pinned to the reference's ref backend"}


def attention_timing(model, segs, sm_mhz) -> dict:
    """The attention's float work of one layer (att_item, core/encoder.c:
    280-326: every head and block of 16 queries of every segment) in one
    launch of pkb_attention_rows_dev, K, V and P as the products' rows,
    timed with CUDA events (the batch's q, K, V and P are 190 MB, over L2).
    FLOPs: 2 x 3 T^2 dk a head (the scores, the position products at the
    pairs the softmax reads, the weighted values); peak: the FP32 pipe's 128
    lanes a cycle per SM (2 FLOPs an FMA) at the clock sampled in the timed
    region. Then the shortest, a middle and the longest segment's outputs
    against the oracle."""
    torch, P = model.torch, model.P
    Ts = [sg[3] for sg in segs]
    q, k, v, p, bu, bv, sl = attention_inputs(torch, Ts, SEED + 123)
    o = torch.empty(sum(Ts) * D, device="cuda")
    s = torch.cuda.current_stream()

    def run():
        P.attention_rows_dev(o, D, q, D, k, D, v, D, p, D, bu, bv, D, HEADS, sl)

    for _ in range(3):
        run()
    s.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record(s)
    for _ in range(reps):
        run()
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    dk = D // HEADS
    flops = sum(6.0 * HEADS * t * t * dk for t in Ts)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    mhz = float(sm_mhz or 1965.0)
    peak = sms * 128 * 2 * mhz * 1e6
    order = sorted(range(len(Ts)), key=lambda i: Ts[i])
    picks = [order[0], order[len(order) // 2], order[-1]]
    return {"us": ms * 1e3, "tflops": flops / (ms * 1e-3) / 1e12, "peak_tflops": peak / 1e12,
            "frac": flops / (ms * 1e-3) / peak, "bound": "fp32",
            "peak_note": f"nominal: {sms} SMs x 128 FP32 lanes x 2 FLOPs at the sampled {mhz:.0f} MHz",
            "flops_per_launch": flops, "segments": len(Ts), "frames": sum(Ts), "heads": HEADS, "dk": dk,
            "launches_per_step": LAYERS,
            "parity": attention_check(torch, o, q, k, v, p, bu, bv, sl, picks)}


def encoder_layer_timing(model, segs) -> dict:
    """One encoder layer on the device (libpktito_b200.encoder.layer_dev:
    layer(), core/encoder.c:338-368) over the rank's segments: its 11
    products, four LayerNorm -> quantize, two SiLU -> quantize, the
    attention over every segment and head, the quantization of its output,
    GLU + depthwise convolution -> quantize a segment at a time and the out
    norm, seeded weights, captured as one CUDA graph and timed with CUDA
    events; then the shortest segment's output against the oracle's
    composition of the same steps."""
    torch, P = model.torch, model.P
    from libpktito_b200.encoder import PRODUCTS, Batch, Buffers, layer_dev, product_shapes
    from oracle import oracle as O
    K, EPS = 9, 1e-5
    g = np.random.default_rng(SEED + 91)
    L, Ld = {}, {}
    for name in PRODUCTS:
        rows, n = product_shapes(D, F)[name]
        w_pk = O.pack_q8(g.integers(-127, 128, (rows, n), dtype=np.int8))
        ws = (1e-4 + 9e-4 * g.random(rows)).astype(np.float32)
        src = torch.from_numpy(w_pk).cuda()
        wd = torch.empty(rows * n, dtype=torch.int8, device="cuda")
        P.repack_q8_dev(wd, src, rows, n)
        L[name], Ld[name] = (w_pk, ws), (wd, torch.from_numpy(ws).cuda())
    for name in ("ff1", "att", "conv", "ff2", "out"):
        L[name + "_nw"] = (1 + 0.1 * g.standard_normal(D)).astype(np.float32)
        L[name + "_nb"] = (0.1 * g.standard_normal(D)).astype(np.float32)
    L["bias_u"], L["bias_v"] = ((0.1 * g.standard_normal(D)).astype(np.float32) for _ in range(2))
    L["dw"], L["dw_b"] = (0.3 * g.standard_normal(D * K)).astype(np.float32), (0.1 * g.standard_normal(D)).astype(
        np.float32)
    for k, v in L.items():
        if not isinstance(v, tuple):
            Ld[k] = torch.from_numpy(v).cuda()
    sl, f, r = [], 0, 0
    for sg in segs:
        sl.append((sg[3], f, r))
        f += sg[3]
        r += 2 * sg[3] - 1
    batch = Batch(sl)
    x0 = torch.randn(batch.frames * D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(SEED + 92))
    ape = torch.randn(batch.positions * D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(SEED + 93))
    aq = torch.empty(batch.positions * D, dtype=torch.int8, device="cuda")
    ad = torch.empty(batch.positions * D // QB, device="cuda")
    P.quantize_dev(aq, ad, ape, D, batch.positions, D, QB)
    buf = Buffers(torch, batch.frames, batch.positions, D, F, QB)
    x = x0.clone()
    s = torch.cuda.Stream()
    l0 = P.launch_count()
    with torch.cuda.stream(s):
        layer_dev(x, Ld, batch, aq, ad, D, F, HEADS, K, QB, EPS, buf)
    s.synchronize()
    launches = P.launch_count() - l0
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s, capture_error_mode="relaxed"):
        layer_dev(x, Ld, batch, aq, ad, D, F, HEADS, K, QB, EPS, buf)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    with torch.cuda.stream(s):
        x.copy_(x0)
        graph.replay()
        e0.record(s)
        for _ in range(reps):
            graph.replay()
        e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    # parity: one layer from x0, the shortest segment against the oracle
    with torch.cuda.stream(s):
        x.copy_(x0)
        graph.replay()
    s.synchronize()
    del graph
    i = min(range(len(sl)), key=lambda j: sl[j][0])
    T, f, r = sl[i]
    xh, ah = x0.view(-1, D)[f:f + T].cpu().numpy().reshape(-1), ape.view(-1, D)[r:r + 2 * T - 1].cpu().numpy()
    want = encoder_layer_oracle(xh, T, L, ah.reshape(-1), K, EPS)
    got = x.view(-1, D)[f:f + T].cpu().numpy().reshape(-1)
    ops = 2.0 * (batch.frames * D * (4 * F + 7 * D) + batch.positions * D * D)
    return {"ms": ms, "segments": len(sl), "frames": batch.frames, "launches": launches,
            "int8_tops": ops / (ms * 1e-3) / 1e12, "encoder_ms_24_layers": 24 * ms,
            "audio_s_per_s": audio_seconds(segs) / (24 * ms * 1e-3),
            "note": "the layer's int8 products, its float steps (norms, SiLU, attention, GLU + depthwise "
                    "convolution) and quantizations, all on the device; the subsampling and the position "
                    "embeddings' quantization once a forward pass are not in it",
            "parity": {"segment_frames": int(T), "equal": bool(got.tobytes() == want.tobytes()),
                       "checker": "the oracle's composition of the layer's steps, each pinned to the reference's"}}


def encoder_layer_oracle(x, T: int, L: dict, ape, K: int, eps: float):
    """layer() (core/encoder.c:338-368) on one segment with the oracle."""
    from oracle import oracle as O
    x = x.copy()
    qb = QB

    def prod(out, name, q, d, n, add, Tn):
        w, ws = L[name]
        O.gemm_q8(out, ws.size, w, ws, None, ws.size, q, d, n, qb, Tn, add)

    def ff(pre):
        q, d = O.layernorm_quantize(x, D, T, D, qb, L[pre + "_nw"], L[pre + "_nb"], eps)
        u = np.zeros(T * F, np.float32)
        prod(u, pre + "_up", q, d, D, False, T)
        q2, d2 = O.silu_quantize(u, F, T, F, qb)
        prod(x, pre + "_down", q2, d2, F, True, T)

    ff("ff1")
    q, d = O.layernorm_quantize(x, D, T, D, qb, L["att_nw"], L["att_nb"], eps)
    Q, Kr, V = (np.zeros(T * D, np.float32) for _ in range(3))
    for name, out in (("q", Q), ("k", Kr), ("v", V)):
        prod(out, name, q, d, D, False, T)
    R = 2 * T - 1
    aq, ad = O.quantize(ape, D, qb, R, D)
    Pr = np.zeros(R * D, np.float32)
    prod(Pr, "pos", aq, ad, D, False, R)
    dk = D // HEADS
    Tp, Pp = (T + 15) // 16 * 16, (R + 15) // 16 * 16 + 16
    vp = np.ascontiguousarray(V.reshape(T, D // 16, 16).transpose(1, 0, 2)).reshape(-1)
    o = O.attention(Q, D, O.panels_kp(Kr, T, Tp, D, dk), O.panels_kp(Pr, R, Pp, D, dk), vp, L["bias_u"], L["bias_v"],
                    T, D, HEADS)
    qo, do = O.quantize(o, D, qb, T, D)
    prod(x, "o", qo, do, D, True, T)
    q, d = O.layernorm_quantize(x, D, T, D, qb, L["conv_nw"], L["conv_nb"], eps)
    U = np.zeros(T * 2 * D, np.float32)
    prod(U, "pw1", q, d, D, False, T)
    qc, dc, _ = O.dwconv_quantize(U, 2 * D, T, D, L["dw"], L["dw_b"], K, True, qb)
    prod(x, "pw2", qc, dc, D, True, T)
    ff("ff2")
    return O.layernorm(x, D, T, D, L["out_nw"], L["out_nb"], eps).reshape(-1)


def tdt_model_synthetic(P_: int = 640, J: int = 640, V: int = 8192, layers: int = 2, seed: int = SEED + 321):
    """The TDT decoder's weights at the model's shapes (pred_hidden 640,
    joint 640, vocab 8192 + blank, durations 0-4: jout 8208 x 640), seeded:
    PK_Q8 bytes uniform, scales and biases in small ranges; the blank's bias
    raised and duration 0's lowered so that a segment emits about a token
    every three frames, most of them moving on 2 frames or more (measured
    with the oracle: 20 tokens over 60 seeded frames), as speech does."""
    from oracle import oracle as O  # PK_Q8 packing of the seeded rows
    g = np.random.default_rng(seed)
    nd = 5
    nop = (V + 1 + nd + 15) // 16 * 16

    def q8(rows, n):
        return O.pack_q8(g.integers(-127, 128, (rows, n), dtype=np.int8))

    def sc(n):
        return (1e-4 + 9e-4 * g.random(n)).astype(np.float32)
    m = dict(P=P_, L=layers, J=J, V=V, n_dur=nd, max_symbols=10, n_out_pad=nop,
             dur=np.arange(nd, dtype=np.uint32), embed=(g.standard_normal((V + 1) * P_) * 0.5).astype(np.float32))
    m["wx"] = np.concatenate([q8(4 * P_, P_) for _ in range(layers)])
    m["wh"] = np.concatenate([q8(4 * P_, P_) for _ in range(layers)])
    m["wxs"], m["whs"] = sc(layers * 4 * P_), sc(layers * 4 * P_)
    m["lb"] = (g.standard_normal(layers * 4 * P_) * 0.1).astype(np.float32)
    m["jpred"], m["jpreds"], m["jpredb"] = q8(J, P_), sc(J), (g.standard_normal(J) * 0.1).astype(np.float32)
    m["jout"], m["jouts"] = q8(nop, J), sc(nop)
    m["joutb"] = (g.standard_normal(nop) * 0.1).astype(np.float32)
    m["joutb"][V] += 7.0
    m["joutb"][V + 1] -= 3.0
    return m


def tdt_device_model(torch, P, m: dict):
    """pkb_tdt_model over device copies of m (PK_Q8 repacked to rows)."""
    keep = []

    def put(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        keep.append(t)
        return t.data_ptr()

    def q8(w_pk, rows, n):
        src = torch.from_numpy(np.ascontiguousarray(w_pk)).cuda()
        out = torch.empty(rows * n, dtype=torch.int8, device="cuda")
        P.repack_q8_dev(out, src, rows, n)
        keep.extend([src, out])
        return out.data_ptr()
    p_, l_, j_ = m["P"], m["L"], m["J"]
    t = P.TdtModel()
    t.P, t.L, t.J, t.V, t.n_dur, t.max_symbols, t.n_out_pad = p_, l_, j_, m["V"], m["n_dur"], m["max_symbols"], \
        m["n_out_pad"]
    for i, d in enumerate(m["dur"]):
        t.dur[i] = int(d)
    t.embed = put(m["embed"])
    for l in range(l_):
        sl, sv = slice(l * 4 * p_ * p_, (l + 1) * 4 * p_ * p_), slice(l * 4 * p_, (l + 1) * 4 * p_)
        t.wx[l], t.wh[l] = q8(m["wx"][sl], 4 * p_, p_), q8(m["wh"][sl], 4 * p_, p_)
        t.wxs[l], t.whs[l], t.lb[l] = put(m["wxs"][sv]), put(m["whs"][sv]), put(m["lb"][sv])
    t.jpred, t.jpreds, t.jpredb = q8(m["jpred"], j_, p_), put(m["jpreds"]), put(m["jpredb"])
    t.jout, t.jouts, t.joutb = q8(m["jout"], m["n_out_pad"], j_), put(m["jouts"]), put(m["joutb"])
    return t, keep


def decoder_search(model, segs) -> dict:
    """TDT's greedy search (core/decoder.c:125-179) over the rank's segments
    in lockstep on the device (pkb_tdt_search_dev): seeded weights at the
    model's shapes, each segment's frames of the joint's encoder half seeded
    (the jenc product's output), one call decoding the whole batch, timed
    with CUDA events; then the shortest segment's tokens against the
    oracle's search."""
    torch, P = model.torch, model.P
    m = tdt_model_synthetic()
    t, keep = tdt_device_model(torch, P, m)
    Ts = np.array([sg[3] for sg in segs], np.uint32)
    f0 = np.concatenate([[0], np.cumsum(Ts)[:-1]]).astype(np.uint32)
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 77)
    f = 2.0 * torch.randn(int(Ts.sum() + 1) * m["J"], device="cuda", generator=g)
    S, cap = len(Ts), int(Ts.max()) * (m["max_symbols"] + 1) + 8
    toks = torch.empty(S * cap * 3, dtype=torch.int32, device="cuda")
    ntok = torch.empty(S, dtype=torch.int32, device="cuda")
    work = torch.empty(P.tdt_work_bytes(t, S) // 4 + 64, device="cuda")
    l0 = P.launch_count()
    P.tdt_search_dev(t, f, f0, Ts, toks, ntok, cap, work)  # warm
    torch.cuda.synchronize()
    launches = P.launch_count() - l0
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record(s)
    for _ in range(reps):
        P.tdt_search_dev(t, f, f0, Ts, toks, ntok, cap, work)
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    n = ntok.cpu().numpy()
    i = int(np.argmin(Ts))
    from oracle import oracle as O
    fh = f.view(-1, m["J"])[int(f0[i]):int(f0[i]) + int(Ts[i])].cpu().numpy().reshape(-1)
    want = O.tdt_search(m, fh, int(Ts[i]))
    got = toks.view(S, cap, 3)[i, :int(n[i])].cpu().numpy()
    rounds = P.tdt_last_rounds()
    return {"ms": ms, "segments": S, "frames": int(Ts.sum()), "tokens": int(n.sum()), "rounds": int(rounds),
            "us_per_round": ms * 1e3 / max(1, rounds), "launches_per_search": int(launches),
            "frames_per_s": float(Ts.sum()) / (ms * 1e-3),
            "shapes": "pred_hidden 640 x 2 LSTM layers, joint 640, jout 8208 x 640, durations 0-4; qb = n",
            "parity": {"segment_frames": int(Ts[i]), "tokens": int(len(want)),
                       "equal": bool(got.shape == want.shape and (got == want).all()),
                       "checker": "the oracle's search (oracle_tdt_search), pinned to the reference's pk_decode"}}


def decoder_batched(model, T: int, segs: int = SEGMENTS, layers: int = 2, P_: int = 640, J: int = 640,
                    vocab_out: int = 8208) -> dict:
    """The TDT decoder's int8 products with the batch's segments stepped in
    lockstep (core/decoder.c:53-79, 149-156: stepped together, its T=1 gemvs
    become products of M = the segment count): one step is, per LSTM layer, quantize + wx (4P x P) and
    quantize + wh (4P x P, added), then quantize + jpred (J x P, bias) and
    quantize + jout (vocab + 1 + durations padded to 16 = 8208 x J, bias),
    every input a whole row a block (core/decoder.c:53-79). Timed as one CUDA
    graph of a step, with CUDA events. Beside it jenc over the batch's frames
    (J x D, qb = D, bias: pk_joint_frames, core/decoder.c:149-156)."""
    torch, P = model.torch, model.P
    s = torch.cuda.current_stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 123)
    S = segs

    def matrix(rows, n):
        w_pk = torch.randint(-127, 128, (rows * n,), dtype=torch.int8, device="cuda", generator=g)
        wp = torch.empty_like(w_pk)
        P.repack_q8_dev(wp, w_pk, rows, n)
        return wp, 1e-3 + 9e-3 * torch.rand(rows, device="cuda", generator=g)

    G = 4 * P_
    mats = [(matrix(G, P_), matrix(G, P_)) for _ in range(layers)]
    jpred, jout = matrix(J, P_), matrix(vocab_out, J)
    jpred_b, jout_b = torch.randn(J, device="cuda", generator=g), torch.randn(vocab_out, device="cuda", generator=g)
    x = torch.randn(S * P_, device="cuda", generator=g)
    h = [torch.randn(S * P_, device="cuda", generator=g) for _ in range(layers)]
    z = torch.randn(S * J, device="cuda", generator=g).clamp_(min=0)
    gates = torch.empty(S * G, device="cuda")
    gp = torch.empty(S * J, device="cuda")
    logit = torch.empty(S * vocab_out, device="cuda")
    q = torch.empty(S * max(P_, J), dtype=torch.int8, device="cuda")
    d = torch.empty(S, device="cuda")

    def prod(out, rows, wm, bias, inp, n, add):
        P.quantize_dev(q, d, inp, n, S, n, n)
        P.gemm_q8_dev(out, rows, wm[0], wm[1], bias, rows, q, d, n, n, S, add)

    def step():
        inp = x
        for l in range(layers):
            prod(gates, G, mats[l][0], None, inp, P_, False)
            prod(gates, G, mats[l][1], None, h[l], P_, True)
            inp = h[l]  # the cell's float update (pk_k_lstm) is off the int8 path
        prod(gp, J, jpred, jpred_b, inp, P_, False)
        prod(logit, vocab_out, jout, jout_b, z, J, False)

    for _ in range(3):
        step()
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    s.synchronize()
    reps = 50
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        graph.replay()
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    ops = 2.0 * S * (layers * 2 * G * P_ + J * P_ + vocab_out * J)
    del graph
    # jenc over the batch's frames
    D_ = D
    xe = torch.randn(T * D_, device="cuda", generator=g)
    qe = torch.empty(T * D_, dtype=torch.int8, device="cuda")
    de = torch.empty(T, device="cuda")
    jenc = matrix(J, D_)
    jenc_b = torch.randn(J, device="cuda", generator=g)
    f = torch.empty(T * J, device="cuda")

    def quant():
        P.quantize_dev(qe, de, xe, D_, T, D_, D_)

    def enc():
        P.gemm_q8_dev(f, J, jenc[0], jenc[1], jenc_b, J, qe, de, D_, D_, T, False)

    def timed(fn) -> float:
        for _ in range(3):
            fn()
        s.synchronize()
        e0.record(s)
        for _ in range(20):
            fn()
        e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) / 20
    qms = timed(quant)
    ems = timed(enc)
    eops = 2.0 * T * J * D_
    return {"segments": S, "step_us": ms * 1e3, "step_tops": ops / (ms * 1e-3) / 1e12,
            "steps_per_s": 1e3 / ms, "launches_per_step": 4 * (2 * layers + 2),
            "shapes": f"per layer wx, wh {G}x{P_}; jpred {J}x{P_}; jout {vocab_out}x{J}; M = {S}, qb = n",
            "jenc_us": ems * 1e3, "jenc_tops": eops / (ems * 1e-3) / 1e12, "jenc_quantize_us": qms * 1e3,
            "jenc_shape": f"M {T} x N {J} x K {D_}, qb {D_}; the product alone, its input's quantization beside it"}


def panels_timing(model, T: int, dk: int = 128) -> dict:
    """The attention's K and V products straight into its panels
    (pk_panels_tile and pk_gemm_panels_on, core/passes.c:119-196) at the
    batch's frame count, against the same
    product into plain rows (D x D, qb 32), each timed with CUDA events."""
    torch, P = model.torch, model.P
    s = torch.cuda.current_stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 321)
    x = torch.randn(T * D, device="cuda", generator=g)
    q = torch.empty(T * D, dtype=torch.int8, device="cuda")
    d = torch.empty(T * D // QB, device="cuda")
    P.quantize_dev(q, d, x, D, T, D, QB)
    w_pk = torch.randint(-127, 128, (D * D,), dtype=torch.int8, device="cuda", generator=g)
    wp = torch.empty_like(w_pk)
    P.repack_q8_dev(wp, w_pk, D, D)
    ws = 1e-3 + 9e-3 * torch.rand(D, device="cuda", generator=g)
    tpad = (T + 15) // 16 * 16
    plain = torch.empty(T * D, device="cuda")
    kp = torch.empty(D * tpad, device="cuda")
    vp = torch.empty(D * T, device="cuda")

    def timed(fn) -> float:
        for _ in range(3):
            fn()
        s.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(20):
            fn()
        e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) / 20

    ops = 2.0 * T * D * D
    t_plain = timed(lambda: P.gemm_q8_dev(plain, D, wp, ws, None, D, q, d, D, QB, T, False))
    t_k = timed(lambda: P.gemm_q8_panels_dev(kp, P.PANELS_KP, 0, dk, tpad, wp, ws, D, q, d, D, QB, T))
    t_v = timed(lambda: P.gemm_q8_panels_dev(vp, P.PANELS_V, 16 * T, 0, 0, wp, ws, D, q, d, D, QB, T))
    return {"shape": f"M {T} x N {D} x K {D}, qb {QB}; K panels dk {dk}, {tpad} frames; V panels ps 16 T",
            "plain_us": t_plain * 1e3, "k_panels_us": t_k * 1e3, "v_panels_us": t_v * 1e3,
            "plain_tops": ops / (t_plain * 1e-3) / 1e12, "k_panels_tops": ops / (t_k * 1e-3) / 1e12,
            "v_panels_tops": ops / (t_v * 1e-3) / 1e12}


def gpu_local_cpus(device: int):
    """The host cores NVML reports as local to this GPU (its NUMA node), or
    None where that cannot be read. Reading only: nothing of the GPU is set."""
    try:
        import torch
        import pynvml
        pr = torch.cuda.get_device_properties(device)
        bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = (os.cpu_count() + 63) // 64
            mask = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * i + b for i, w in enumerate(mask) for b in range(64) if (int(w) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        return cpus or None
    except Exception:  # no NVML, no such attribute: leave the threads where they are
        return None


class near_gpu:
    """Within the block the process's threads run on the GPU's own NUMA
    node, and the page-locked buffers made there sit in its memory: the
    host side of an engine deployed beside its GPU. The affinity is put back
    after."""

    def __init__(self, device: int):
        self.cpus = gpu_local_cpus(device)
        self.was = None

    def __enter__(self):
        if self.cpus and os.environ.get("PKB_BENCH_NO_BIND") != "1":
            self.was = os.sched_getaffinity(0)
            os.sched_setaffinity(0, self.cpus)
        return self

    def __exit__(self, *exc):
        if self.was is not None:
            os.sched_setaffinity(0, self.was)


def e2e_host(prods, steps: int, seed: int, lanes: int) -> dict:
    """The same step through the reference-facing table (pk_kernels_cuda_b200:
    quantize and gemm_q8 on HOST buffers, copies inside each call), called
    as the reference engine calls a backend: whole matrices a call, from
    `lanes` threads at once, each lane its own products' outputs and
    activations (the reference runs independent chunks in lanes the same
    way, core/asr.c:346-572; every call is synchronous, and ctypes releases
    the interpreter while it runs). The activations and results live in
    page-locked host memory, as an engine that pins its buffers once at
    start-up holds them, so each call's copies run by DMA from and into them;
    the weights stay in ordinary memory (uploaded on first use)."""
    import threading
    import torch
    import libpktito_b200 as P
    tab = P.Table()
    rng = np.random.default_rng(seed)
    keep = []  # the page-locked tensors behind the arrays

    def locked(nelem: int, dtype) -> np.ndarray:
        t = torch.empty(nelem, dtype={np.float32: torch.float32, np.int8: torch.int8}[dtype], pin_memory=True)
        keep.append(t)
        return t.numpy()

    w, ws, bias, xs = {}, {}, {}, {}
    for p in prods:
        key, xk = (p["layer"], p["name"]), (p["M"], p["n"])
        if key not in w:
            w[key] = rng.integers(-127, 128, p["rows"] * p["n"], dtype=np.int8)  # PK_Q8 bytes, random
            ws[key] = (1e-3 + 9e-3 * rng.random(p["rows"])).astype(np.float32)
            bias[key] = rng.standard_normal(p["rows"]).astype(np.float32) if p["bias"] else None
        if xk not in xs:
            xs[xk] = locked(p["M"] * p["n"], np.float32)
            xs[xk][:] = rng.standard_normal(p["M"] * p["n"], dtype=np.float32)
    lane_prods = [prods[i::lanes] for i in range(lanes)]
    bufs = []
    for lp in lane_prods:
        qs, ds, outs = {}, {}, {}
        for p in lp:
            xk, ok = (p["M"], p["n"]), (p["M"], p["rows"])
            if xk not in qs:
                qs[xk] = locked(p["M"] * p["n"], np.int8)
                ds[xk] = locked(p["M"] * p["n"] // QB, np.float32)
            if ok not in outs:
                outs[ok] = locked(p["M"] * p["rows"], np.float32)
                outs[ok][:] = 0.0
        bufs.append((qs, ds, outs))
    device = __import__("torch").cuda.current_device()

    def lane(i: int):
        P.set_thread_device(device)
        qs, ds, outs = bufs[i]
        held = {}
        for p in lane_prods[i]:
            key, xk, ok = (p["layer"], p["name"]), (p["M"], p["n"]), (p["M"], p["rows"])
            act = P.PkAct(qs[xk].ctypes.data, ds[xk].ctypes.data, p["n"], QB, p["M"])
            if held.get(xk) != p["inp"]:  # a lane quantizes what it has not got
                tab.quantize(act, xs[xk], p["n"])
                held[xk] = p["inp"]
            tab.gemm_q8(outs[ok], p["rows"], w[key], ws[key], bias[key], p["rows"], act, bool(p["add"]))

    def one():
        ts = [threading.Thread(target=lane, args=(i,)) for i in range(lanes)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    one()  # uploads and caches the weights, grows each lane's staging
    # the bytes the library copied, as it counts them: a quantize takes x in
    # and gives q, d back; a product takes q, d (unless it reads the device
    # copy of the quantize that made them), row scales, biases and the rows
    # it adds to in and gives its results back
    up0, down0 = P.host_bytes()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    sec = (time.perf_counter() - t0) / steps
    up1, down1 = P.host_bytes()
    return {"seconds_per_step": sec, "h2d_bytes_per_step": (up1 - up0) // steps,
            "d2h_bytes_per_step": (down1 - down0) // steps}


def gemm_items(rows: int, T: int, nth: int) -> list[tuple[int, int, int, int]]:
    """(r0, nr, c0, nc) of every call pk_gemm_on makes for a product
    (core/passes.c:90-109): rows in steps of 256 where rows/256 >= 2 threads,
    else 64; the frames in the chunk count (1..8, chunks of at least 48
    frames, whole multiples of 12) that leaves the pool's last round least
    idle."""
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
    return [((i % rb) * step, min(step, rows - (i % rb) * step), (i // rb) * cstep,
             min(cstep, T - (i // rb) * cstep)) for i in range(rb * cc)]


def e2e_host_sliced(prods, steps: int, seed: int, nth: int) -> dict:
    """The same step through the reference-facing table as the reference's
    engine calls a backend: each input quantized in one call, then each
    product in the calls pk_gemm_on makes (slices of 64 or 256 rows of the
    PK_Q8 matrix from inside it, frames in column chunks), dealt to `nth`
    host threads from a shared counter as its pool deals them
    (core/pool.c:115-122); one product after another. Activations and results
    page-locked, weights in ordinary memory, as e2e_host."""
    import threading
    import torch
    import libpktito_b200 as P
    tab = P.Table()
    rng = np.random.default_rng(seed)
    keep = []

    def locked(nelem: int, dtype) -> np.ndarray:
        t = torch.empty(nelem, dtype={np.float32: torch.float32, np.int8: torch.int8}[dtype], pin_memory=True)
        keep.append(t)
        return t.numpy()

    w, ws, bias, xs, qs, ds, outs = {}, {}, {}, {}, {}, {}, {}
    for p in prods:
        key, xk, ok = (p["layer"], p["name"]), (p["M"], p["n"]), (p["M"], p["rows"])
        if key not in w:
            w[key] = rng.integers(-127, 128, p["rows"] * p["n"], dtype=np.int8)
            ws[key] = (1e-3 + 9e-3 * rng.random(p["rows"])).astype(np.float32)
            bias[key] = rng.standard_normal(p["rows"]).astype(np.float32) if p["bias"] else None
        if xk not in xs:
            xs[xk] = locked(p["M"] * p["n"], np.float32)
            xs[xk][:] = rng.standard_normal(p["M"] * p["n"], dtype=np.float32)
            qs[xk] = locked(p["M"] * p["n"], np.int8)
            ds[xk] = locked(p["M"] * p["n"] // QB, np.float32)
        if ok not in outs:
            outs[ok] = locked(p["M"] * p["rows"], np.float32)
            outs[ok][:] = 0.0
    device = torch.cuda.current_device()
    work = {"items": [], "next": 0, "p": None}
    lock = threading.Lock()
    start, done = threading.Barrier(nth + 1), threading.Barrier(nth + 1)
    calls = [0]

    def worker():
        P.set_thread_device(device)
        while True:
            start.wait()
            p = work["p"]
            if p is None:
                return
            key, xk, ok = (p["layer"], p["name"]), (p["M"], p["n"]), (p["M"], p["rows"])
            n, nb = p["n"], p["n"] // QB
            while True:
                with lock:
                    i = work["next"]
                    work["next"] += 1
                if i >= len(work["items"]):
                    break
                r0, nr, c0, nc = work["items"][i]
                act = P.PkAct(qs[xk][c0 * n:].ctypes.data, ds[xk][c0 * nb:].ctypes.data, n, QB, nc)
                b = bias[key]
                tab.gemm_q8(outs[ok][c0 * p["rows"] + r0:], p["rows"], w[key][r0 * n:], ws[key][r0:],
                            None if b is None else b[r0:], nr, act, bool(p["add"]))
            done.wait()

    ts = [threading.Thread(target=worker, daemon=True) for _ in range(nth)]
    for t in ts:
        t.start()

    def one():
        held = {}
        for p in prods:
            xk = (p["M"], p["n"])
            if held.get(xk) != p["inp"]:
                tab.quantize(P.PkAct(qs[xk].ctypes.data, ds[xk].ctypes.data, p["n"], QB, p["M"]), xs[xk], p["n"])
                held[xk] = p["inp"]
            work["items"] = gemm_items(p["rows"], p["M"], nth)
            work["next"] = 0
            work["p"] = p
            calls[0] += len(work["items"])
            start.wait()
            done.wait()

    one()  # uploads and caches the weights
    calls[0] = 0
    up0, down0 = P.host_bytes()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    sec = (time.perf_counter() - t0) / steps
    up1, down1 = P.host_bytes()
    work["p"] = None
    start.wait()
    for t in ts:
        t.join()
    return {"seconds_per_step": sec, "calls_per_step": calls[0] // max(1, steps), "threads": nth,
            "h2d_bytes_per_step": (up1 - up0) // steps, "d2h_bytes_per_step": (down1 - down0) // steps}


# -------------------------------------------------------------- the arms --

def dist_setup(gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist
    return rank, world, local, pg


def job_totals(dist, dev, ms: float, ops: float, audio_s: float) -> tuple[float, float, float]:
    """The whole job's figures from every rank's own: the time is the max
    over ranks, the work (int8 ops, audio seconds) the sum, since each rank
    draws its own segments. One process per rank; `dist` is None alone."""
    if not dist:
        return ms, ops, audio_s
    import torch
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    w = torch.tensor([ops, audio_s], dtype=torch.float64, device=dev)
    dist.all_reduce(w, op=dist.ReduceOp.SUM)
    return float(t.item()), float(w[0].item()), float(w[1].item())


def run_ours(args) -> None:
    import torch
    rank, world, local, dist = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    import libpktito_b200 as P
    P.set_thread_device(local)
    dev = torch.device("cuda", local)
    segs = segments(rank, world, args.scaling)
    prods = products(segs)
    ops = step_ops(prods, segs)
    model = Model(prods, dev, SEED + 1000, segs)  # one model, replicated on every GPU

    def barrier():
        if dist:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        model.step()
    l0 = P.launch_count()
    model.step()
    launches_per_step = P.launch_count() - l0
    graph = None
    if not args.no_graph:
        # the step captured once and replayed: no host work between launches
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            model.step()
        graph.replay()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    e0.record(stream)
    for _ in range(args.steps):
        if graph:
            graph.replay()
        else:
            model.step()
    e1.record(stream)
    barrier()
    wall = time.perf_counter() - t_wall
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    if P.device_errors(local):
        raise RuntimeError("a kernel reported a timeout during the timed steps")
    ms, ops_job, audio_job = job_totals(dist, dev, ms, ops, audio_seconds(segs))
    used_graph = graph is not None
    parity = parity_check(model, graph, world)
    if dist:  # every rank checked its own share; the job's counts are the sums
        c = torch.tensor([parity["checked"], parity["equal"]], dtype=torch.float64, device=dev)
        dist.all_reduce(c, op=dist.ReduceOp.SUM)
        parity["checked"], parity["equal"] = int(c[0].item()), int(c[1].item())
        parity["ranks"] = world
    del graph  # released before the process group goes (it holds no collective, but keep the order safe)
    roof = kernel_roofline(model, prods, clk.get("sm_mhz")) if rank == 0 else None
    if roof is not None and not args.no_producers:
        roof["producers"] = producers_roofline(model, sum(sg[3] for sg in segs))
        roof["decoder_batched"] = decoder_batched(model, sum(sg[3] for sg in segs))
        roof["panels"] = panels_timing(model, sum(sg[3] for sg in segs))
        roof["attention"] = attention_timing(model, segs, clk.get("sm_mhz"))
        roof["decoder_search"] = decoder_search(model, segs)
        try:
            roof["encoder_layer"] = encoder_layer_timing(model, segs)
        except Exception as e:  # a measurement beside the headline: its failure is reported, not fatal
            roof["encoder_layer"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    e2e = None
    if not args.no_e2e:
        # every rank at once through the host table, each on its own
        # segments; the job's time is the slowest rank's
        if dist:
            dist.barrier(device_ids=[local])
        e2e_steps = args.e2e_steps or (args.steps if WORKLOAD == "batched" else min(args.steps, 3))
        with near_gpu(local) as near:
            e = e2e_host(prods, e2e_steps, SEED + 7 + rank, args.e2e_lanes)
        sec, e_ops, e_audio = job_totals(dist, dev, e["seconds_per_step"], step_ops(prods), audio_seconds(segs))
        h2d, d2h = job_totals(dist, dev, 0.0, e["h2d_bytes_per_step"], e["d2h_bytes_per_step"])[1:]
        e2e = {"value": e_ops / sec / 1e12, "unit": "TOPS",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "audio_s_per_s": e_audio / sec,
               "path": "pk_kernels_cuda_b200 table (quantize + gemm_q8 on host buffers: activations and results "
                       "page-locked, weights in ordinary memory), whole matrices a call, "
                       f"{args.e2e_lanes} lanes of calls at once on each rank; the encoder's products; "
                       "bytes as the library counts its copies (pkb_host_bytes): a product whose q and d "
                       "are a quantize result still held on the device does not upload them",
               "steps": e2e_steps,
               "lanes": args.e2e_lanes,
               "host_cpus": len(near.cpus) if near.was is not None else None}
    if e2e is not None and not args.no_sliced and world == 1:
        # the engine's call pattern (slices from a pool of host threads); one
        # GPU only, as the pool's threads of several ranks would share the
        # host's cores
        with near_gpu(local):
            sl = e2e_host_sliced(prods, max(1, min(args.steps, 3)), SEED + 11 + rank, args.e2e_threads)
        sec, e_ops, _ = job_totals(dist, dev, sl["seconds_per_step"], step_ops(prods), audio_seconds(segs))
        e2e["engine_sliced"] = {"value": e_ops / sec / 1e12, "unit": "TOPS", "calls_per_step": sl["calls_per_step"],
                                "h2d_bytes_per_step": int(sl["h2d_bytes_per_step"]),
                                "d2h_bytes_per_step": int(sl["d2h_bytes_per_step"]),
                                "threads": sl["threads"], "steps": max(1, min(args.steps, 3)),
                                "path": "pk_kernels_cuda_b200 table as the reference's engine calls it: each input "
                                        "quantized in one call, each product in pk_gemm_on's slices of 64/256 rows "
                                        "and column chunks (core/passes.c:90-109), dealt to a pool of host threads"}
    cpu = cpu_baseline(prods) if (rank == 0 and world == 1 and not args.no_cpu) else None
    if dist:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    ms_step = ms / args.steps
    value = ops_job / (ms_step * 1e-3) / 1e12
    t3 = sum(s[3] for s in segs)
    nseg = SEGMENTS if args.scaling == "strong" else SEGMENTS * world
    if WORKLOAD == "longform":
        nseg = len(longform_chunks())
        workload = ("configs[4] long-form: one hour of synthetic audio cut at its pauses by the reference's "
                    f"segmenter and chunker into {nseg} chunks of up to 30.72 s, dealt across the GPUs longest "
                    "first; per chunk the 24-layer encoder's 11 products a layer + 3 subsampling products, then "
                    f"the TDT joint: jenc over every frame (qb 1024) and jout ({VOCAB_OUT} x {J}, qb 640) at each "
                    f"lockstep decode step over the rank's chunks; qb {QB} in the encoder")
    else:
        workload = (("configs[3] batched encoder: one batch of 64 segments of 2-30 s dealt across the "
                     "GPUs longest first" if args.scaling == "strong" else
                     "configs[3] batched encoder, weak scaling: the batch of 64 segments of 2-30 s on every GPU") +
                    ", 24 layers x 11 products + 3 subsampling products, 196 quantizations (q, k, v share "
                    f"one input; the position input is quantized once), qb {QB}")
    line = {
        "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if WORKLOAD == "longform" else args.scaling,
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded segments, random int8 weights, N(0,1) activations)",
        "config": {"workload": workload,
                   "segments_rank0": len(segs), "encoder_frames_rank0": t3, "layers": LAYERS, "d_model": D,
                   "ff_dim": F, "qb": QB, "global_batch": nseg, "seq_len": t3 // max(1, len(segs)),
                   "parallelism": f"dp{world}", "l2": "no flush: each step streams 576 MiB of weights and "
                                                       "~1.4 GB of activations, well over the 126 MB L2",
                   "cuda_graph": used_graph},
        "audio_s_per_s": audio_job / (ms_step * 1e-3),
        "ops_per_step": ops_job, "wall_s": wall,
        "e2e": e2e, "gpu_launches": launches_per_step * args.steps, "clocks": clk,
        "roofline": roof, "cpu_baseline": cpu, "parity": parity,
    }
    print(json.dumps(line))
    if parity["equal"] != parity["checked"]:
        print(f"parity: {parity['checked'] - parity['equal']} of {parity['checked']} checks differ from the "
              f"reference: {parity['mismatches']}", file=sys.stderr)
        sys.exit(3)


def reference_step(prods, seed: int, threads: int):
    """The step on the reference's own CPU int8 path: the backend its picker
    chooses on this host (backend/kernels.c:277-305; amx-int8 on an AMX
    Xeon), built from its sources into oracle/_ref, driven over `threads`
    threads as its passes deal work (quantize in items of 16 columns,
    core/passes.c:39-46; products in slices of 64 rows, core/passes.c:60-109).
    Every product of the step, each input quantized once as the GPU arm does,
    on seeded random weights and N(0,1) inputs of the same shapes. Returns
    (step function, backend name) or (None, why)."""
    import ctypes
    so = os.path.join(ROOT, "oracle", "_ref", "libcpubench.so")
    if not os.path.exists(so):
        return None, "oracle/_ref/libcpubench.so (the reference's backends, built from its sources) is not built"
    lib = ctypes.CDLL(so)
    vp, u32, sz = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_size_t
    lib.cpub_backend.restype = ctypes.c_char_p
    lib.cpub_backend.argtypes = [ctypes.c_char_p, sz]
    lib.cpub_quantize.restype = None
    lib.cpub_quantize.argtypes = [vp, vp, vp, sz, u32, u32, u32, ctypes.c_int]
    lib.cpub_gemm.restype = None
    lib.cpub_gemm.argtypes = [vp, sz, vp, vp, vp, u32, vp, vp, u32, u32, u32, ctypes.c_int, ctypes.c_int]
    backend = lib.cpub_backend(None, 0).decode()
    rng = np.random.default_rng(seed)
    w, ws, bias, x, q, d, out = {}, {}, {}, {}, {}, {}, {}
    for p in prods:
        key, xk, ok = (p["layer"], p["name"]), (p["M"], p["n"]), (p["M"], p["rows"])
        if key not in w:
            w[key] = rng.integers(-127, 128, p["rows"] * p["n"], dtype=np.int8)
            ws[key] = (1e-3 + 9e-3 * rng.random(p["rows"])).astype(np.float32)
            bias[key] = rng.standard_normal(p["rows"], dtype=np.float32) if p["bias"] else None
        if xk not in x:
            x[xk] = rng.standard_normal(p["M"] * p["n"], dtype=np.float32)
            q[xk] = np.empty(p["M"] * p["n"], np.int8)
            d[xk] = np.empty(p["M"] * p["n"] // QB, np.float32)
        if ok not in out:
            out[ok] = np.zeros(p["M"] * p["rows"], np.float32)
    ptr = lambda a: 0 if a is None else a.ctypes.data

    def step():
        held = {}
        for p in prods:
            key, xk, ok = (p["layer"], p["name"]), (p["M"], p["n"]), (p["M"], p["rows"])
            if held.get(xk) != p["inp"]:
                lib.cpub_quantize(ptr(q[xk]), ptr(d[xk]), ptr(x[xk]), p["n"], p["n"], QB, p["M"], threads)
                held[xk] = p["inp"]
            lib.cpub_gemm(ptr(out[ok]), p["rows"], ptr(w[key]), ptr(ws[key]), ptr(bias[key]), p["rows"], ptr(q[xk]),
                          ptr(d[xk]), p["n"], QB, p["M"], p["add"], threads)

    return step, backend


def run_reference(args) -> None:
    """The reference arm: one GPU's workload (the whole batch of 64 segments,
    what rank 0 takes at every N under weak scaling and at N = 1 under
    strong) through the reference's own CPU int8 path on all host cores,
    every one of the step's products each step. Under torchrun only rank 0
    runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    segs = segments(0)
    prods = products(segs)
    ops = step_ops(prods)
    cores = os.cpu_count() or 1
    step, backend = reference_step(prods, SEED + 77, cores)
    if step is None:
        print(json.dumps({"impl": "reference", "unavailable": backend}))
        return
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    step_s = float(sum(times)) / len(times)
    value = ops / step_s / 1e12
    cpu = {"value": value, "unit": "TOPS", "cores": cores, "kind": "reference", "backend": backend,
           "sample": f"the whole step ({len(prods)} products and their quantizations at the batch's M) every step, "
                     f"{args.steps} timed steps after {args.warmup} warm-up steps; median step "
                     f"{float(np.median(times)):.3f} s"}
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "strong" if WORKLOAD == "longform" else args.scaling, "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded segments, random int8 weights, N(0,1) activations)",
            "config": {"workload": "configs[3] batched encoder (the GPU arm's whole batch): 64 segments of 2-30 s, "
                                   "24 layers x 11 products + 3 subsampling products, every product timed every "
                                   f"step, qb {QB}", "segments": SEGMENTS, "layers": LAYERS, "qb": QB,
                       "encoder_frames": sum(sg[3] for sg in segs)},
            "audio_s_per_s": audio_seconds(segs) / step_s,
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_kernel_only() -> None:
    """The dominant product alone: quantize once, then three launches of the
    product kernel on the FF-up shape at the batch's M (11521 x 4096 x 1024,
    qb 32; 12 MB of activations, 4 MB of weights, 189 MB of output, which
    is more than the 126 MB L2)."""
    import torch
    import libpktito_b200 as P
    segs = segments(0)
    p = next(x for x in products(segs) if x["name"] == "ff1_up")
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(SEED)
    M, rows, n = p["M"], p["rows"], p["n"]
    x = torch.randn(M * n, device=dev, generator=g)
    q = torch.empty(M * n, dtype=torch.int8, device=dev)
    d = torch.empty(M * n // QB, device=dev)
    w_pk = torch.randint(-127, 128, (rows * n,), dtype=torch.int8, device=dev, generator=g)
    wpack = torch.empty_like(w_pk)
    ws = 1e-3 + 9e-3 * torch.rand(rows, device=dev, generator=g)
    out = torch.zeros(M * rows, device=dev)
    P.quantize_dev(q, d, x, n, M, n, QB)
    P.repack_q8_dev(wpack, w_pk, rows, n)
    for _ in range(3):
        P.gemm_q8_dev(out, rows, wpack, ws, None, rows, q, d, n, QB, M, False)
    torch.cuda.synchronize()
    print(json.dumps({"kernel_only": f"M {M} x N {rows} x K {n} qb {QB}", "launches": P.launch_count(),
                      "device_errors": P.device_errors(0)}))


def run_producers_only() -> None:
    """The three fused producers at the batch's frame count, two launches
    each in the order LayerNorm, SiLU, GLU + dwconv (the ncu capture's case:
    inputs 47, 189 and 94 MB)."""
    import torch
    import libpktito_b200 as P
    T = sum(s[3] for s in segments(0))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(SEED)
    q = torch.empty(T * F, dtype=torch.int8, device=dev)
    d = torch.empty(T * F // QB, device=dev)
    x = torch.randn(T * D, device=dev, generator=g)
    w, b = torch.randn(D, device=dev, generator=g), torch.randn(D, device=dev, generator=g)
    u = torch.randn(T * F, device=dev, generator=g) * 4
    xg = torch.randn(T * 2 * D, device=dev, generator=g)
    wd, bd = torch.randn(D * 9, device=dev, generator=g) * 0.3, torch.randn(D, device=dev, generator=g)
    for _ in range(2):
        P.layernorm_quantize_dev(q, d, x, D, T, D, QB, w, b, 1e-5)
        P.silu_quantize_dev(q, d, u, F, T, F, QB)
        P.dwconv_quantize_dev(q, d, None, D, xg, 2 * D, T, D, wd, bd, 9, True, QB)
    torch.cuda.synchronize()
    print(json.dumps({"producers_only": f"T {T}: layernorm n {D}, silu n {F}, glu+dwconv C {D} K 9, qb {QB}",
                      "launches": P.launch_count(), "device_errors": P.device_errors(0)}))


def run_panels_only() -> None:
    """The attention's K and V products at the batch's frame count (M 11521
    x N 1024 x K 1024, qb 32; dk 128): one launch each into plain rows, K
    panels and V panels, in that order (the ncu capture's case: 12 MB of
    activations in, 47 MB of results out each)."""
    import torch
    import libpktito_b200 as P
    T = sum(s[3] for s in segments(0))
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(SEED)
    x = torch.randn(T * D, device=dev, generator=g)
    q = torch.empty(T * D, dtype=torch.int8, device=dev)
    d = torch.empty(T * D // QB, device=dev)
    w_pk = torch.randint(-127, 128, (D * D,), dtype=torch.int8, device=dev, generator=g)
    wp = torch.empty_like(w_pk)
    ws = 1e-3 + 9e-3 * torch.rand(D, device=dev, generator=g)
    tpad = (T + 15) // 16 * 16
    plain, kp, vp = (torch.empty(T * D, device=dev), torch.empty(D * tpad, device=dev),
                     torch.empty(D * T, device=dev))
    P.quantize_dev(q, d, x, D, T, D, QB)
    P.repack_q8_dev(wp, w_pk, D, D)
    P.gemm_q8_dev(plain, D, wp, ws, None, D, q, d, D, QB, T, False)
    P.gemm_q8_panels_dev(kp, P.PANELS_KP, 0, 128, tpad, wp, ws, D, q, d, D, QB, T)
    P.gemm_q8_panels_dev(vp, P.PANELS_V, 16 * T, 0, 0, wp, ws, D, q, d, D, QB, T)
    torch.cuda.synchronize()
    print(json.dumps({"panels_only": f"M {T} x N {D} x K {D} qb {QB}: rows, K panels (dk 128), V panels",
                      "launches": P.launch_count(), "device_errors": P.device_errors(0)}))


def run_attention_only() -> None:
    """One layer's attention over the batch's 64 segments (the ncu capture's
    case: 190 MB of q, K, V and P rows in, 47 MB of o out), one launch."""
    import torch
    import libpktito_b200 as P
    torch.cuda.set_device(0)
    Ts = [s[3] for s in segments(0)]
    q, k, v, p, bu, bv, sl = attention_inputs(torch, Ts, SEED + 123)
    o = torch.empty(sum(Ts) * D, device="cuda")
    P.attention_rows_dev(o, D, q, D, k, D, v, D, p, D, bu, bv, D, HEADS, sl)
    torch.cuda.synchronize()
    print(json.dumps({"attention_only": f"{len(Ts)} segments, {sum(Ts)} frames, D {D}, {HEADS} heads",
                      "launches": P.launch_count(), "device_errors": P.device_errors(0)}))


def run_decoder_only() -> None:
    """TDT's search over the batch's 64 segments on the device, once (the ncu
    capture's case: the search as one cooperative launch, after the
    embedding's quantization and the states' set-up)."""
    import torch
    import libpktito_b200 as P
    torch.cuda.set_device(0)
    segs = segments(0)
    m = tdt_model_synthetic()
    t, keep = tdt_device_model(torch, P, m)
    Ts = np.array([sg[3] for sg in segs], np.uint32)
    f0 = np.concatenate([[0], np.cumsum(Ts)[:-1]]).astype(np.uint32)
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 77)
    f = 2.0 * torch.randn(int(Ts.sum() + 1) * m["J"], device="cuda", generator=g)
    S, cap = len(Ts), int(Ts.max()) * (m["max_symbols"] + 1) + 8
    toks = torch.empty(S * cap * 3, dtype=torch.int32, device="cuda")
    ntok = torch.empty(S, dtype=torch.int32, device="cuda")
    work = torch.empty(P.tdt_work_bytes(t, S) // 4 + 64, device="cuda")
    P.tdt_search_dev(t, f, f0, Ts, toks, ntok, cap, work)
    torch.cuda.synchronize()
    print(json.dumps({"decoder_only": f"{S} segments, {int(Ts.sum())} frames", "rounds": P.tdt_last_rounds(),
                      "tokens": int(ntok.sum().item()), "launches": P.launch_count(),
                      "device_errors": P.device_errors(0)}))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["batched", "longform"], default="batched",
                    help="batched: configs[3] (64 segments of 2-30 s); longform: configs[4] (an hour cut by the "
                         "reference's segmenter, the TDT joint included)")
    ap.add_argument("--qb", type=int, choices=[32, 64], default=32,
                    help="blocks of the activations' quantization: 32, or 64 in the reference's fast mode")
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the e2e leg (default: --steps)")
    ap.add_argument("--e2e-lanes", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sliced", action="store_true", help="skip the e2e figure at the engine's slicing")
    ap.add_argument("--e2e-threads", type=int, default=16, help="host threads of the engine-sliced e2e figure")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-producers", action="store_true", help="skip timing the fused producers (rank 0)")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="weak",
                    help="weak: configs[3]'s batch of 64 segments on every GPU; "
                         "strong: the one batch of 64 segments split across the GPUs")
    ap.add_argument("--kernel-only", action="store_true",
                    help="only the dominant product (FF up at the batch's M), 3 launches: the ncu capture's case")
    ap.add_argument("--producers-only", action="store_true",
                    help="only the fused producers at the batch's frame count, 2 launches each: the ncu capture's case")
    ap.add_argument("--decoder-only", action="store_true",
                    help="TDT's search over the batch once and exit (for an ncu capture of the search)")
    ap.add_argument("--attention-only", action="store_true",
                    help="only one layer's attention over the batch, 1 launch: the ncu capture's case")
    ap.add_argument("--panels-only", action="store_true",
                    help="only the K/V products into plain rows, K panels and V panels, 1 launch each: the ncu "
                         "capture's case")
    args = ap.parse_args()
    global QB, WORKLOAD
    QB = args.qb
    WORKLOAD = args.workload
    if args.kernel_only:
        run_kernel_only()
    elif args.panels_only:
        run_panels_only()
    elif args.producers_only:
        run_producers_only()
    elif args.attention_only:
        run_attention_only()
    elif args.decoder_only:
        run_decoder_only()
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
