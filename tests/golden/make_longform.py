"""Writes tests/golden/longform_chunks.json: the chunks of the long-form
workload, cut by the reference's own code.

TEST INFRASTRUCTURE (a fixture generator): it runs the reference's segmenter
and chunker, compiled from its sources into oracle/_ref/libpkcore.so by
oracle/Makefile, and writes only their output.

The recording: one hour at 16 kHz of white noise N(0, 0.1) with silences
(exact zeros) of lengths uniform in 0.3-2 s every 5-25 s of sound, seeded.
Silero's weights are not in the reference's tree, so its probabilities are
made from the layout: one per 512-sample window (Silero's at 16 kHz), 1
where the window is mostly sound, 0 where it is mostly silence. The
reference then cuts it as its low-level path does for chunks without
context: pk_segments (core/segment.c:175) with Silero's defaults and
max_speech_s = 30.72 - 2 * 0.03 - 0.1 (core/transcribe.c:1045, context
off), and pk_chunks (core/asr.c:1064-1066) with chunks of at most 30.72 s
(core/transcribe.c:177).

    python tests/golden/make_longform.py
"""
import ctypes
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
CORE = os.path.join(ROOT, "oracle", "_ref", "libpkcore.so")
OUT = os.path.join(HERE, "longform_chunks.json")

SEED = 20261205
RATE = 16000
SECONDS = 3600
WINDOW = 512
MAX_CHUNK_S = 30.72


class SegParams(ctypes.Structure):
    """pk_seg_params (core/pktito.h:479-488)"""
    _fields_ = [("threshold", ctypes.c_double), ("neg_threshold", ctypes.c_double),
                ("min_speech_ms", ctypes.c_double), ("max_speech_s", ctypes.c_double),
                ("min_silence_ms", ctypes.c_double), ("speech_pad_ms", ctypes.c_double),
                ("min_silence_at_max_speech_ms", ctypes.c_double), ("use_max_poss_sil_at_max_speech", ctypes.c_int)]


class Seg(ctypes.Structure):
    """pk_seg (core/pktito.h:272)"""
    _fields_ = [("start", ctypes.c_int64), ("end", ctypes.c_int64)]


READ = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_float), ctypes.c_size_t)


class Audio(ctypes.Structure):
    """pk_audio (core/pktito.h:149-154)"""
    _fields_ = [("n", ctypes.c_int64), ("read", READ), ("arg", ctypes.c_void_p), ("wait", ctypes.c_void_p)]


def recording(seed: int = SEED):
    """(samples, runs): the hour of noise and silences, and its (start, end, sound) runs"""
    rng = np.random.default_rng(seed)
    n = SECONDS * RATE
    runs, t = [], 0
    while t < n:
        s = min(n, t + int(rng.uniform(5.0, 25.0) * RATE))
        runs.append((t, s, 1))
        t = s
        if t >= n:
            break
        s = min(n, t + int(rng.uniform(0.3, 2.0) * RATE))
        runs.append((t, s, 0))
        t = s
    x = np.zeros(n, np.float32)
    for a, b, sound in runs:
        if sound:
            x[a:b] = rng.normal(0.0, 0.1, b - a).astype(np.float32)
    return x, runs


def probabilities(runs, n: int) -> np.ndarray:
    """one a 512-sample window: the share of its samples that are sound, rounded to 0 or 1"""
    sound = np.zeros(n, np.float32)
    for a, b, s in runs:
        if s:
            sound[a:b] = 1.0
    w = n // WINDOW
    return (sound[:w * WINDOW].reshape(w, WINDOW).mean(axis=1) >= 0.5).astype(np.float32)


def cut(x: np.ndarray, probs: np.ndarray):
    lib = ctypes.CDLL(CORE)
    lib.pk_seg_defaults.argtypes = [ctypes.POINTER(SegParams)]
    lib.pk_segments.restype = ctypes.c_size_t
    lib.pk_segments.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int64,
                                ctypes.POINTER(SegParams), ctypes.POINTER(Seg), ctypes.c_size_t]
    lib.pk_chunks.restype = ctypes.c_long
    lib.pk_chunks.argtypes = [ctypes.POINTER(Audio), ctypes.POINTER(Seg), ctypes.c_size_t, ctypes.c_int64,
                              ctypes.POINTER(Seg)]
    p = SegParams()
    lib.pk_seg_defaults(ctypes.byref(p))
    p.max_speech_s = MAX_CHUNK_S - 2 * p.speech_pad_ms / 1000 - 0.1
    cap = 2 * probs.size + 1
    segs = (Seg * cap)()
    nseg = lib.pk_segments(probs.ctypes.data, probs.size, RATE, x.size, ctypes.byref(p), segs, cap)

    def read(arg, at, out, count):
        ctypes.memmove(out, x[at:at + count].ctypes.data, 4 * count)
        return 0

    rd = READ(read)
    audio = Audio(x.size, rd, None, None)
    chunks = (Seg * (4 * nseg + 16))()
    nch = lib.pk_chunks(ctypes.byref(audio), segs, nseg, int(MAX_CHUNK_S * RATE), chunks)
    assert nch > 0
    return [(s.start, s.end) for s in segs[:nseg]], [(c.start, c.end) for c in chunks[:nch]]


def main() -> None:
    x, runs = recording()
    probs = probabilities(runs, x.size)
    segs, chunks = cut(x, probs)
    doc = {"workload": "BASELINE.json configs[4]: one hour of N(0, 0.1) noise at 16 kHz with silences of "
                       "0.3-2 s every 5-25 s, cut by the reference's pk_segments and pk_chunks",
           "seed": SEED, "rate": RATE, "seconds": SECONDS, "window": WINDOW, "max_chunk_s": MAX_CHUNK_S,
           "sound_runs": sum(1 for r in runs if r[2]), "segments": len(segs),
           "chunks": [[int(a), int(b)] for a, b in chunks]}
    with open(OUT, "w") as f:
        json.dump(doc, f, indent=0)
    sec = sum(b - a for a, b in chunks) / RATE
    print(f"{len(segs)} segments, {len(chunks)} chunks, {sec:.1f} s of audio in chunks -> {OUT}")


if __name__ == "__main__":
    main()
