"""The drop-in, proved inside the reference's own engine.

oracle/_ref/pktito-c_cuda is the reference's CLI and engine (core/cli.c and
every core/*.c), compiled unmodified from its sources, whose backend list is
cuda-b200-f32, cuda-b200, then ref (oracle/Makefile). It transcribes the
reference's test recording with its tiny model on each backend
(PKTITO_KERNELS), at one and at eight pool threads and in fast mode, and the
transcripts must be the same bytes: every int8 product and quantization of
the encoder and decoder then went through the GPU with the reference's call
pattern (slices of 64/256 rows and column chunks from every pool thread at
once, fused tile callbacks, chunks in lanes) and changed no bit of the
result; with cuda-b200-f32 every float product (the attention's scores,
positions and weighted values, a head and block of 16 queries a call, and
the decoder's) and every softmax row did too.
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")
CLI = os.path.join(REF, "pktito-c_cuda")


def transcribe(backend: str, threads: int, fast: bool) -> bytes:
    args = [CLI, "-t", str(threads), "--json", "-m", "tiny.pkf", "test.wav"] + (["--fast"] if fast else [])
    r = subprocess.run(args, cwd=REF, capture_output=True, env=dict(os.environ, PKTITO_KERNELS=backend),
                       timeout=600)
    assert r.returncode == 0, r.stderr.decode(errors="replace")[-2000:]
    return r.stdout


@pytest.mark.skipif(not os.path.exists(CLI), reason="the reference's engine is not built (make -C oracle ref)")
@pytest.mark.parametrize("threads,fast", [(1, False), (8, False), (8, True)])
def test_reference_engine_transcribes_the_same_bytes_on_cuda_b200(cuda_device, threads, fast):
    want = transcribe("ref", threads, fast)
    got = transcribe("cuda-b200", threads, fast)
    assert b'"segments"' in want
    assert got == want


@pytest.mark.skipif(not os.path.exists(CLI), reason="the reference's engine is not built (make -C oracle ref)")
@pytest.mark.parametrize("threads", [1, 8])
def test_reference_engine_with_the_float_kernels_on_the_gpu(cuda_device, threads):
    assert transcribe("cuda-b200-f32", threads, False) == transcribe("ref", threads, False)
