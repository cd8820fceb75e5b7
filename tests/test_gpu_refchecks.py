"""The reference's own checks, compiled from its sources unmodified
(oracle/Makefile), run against the cuda-b200 table: tests/q8check.c walks
every backend before ref in pk_kernels_built and holds its gemm_q8 to ref's
bits at guard pages, in four rounding modes (385 cases); tests/kcheck.c does
the same for all thirteen kernels on random data, and on a real model's
matrices given tiny.pkf."""
import os
import subprocess

import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

Q8CHECK = os.path.join(O.REF_DIR, "q8check_cuda")
KCHECK = os.path.join(O.REF_DIR, "kcheck_cuda")
TINY = os.path.join(O.REF_DIR, "tiny.pkf")


def run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    return r.returncode, r.stdout + r.stderr


@pytest.mark.skipif(not os.path.exists(Q8CHECK), reason="reference checks not built here (make -C oracle ref)")
def test_reference_q8check(cuda_device):
    rc, out = run([Q8CHECK])
    assert "cuda-b200" in out and "every one ref's bits" in out, out
    assert rc == 0, out


@pytest.mark.skipif(not os.path.exists(KCHECK), reason="reference checks not built here (make -C oracle ref)")
def test_reference_kcheck(cuda_device):
    rc, out = run([KCHECK])
    lines = [l for l in out.splitlines() if l.startswith("kcheck:")]
    assert any("cuda-b200" in l and "every one ref's bits" in l for l in lines), out
    assert rc == 0, out


@pytest.mark.skipif(not (os.path.exists(KCHECK) and os.path.exists(TINY)), reason="reference checks not built here")
def test_reference_kcheck_tiny_model(cuda_device):
    """With the tiny model, every backend (ref included) prints one known line
    from kcheck's own tiny-block case: its planted maximum can be overwritten
    by the zeros it plants after it (tests/kcheck.c:158-160), so d = 0 is
    right and the check's expectation (tests/kcheck.c:170) is not. Every
    other case must hold ref's bits."""
    rc, out = run([KCHECK, TINY])
    fails = [l for l in out.splitlines() if l.startswith("FAIL")]
    assert all(l.startswith("FAIL tiny quantize: block of") for l in fails), out
    assert not any("gemm_q8" in l or "quantize T" in l or "quantize non-finite" in l for l in fails), out
