"""The boundary without a GPU: the library loads, exports every symbol
include/*.h declares, exports the backend table with the reference's layout,
and refuses bad arguments before touching a device."""
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in ("pktito_b200.h",):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"\b(pkb_\w+)\s*\(", src)
    return sorted(set(names))


def test_every_declared_symbol_is_exported(pkb):
    lib = pkb.lib()
    decl = declared_functions()
    assert len(decl) >= 12
    for name in decl:
        assert hasattr(lib, name), name
    assert set(decl) == set(pkb.exported_symbols())


def test_table_symbol_and_id(pkb):
    tab = pkb.Table()
    assert tab.id == "cuda-b200"
    assert tab.k.quantize and tab.k.gemm_q8


def test_dynamic_symbols_with_nm(pkb):
    out = subprocess.run(["nm", "-D", "--defined-only", pkb.LIB_PATH], capture_output=True, text=True).stdout
    for name in declared_functions() + ["pk_kernels_cuda_b200", "pk_kernels_cuda_b200_f32"]:
        assert re.search(r"\b%s\b" % name, out), name


def test_table_layout_matches_reference():
    ref = os.path.join(ROOT, "oracle", "_ref", "abi_ref")
    mine = os.path.join(ROOT, "oracle", "_ref", "abi_mine")
    if not (os.path.exists(ref) and os.path.exists(mine)):
        pytest.skip("oracle/_ref not built (reference sources absent)")
    a = subprocess.run([ref], capture_output=True, text=True, check=True).stdout
    b = subprocess.run([mine], capture_output=True, text=True, check=True).stdout
    assert a == b and "pk_kernels" in a


@pytest.mark.parametrize("n,qb", [(0, 32), (48, 32), (64, 48), (96, 64), (16416, 32)])
def test_bad_shapes_refused_before_any_device(pkb, n, qb):
    x = np.zeros(max(n, 1) * 2, np.float32)
    with pytest.raises(pkb.PkbError) as e:
        pkb.quantize_host(x, n, qb, T=1)
    assert e.value.code == 1  # PKB_EINVAL


def test_bad_rows_and_stride_refused(pkb):
    lib = pkb.lib()
    out = np.zeros(64, np.float32)
    assert lib.pkb_gemm_q8_host(out.ctypes.data, 32, None, None, None, 24, None, None, 32, 32, 1, 0, 0) == 1
    assert lib.pkb_gemm_q8_host(out.ctypes.data, 8, None, None, None, 16, None, None, 32, 32, 2, 0, 0) == 1
    assert b"output stride" in lib.pkb_last_error()
    assert lib.pkb_gemm_q8_host(out.ctypes.data, 16, None, None, None, 16, None, None, 32, 32, 1, 0, 7) == 1
    assert b"rounding mode" in lib.pkb_last_error()


def test_no_device_is_an_error_not_a_fallback(pkb):
    """Without a GPU the compute entries fail; nothing is computed on the CPU."""
    if pkb.device_count() > 0:
        pytest.skip("a GPU is present")
    x = np.ones(64, np.float32)
    with pytest.raises(pkb.PkbError) as e:
        pkb.quantize_host(x, 32, 32, T=2)
    assert e.value.code in (2, 5)
