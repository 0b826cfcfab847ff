"""CPU: the C-ABI library loads and exports every symbol include/*.h declares;
host-side validation answers before any launch (no GPU needed)."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//.*", "", src)
        names |= set(re.findall(r"\b(madi_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from madi_b200 import _lib, build
    build.build()
    return _lib.load()


def test_header_declares_the_boundary():
    names = _declared_symbols()
    for must in ("madi_init", "madi_dispatch", "madi_get_function", "madi_sync", "madi_q8_linear"):
        assert must in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in _declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_the_header():
    from madi_b200 import _lib
    assert set(_declared_symbols()) == set(_lib.SIGNATURES), "ctypes signatures out of sync with include/madi_q8.h"


def test_reference_kernel_names_resolve_without_a_device(lib):
    out = ctypes.c_int(-1)
    names = ["gemv_q8", "gemv_q8_bias", "gemv_q8_bias_gelu", "gemv_q8_bias_res", "gemv_q8_qkv", "logit_gemv_q8",
             "dequant_q8_f16", "mul_mm_q8", "m4_gemm_q8tg", "m4_gemm_q8_bias_gelu"]
    ids = set()
    for n in names:
        assert lib.madi_get_function(n.encode(), ctypes.byref(out)) == 0, n
        ids.add(out.value)
    assert len(ids) == len(names)
    assert lib.madi_get_function(b"no_such_kernel", ctypes.byref(out)) == -3
    assert b"no_such_kernel" in lib.madi_last_error()


def test_calls_before_init_fail_cleanly(lib):
    from madi_b200 import _lib
    w = _lib.madi_q8w(0x1000, 0x2000, 64, 64)
    rc = lib.madi_q8_linear(ctypes.byref(w), 0x3000, 1, 16, None, 0, 0, None, 0x4000, 1, None)
    assert rc == _lib.MADI_ENOINIT
    assert lib.madi_sync(10) == _lib.MADI_ENOINIT
    assert lib.madi_dispatch(0, 1, 1, 1, 1, 1, 1, None, None, 0) == _lib.MADI_ENOINIT
    assert lib.madi_alloc(64) is None


def test_init_without_gpu_reports_an_error(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; the no-device path is exercised only on CPU hosts")
    rc = lib.madi_init(0)
    assert rc != 0
    assert len(lib.madi_last_error()) > 0


def test_product_package_never_imports_the_oracle():
    for path in glob.glob(os.path.join(ROOT, "madi_b200", "**", "*.*"), recursive=True):
        if path.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
            src = open(path).read()
            assert "oracle" not in re.sub(r"#.*|//.*", "", src).replace("oracle's", ""), path
