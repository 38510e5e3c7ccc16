"""The C ABI (include/nimf_cuda.h) without a GPU: the library loads, exports
every declared symbol, and its host-side argument / state checks answer with
status codes (no kernel is launched in these tests)."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import nimf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nimf_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nimf_[a-z0-9_]+)\s*\(", src)))


def test_header_and_python_binding_agree():
    assert declared_symbols() == sorted(nimf.EXPORTS)


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(nimf.library_path())
    for name in declared_symbols():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", nimf.library_path()], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (nimf_[a-z0-9_]+)$", out, flags=re.M))
    assert set(declared_symbols()) <= exported


def test_calls_before_init_report_state_error():
    L = nimf.lib()
    if nimf._initialised_device is not None:
        pytest.skip("library already initialised in this process")
    y = np.zeros(4, np.float32)
    x = np.zeros(4, np.float32)
    st = L.nimf_matmul_w(1, x.ctypes.data_as(ctypes.c_void_p), 1, y.ctypes.data_as(ctypes.c_void_p))
    assert st == -7
    assert b"nimf_init" in L.nimf_last_error()
    with pytest.raises(nimf.CatchableError, match="STATE"):
        nimf.check(st)


def test_init_without_gpu_is_an_error_not_a_fallback():
    n = ctypes.c_int(-1)
    st = nimf.lib().nimf_device_count(ctypes.byref(n))
    if st == 0 and n.value > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(nimf.CatchableError):
        nimf.newBackend()


def test_only_cuda_backend_is_offered():
    with pytest.raises(nimf.CatchableError):
        nimf.newBackend("cpu")


def test_customfloat_fields_mirror_newCustomFloat():
    """customfloat.nim:15-31 field derivation and presets :34-43."""
    cf = nimf.newCustomFloat(4, 3)
    assert (cf.totalBits, cf.itemSize, cf.bias, cf.maxExp, cf.name) == (8, 1, 7, 15, "float8_e4m3")
    cf = nimf.newCustomFloat(6, 10)
    assert (cf.totalBits, cf.itemSize, cf.bias, cf.maxExp) == (17, 3, 31, 63)
    cf = nimf.newCustomFloat(0, 7)
    assert (cf.bias, cf.maxExp, cf.itemSize) == (0, 0, 1)
    assert nimf.FP64C.itemSize == 8 and nimf.FP64C.usesUint64
    assert not nimf.newCustomFloat(11, 60).usesUint64
    assert nimf.FP8_E4M3.name == "fp8_e4m3"
