"""The C-ABI library builds, loads and exports every symbol include/talos_cuda.h
declares; argument checks that run before any GPU work return the right status.
No compute calls: these run without a GPU."""
import ctypes as C
import os
import re
import subprocess

import pytest

from talos_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "talos_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(talos_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    build.build_cuda()
    return _lib.load()


def test_header_and_bindings_agree():
    assert declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.lib_path()], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (talos_[a-z0-9_]+)$", out, flags=re.M))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing


def test_build_targets_sm100a():
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.NVCC_FLAGS)


def test_bad_config_rejected_before_gpu(lib):
    cfg = _lib.Cfg(2, 6, 4, 288, 768, 256, 4096, 48, 1e-5, 1e4)  # 6 % 4 != 0
    h = C.c_void_p()
    st = lib.talos_ctx_create(C.byref(cfg), 0, C.byref(h))
    assert st == _lib.INVALID_ARG
    assert b"multiple of head_count_kv" in lib.talos_last_error()


def test_null_arguments(lib):
    assert lib.talos_ctx_create(None, 0, None) == _lib.INVALID_ARG
    assert lib.talos_forward(None, 0, 0, None) == _lib.INVALID_ARG
    assert lib.talos_weight_upload(None, b"x", None, 0, 0, 1, 1) == _lib.INVALID_ARG
    assert lib.talos_ctx_destroy(None) == _lib.OK


def test_dequant_argument_checks(lib):
    buf = (C.c_uint8 * 18)()
    out = (C.c_float * 32)()
    assert lib.talos_dequant(3, buf, 32, out) == _lib.UNSUPPORTED  # Q4_1
    assert lib.talos_dequant(2, buf, 31, out) == _lib.INVALID_ARG  # not a block multiple


def test_device_count_callable(lib):
    n = C.c_int(-1)
    assert lib.talos_device_count(C.byref(n)) == _lib.OK
    assert n.value >= 0
