"""CPU tests of the C-ABI library: it loads, exports every symbol the header
declares, and answers calls without a GPU with a status code (no crash)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from moonxi_net_b200 import _lib

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, re.M):
            if m.group(1) not in ("if", "defined"):
                names.append(m.group(1))
    return sorted(set(names))


def test_header_declares_the_reference_stub_names():
    names = declared_functions()
    for n in ("cuda_matmul", "moonbit_cuda_matmul", "moonbit_cuda_matmul_ex",
              "moonbit_cuda_linear_fwd", "moonbit_cuda_set_device"):
        assert n in names


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for name in declared_functions():
        assert name in exported, name
        assert getattr(L, name) is not None
    # the Python binding covers the same set
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_no_internal_symbols_leak():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(declared_functions())


def test_status_strings():
    L = _lib.lib()
    assert L.mx_status_string(0) == b"ok"
    assert b"timed out" in L.mx_status_string(_lib.MX_ERR_TIMEOUT)
    assert L.mx_status_string(12345) == b"unknown status"


def test_calls_without_device_report_status():
    """In a container without a GPU every entry point returns a status code."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = _lib.lib()
    buf = (ctypes.c_float * 4)()
    p = ctypes.addressof(buf)
    assert L.cuda_matmul(None, p, p, p, 2, 2, 2, 0, 0, 1.0, 0.0) == _lib.MX_ERR_NO_DEVICE
    assert L.moonbit_cuda_matmul(None, p, p, p, 2, 2, 2, 0, 0, 1.0, 0.0) == _lib.MX_ERR_NO_DEVICE
    assert L.mx_context_create(0) is None
    assert L.mx_relu_backward(None, p, p, p, 4, None) == _lib.MX_ERR_NO_DEVICE
    g = _lib.SplitGemm()
    assert L.mx_gemm_split_pair(None, ctypes.byref(g), ctypes.byref(g), None) == \
        _lib.MX_ERR_NO_DEVICE
    out = (ctypes.c_int32 * 6)()
    assert L.mx_tc_split_plan(None, 128, 256, 64, 3, out) == _lib.MX_ERR_NO_DEVICE


def test_product_does_not_import_oracle():
    """The package never reaches the CPU oracle (the checker)."""
    pkg = os.path.join(ROOT, "moonxi-net_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".c")):
                text = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in text and "np_oracle" not in text, f
