"""GPU tests of mx_gemm_3xtf32_noalloc, the allocation-free GEMM entry point.

Some callers may not allocate device memory inside a library call: a host
runtime that reserved its whole device-memory budget up front and carves it
up itself (the reference GPU backend runs everything out of one bump pool),
or a process under a fixed memory budget.  This entry point serves them: its
scratch is a fixed 64 MiB array inside the library.  These tests call it
through the C ABI and hold it to the regular 3xTF32 entry point (mx_gemm_ex)
on the same inputs, and to an fp64 evaluation of the same expression, for
two different problems in a row, so stale scratch contents from the previous
call would show.  This file is named to run last.
"""
from __future__ import annotations

import math

import pytest
import torch

from moonxi_net_b200 import _lib

pytestmark = pytest.mark.gpu

# the tolerance of the fp32-class paths: componentwise relative error
# |c - c_ref| / (|alpha| sum_k |a b| + |beta c0| + |bias|) <= 1e-5 * sqrt(K)


def _tol(K):
    return 1e-5 * math.sqrt(K)


def _problem(M, K, N, ta, tb, seed):
    g = torch.Generator("cuda").manual_seed(seed)
    a = torch.randn((K, M) if ta else (M, K), device="cuda", generator=g)
    b = torch.randn((N, K) if tb else (K, N), device="cuda", generator=g)
    bias = torch.randn(N, device="cuda", generator=g)
    c0 = torch.randn((M, N), device="cuda", generator=g)
    return a, b, bias, c0


def _scale(a, b, M, K, N, ta, tb, alpha, beta, c0, bias):
    A = a.double().t() if ta else a.double()
    B = b.double().t() if tb else b.double()
    return abs(alpha) * (A.abs() @ B.abs()) + abs(beta) * c0.double().abs() + \
        bias.double().abs()[None, :]


def _fp64(a, b, bias, c0, M, K, N, ta, tb, alpha, beta, relu):
    A = a.double().t() if ta else a.double()
    B = b.double().t() if tb else b.double()
    c = alpha * (A @ B) + beta * c0.double() + bias.double()[None, :]
    return torch.clamp_min(c, 0.0) if relu else c


def _regular(a, b, bias, c0, M, K, N, ta, tb, alpha, beta, relu):
    c = c0.clone()
    rc = _lib.lib().mx_gemm_ex(None, a.data_ptr(), b.data_ptr(), c.data_ptr(), bias.data_ptr(),
                               M, K, N, ta, tb, 0, 0, 0, alpha, beta, relu,
                               torch.cuda.current_stream().cuda_stream, _lib.PREC_3XTF32)
    assert rc == 0
    return c


def _noalloc(a, b, bias, c0, M, K, N, ta, tb, alpha, beta, relu, status=None):
    c = c0.clone()
    rc = _lib.lib().mx_gemm_3xtf32_noalloc(
        a.data_ptr(), b.data_ptr(), c.data_ptr(), bias.data_ptr(), M, K, N, ta, tb, alpha, beta,
        relu, status.data_ptr() if status is not None else None,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.lib().mx_status_string(rc)
    return c


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_noalloc_matches_regular_entry_point_two_calls(cuda_device, ta, tb):
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    # two different problems back to back: the second reuses the scratch
    for (M, K, N, alpha, beta, relu, seed) in [(1000, 1536, 768, 1.0, 0.0, 1, 11),
                                               (333, 517, 1290, 0.5, -2.0, 0, 12)]:
        a, b, bias, c0 = _problem(M, K, N, ta, tb, seed)
        want = _regular(a, b, bias, c0, M, K, N, ta, tb, alpha, beta, relu)
        got = _noalloc(a, b, bias, c0, M, K, N, ta, tb, alpha, beta, relu, status)
        torch.cuda.synchronize()
        scale = _scale(a, b, M, K, N, ta, tb, alpha, beta, c0, bias)
        err = float(((got.double() - want.double()).abs() / scale).max())
        assert err <= _tol(K), (M, K, N, err)
        exact = _fp64(a, b, bias, c0, M, K, N, ta, tb, alpha, beta, relu)
        err64 = float(((got.double() - exact).abs() / scale).max())
        assert err64 <= _tol(K), (M, K, N, err64)
    assert status.tolist() == [0, 0]


def test_noalloc_allocates_nothing(cuda_device):
    M, K, N = 1024, 2048, 1024
    a, b, bias, c0 = _problem(M, K, N, 0, 1, 21)
    c = c0.clone()
    args = (a.data_ptr(), b.data_ptr(), c.data_ptr(), bias.data_ptr(), M, K, N, 0, 1, 1.0, 0.0, 0,
            None, torch.cuda.current_stream().cuda_stream)
    assert _lib.lib().mx_gemm_3xtf32_noalloc(*args) == 0  # first call: per-device setup
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert _lib.lib().mx_gemm_3xtf32_noalloc(*args) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    M = K = N = 4096  # split copies need 256 MiB > 64 MiB
    a = torch.zeros((M, K), device="cuda")
    b = torch.zeros((K, N), device="cuda")
    c = torch.full((M, N), 7.0, device="cuda")
    rc = _lib.lib().mx_gemm_3xtf32_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), None, M, K,
                                           N, 0, 0, 1.0, 0.0, 0, None, None)
    assert rc == _lib.MX_ERR_UNSUPPORTED
    torch.cuda.synchronize()
    assert bool((c == 7.0).all())  # nothing was launched


def test_noalloc_status_word_reads_clear(cuda_device):
    """Calls without a dev_status report through the library's own word,
    which mx_noalloc_status reads and clears; after good calls it is zero."""
    import ctypes
    M, K, N = 256, 384, 512
    a, b, bias, c0 = _problem(M, K, N, 1, 0, 31)
    got = _noalloc(a, b, bias, c0, M, K, N, 1, 0, 1.0, 0.0, 1)
    where = ctypes.c_int32(-1)
    assert _lib.lib().mx_noalloc_status(ctypes.byref(where)) == _lib.MX_OK
    assert where.value == 0
    exact = _fp64(a, b, bias, c0, M, K, N, 1, 0, 1.0, 0.0, 1)
    scale = _scale(a, b, M, K, N, 1, 0, 1.0, 0.0, c0, bias)
    assert float(((got.double() - exact).abs() / scale).max()) <= _tol(K)
