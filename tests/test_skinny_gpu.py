"""GPU tests of the skinny-shape kernel (min(M, N) <= 64, gemm_skinny.cu),
through the C ABI at the exact-fp32 precision: both orientations (small M
streams B; small N runs as C^T = B^T A^T and streams A), split-K with the
arrival-counter reduction, alpha/beta/bias/ReLU, sub-matrix leading
dimensions, unaligned pointers, determinism, and one launch per call.
Tolerance as for every fp32-class path: componentwise 1e-5 sqrt(K)."""
from __future__ import annotations

import math

import pytest
import torch

from moonxi_net_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _check(M, K, N, ta, tb, seed, alpha=1.0, beta=0.0, bias=True, relu=True):
    g = torch.Generator("cuda").manual_seed(seed)
    A = torch.randn((K, M) if ta else (M, K), device="cuda", generator=g)
    B = torch.randn((N, K) if tb else (K, N), device="cuda", generator=g)
    bv = torch.randn(N, device="cuda", generator=g) if bias else None
    c0 = torch.randn((M, N), device="cuda", generator=g)
    C = c0.clone()
    ops.gemm(A, B, M, K, N, ta=ta, tb=tb, alpha=alpha, beta=beta, bias=bv, relu=relu, out=C,
             precision="fp32")
    torch.cuda.synchronize()
    a = A.double().t() if ta else A.double()
    b = B.double().t() if tb else B.double()
    ref = alpha * (a @ b) + beta * c0.double()
    scale = abs(alpha) * (a.abs() @ b.abs()) + abs(beta) * c0.double().abs()
    if bias:
        ref = ref + bv.double()[None, :]
        scale = scale + bv.double().abs()[None, :]
    if relu:
        ref = ref.clamp_min(0.0)
    err = float(((C.double() - ref).abs() / scale.clamp_min(1e-30)).max())
    assert err <= 1e-5 * math.sqrt(K), (M, K, N, ta, tb, err)
    return C


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,K,N", [(1, 4096, 1000), (33, 3072, 257), (64, 777, 4096),
                                   (1000, 4096, 10), (4096, 512, 64), (5, 20000, 3),
                                   (1, 1, 1), (60, 33, 61)])
def test_skinny_shapes(cuda_device, M, K, N, ta, tb):
    _check(M, K, N, ta, tb, seed=M + 7 * N + K, alpha=0.75, beta=-0.5)


def test_skinny_wide_single_row(cuda_device):
    _check(1, 96, 200_003, 0, 0, seed=3)  # thousands of column tiles, one split


def test_skinny_leading_dimensions_and_unaligned(cuda_device):
    M, K, N = 20, 300, 150
    big_a = torch.randn((M, K + 37), device="cuda")
    big_b = torch.randn((K, N + 5), device="cuda")
    big_c = torch.zeros((M, N + 11), device="cuda")
    ops.gemm(big_a, big_b, M, K, N, lda=K + 37, ldb=N + 5, ldc=N + 11, out=big_c,
             precision="fp32")
    torch.cuda.synchronize()
    A, B = big_a[:, :K], big_b[:, :N]
    err = float(((big_c[:, :N].double() - A.double() @ B.double()).abs() /
                 (A.double().abs() @ B.double().abs())).max())
    assert err <= 1e-5 * math.sqrt(K)
    assert float(big_c[:, N:].abs().max()) == 0.0
    # operands one float off a 16-byte boundary
    abuf = torch.randn(M * K + 1, device="cuda")
    bbuf = torch.randn(K * N + 3, device="cuda")
    A, B = abuf[1:], bbuf[3:]
    C = ops.gemm(A, B, M, K, N, precision="fp32")
    torch.cuda.synchronize()
    a, b = A.view(M, K).double(), B.view(K, N).double()
    err = float(((C.double() - a @ b).abs() / (a.abs() @ b.abs())).max())
    assert err <= 1e-5 * math.sqrt(K)


def test_skinny_deterministic_single_launch(cuda_device):
    M, K, N = 7, 4096, 1000   # split over K: partials + arrival counters
    A = torch.randn((M, K), device="cuda")
    B = torch.randn((K, N), device="cuda")
    n0 = _lib.lib().mx_kernel_launch_count()
    c1 = ops.gemm(A, B, M, K, N, precision="fp32")
    n1 = _lib.lib().mx_kernel_launch_count()
    c2 = ops.gemm(A, B, M, K, N, precision="fp32")
    torch.cuda.synchronize()
    assert n1 - n0 == 1
    assert torch.equal(c1, c2)
    assert ops.resolve_precision(M, K, N) == "fp32"
