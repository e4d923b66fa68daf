"""GPU parity tests of the matmul kernels, called through the C ABI.

Error measure (componentwise, so cancellation cannot inflate it):
    rel = max |c - c64| / (|alpha| sum_k |a_ik b_kj| + |beta c0| + |bias_j|)
with c64 an fp64 evaluation of the same expression.
Tolerances (stated by the path's specification):
    exact-fp32 SIMT and 3xTF32:  rel <= 1e-5 * sqrt(K)
    plain TF32 (opt-in):          rel <= 5e-3
The CPU oracle (NpArray restatement) and the reference's own cuda_matmul
(cuBLAS, built from the reference sources into oracle/_ref) are checked at the
same bound (twice the tolerance, since both sides carry rounding error).
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np
import pytest
import torch

import oracle
from moonxi_net_b200 import _lib, ops, synthetic

pytestmark = pytest.mark.gpu

PRECS = ["fp32", "3xtf32", "tf32"]
LAYOUTS = [(0, 0), (0, 1), (1, 0), (1, 1)]


def tol(prec: str, K: int) -> float:
    return 5e-3 if prec == "tf32" else 1e-5 * math.sqrt(max(K, 1))


def fp64_ref(a, b, M, K, N, ta, tb, alpha=1.0, beta=0.0, c0=None, bias=None, relu=False):
    """(c64, scale) on the GPU in float64 (test-side checker only)."""
    A = a.double().reshape((K, M) if ta else (M, K))
    B = b.double().reshape((N, K) if tb else (K, N))
    A = A.t() if ta else A
    B = B.t() if tb else B
    c = alpha * (A @ B)
    scale = abs(alpha) * (A.abs() @ B.abs())
    if beta != 0.0:
        c = c + beta * c0.double()
        scale = scale + abs(beta) * c0.double().abs()
    if bias is not None:
        c = c + bias.double()[None, :]
        scale = scale + bias.double().abs()[None, :]
    if relu:
        c = torch.clamp_min(c, 0.0)
    return c, scale


def rel_err(c, c64, scale) -> float:
    d = (c.double() - c64).abs()
    s = torch.where(scale > 0, scale, torch.ones_like(scale))
    r = torch.where(scale > 0, d / s, d)
    return float(r.max()) if r.numel() else 0.0


def make(M, K, N, ta, tb, seed, bias=False, dev="cuda"):
    a, b, bv = synthetic.gemm_problem(M, K, N, ta, tb, seed, bias)
    A = torch.from_numpy(a).to(dev)
    B = torch.from_numpy(b).to(dev)
    BV = torch.from_numpy(bv).to(dev) if bias else None
    return a, b, bv, A, B, BV


def run_case(M, K, N, ta, tb, prec, seed=1, bias=False, relu=False, alpha=1.0, beta=0.0):
    a, b, bv, A, B, BV = make(M, K, N, ta, tb, seed, bias)
    c0 = torch.randn((M, N), device="cuda", generator=torch.Generator("cuda").manual_seed(7))
    C = c0.clone()
    ops.gemm(A, B, M, K, N, ta=ta, tb=tb, alpha=alpha, beta=beta, bias=BV, relu=relu, out=C,
             precision=prec)
    torch.cuda.synchronize()
    c64, scale = fp64_ref(A, B, M, K, N, ta, tb, alpha, beta, c0, BV, relu)
    return C, c64, scale, (a, b, bv)


# --------------------------------------------------------------------------- KATs
def test_reference_kat_matmul_2x2(cuda_device):
    """nparray/nparray_wbtest.mbt:205-214 through the reference-compatible ABI."""
    a = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="cuda")
    b = torch.tensor([[5.0, 6.0], [7.0, 8.0]], device="cuda")
    for prec in PRECS:
        c = ops.matmul(a, b, 2, 2, 2, precision=prec)
        torch.cuda.synchronize()
        assert c.flatten().tolist() == [19.0, 22.0, 43.0, 50.0], prec
    # the unchanged moonbit stub signature, default stream, default precision
    c = torch.zeros((2, 2), device="cuda")
    rc = _lib.lib().moonbit_cuda_matmul(None, a.data_ptr(), b.data_ptr(), c.data_ptr(), 2, 2, 2,
                                        0, 0, 1.0, 0.0)
    torch.cuda.synchronize()
    assert rc == 0 and c.flatten().tolist() == [19.0, 22.0, 43.0, 50.0]


def test_reference_kat_matmul_backward(cuda_device):
    """grad/grad_wbtest.mbt:104-134: dA = og B^T (NT), dB = A^T og (TN), exact."""
    a = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="cuda")
    b = torch.tensor([[5.0, 6.0], [7.0, 8.0]], device="cuda")
    og = torch.full((2, 2), 0.25, device="cuda")
    for prec in PRECS:
        da = ops.matmul(og, b, 2, 2, 2, tb=True, precision=prec)
        db = ops.matmul(a, og, 2, 2, 2, ta=True, precision=prec)
        torch.cuda.synchronize()
        assert da.flatten().tolist() == [2.75, 3.75, 2.75, 3.75], prec
        assert db.flatten().tolist() == [1.0, 1.0, 1.5, 1.5], prec


def test_reference_kat_linear(cuda_device):
    """model/model_wbtest.mbt:11-44: Linear forward with and without bias."""
    x = torch.tensor([[3.0, 5.0]], device="cuda")
    w = torch.tensor([[1.0, 0.0, 1.0], [0.0, 1.0, 1.0]], device="cuda")
    y = ops.linear(x, w, torch.zeros(3, device="cuda"))
    x2 = torch.tensor([[1.0, 1.0]], device="cuda")
    w2 = torch.tensor([[2.0, 4.0], [3.0, 5.0]], device="cuda")
    y2 = ops.linear(x2, w2, torch.tensor([10.0, 20.0], device="cuda"))
    torch.cuda.synchronize()
    assert y.flatten().tolist() == [3.0, 5.0, 8.0]
    assert y2.flatten().tolist() == [15.0, 29.0]


# --------------------------------------------------------------- square sweep
@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("ta,tb", LAYOUTS)
@pytest.mark.parametrize("n", [512, 1024, 2048])
def test_square(cuda_device, n, ta, tb, prec):
    C, c64, scale, _ = run_case(n, n, n, ta, tb, prec, seed=1)
    assert rel_err(C, c64, scale) <= tol(prec, n)


@pytest.mark.parametrize("prec", ["fp32", "3xtf32", "tf32"])
@pytest.mark.parametrize("n", [4096, 8192])
def test_square_large(cuda_device, n, prec):
    C, c64, scale, _ = run_case(n, n, n, 0, 0, prec, seed=1)
    assert rel_err(C, c64, scale) <= tol(prec, n)


@pytest.mark.parametrize("ta,tb", LAYOUTS)
def test_fp32_wide_tile_edges(cuda_device, ta, tb):
    """Exact FP32 on a grid the 128x256 warp-specialised kernel takes (63 x 32
    tiles fill 97 % of the waves) with partial tiles in M and N, a K tail
    (K % 16 = 8), alpha, beta, bias and ReLU, every layout."""
    M, K, N = 7940, 1000, 8004
    C, c64, scale, _ = run_case(M, K, N, ta, tb, "fp32", seed=3, bias=True, relu=True,
                                alpha=0.5, beta=0.25)
    assert rel_err(C, c64, scale) <= tol("fp32", K)


@pytest.mark.parametrize("prec", ["fp32", "3xtf32"])
@pytest.mark.parametrize("ta,tb", LAYOUTS)
def test_bias_relu_epilogue(cuda_device, ta, tb, prec):
    C, c64, scale, _ = run_case(1024, 1024, 1024, ta, tb, prec, seed=1, bias=True, relu=True)
    assert rel_err(C, c64, scale) <= tol(prec, 1024)
    assert float(C.min()) >= 0.0


@pytest.mark.parametrize("prec", PRECS)
def test_alpha_beta(cuda_device, prec):
    C, c64, scale, _ = run_case(640, 384, 520, 1, 0, prec, alpha=0.5, beta=-1.5, bias=True)
    assert rel_err(C, c64, scale) <= tol(prec, 384)


# ---------------------------------------------------------- ragged / skinny
RAGGED = synthetic.ragged_shapes()


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0)])
def test_ragged_default_precision(cuda_device, ta, tb):
    worst = 0.0
    for (M, K, N) in RAGGED:
        C, c64, scale, _ = run_case(M, K, N, ta, tb, "default", seed=4, bias=True, relu=True)
        e = rel_err(C, c64, scale)
        assert e <= tol("fp32", K), (M, K, N, e)
        worst = max(worst, e)


@pytest.mark.parametrize("prec", ["3xtf32", "tf32", "fp32"])
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0)])
def test_ragged_forced(cuda_device, prec, ta, tb):
    for (M, K, N) in [(1, 4096, 1000), (7, 784, 257), (33, 3072, 10), (127, 512, 257),
                      (1000, 784, 10), (1000, 4096, 1000), (127, 3072, 100)]:
        C, c64, scale, _ = run_case(M, K, N, ta, tb, prec, seed=4, bias=True, relu=True)
        assert rel_err(C, c64, scale) <= tol(prec, K), (M, K, N)


@pytest.mark.parametrize("prec", PRECS)
def test_tiny_and_odd(cuda_device, prec):
    for M in (1, 2, 3, 17):
        for N in (1, 3, 5, 129):
            for K in (1, 3, 5, 17, 33, 300):
                for ta, tb in LAYOUTS:
                    C, c64, scale, _ = run_case(M, K, N, ta, tb, prec, seed=M * 131 + N * 7 + K)
                    assert rel_err(C, c64, scale) <= tol(prec, K), (M, K, N, ta, tb)


def test_k_zero(cuda_device):
    """K = 0: C = beta C + bias (no product), for every precision."""
    for prec in PRECS:
        a = torch.zeros(1, device="cuda")
        b = torch.zeros(1, device="cuda")
        bias = torch.arange(5, dtype=torch.float32, device="cuda")
        c0 = torch.ones((3, 5), device="cuda")
        C = c0.clone()
        ops.gemm(a, b, 3, 0, 5, alpha=1.0, beta=2.0, bias=bias, out=C, precision=prec)
        torch.cuda.synchronize()
        assert torch.equal(C, 2.0 * c0 + bias[None, :]), prec


def test_unaligned_pointers(cuda_device):
    """Operands starting off a 16-byte boundary take the cp.async feed."""
    M, K, N = 300, 257, 199
    for prec in PRECS:
        for ta, tb in LAYOUTS:
            a, b, _ = synthetic.gemm_problem(M, K, N, ta, tb, 9)
            abuf = torch.zeros(a.size + 1, device="cuda")
            bbuf = torch.zeros(b.size + 3, device="cuda")
            abuf[1:].copy_(torch.from_numpy(a.reshape(-1)))
            bbuf[3:].copy_(torch.from_numpy(b.reshape(-1)))
            A, B = abuf[1:], bbuf[3:]
            C = ops.gemm(A, B, M, K, N, ta=ta, tb=tb, precision=prec)
            torch.cuda.synchronize()
            c64, scale = fp64_ref(A, B, M, K, N, ta, tb)
            assert rel_err(C, c64, scale) <= tol(prec, K), (prec, ta, tb)


def test_leading_dimensions(cuda_device):
    """Sub-matrix views through explicit lda/ldb/ldc."""
    M, K, N = 200, 300, 150
    big_a = torch.randn((M, K + 37), device="cuda")
    big_b = torch.randn((K, N + 5), device="cuda")
    big_c = torch.zeros((M, N + 11), device="cuda")
    for prec in PRECS:
        big_c.zero_()
        ops.gemm(big_a, big_b, M, K, N, lda=K + 37, ldb=N + 5, ldc=N + 11, out=big_c,
                 precision=prec)
        torch.cuda.synchronize()
        A = big_a[:, :K]
        B = big_b[:, :N]
        c64 = A.double() @ B.double()
        scale = A.double().abs() @ B.double().abs()
        assert rel_err(big_c[:, :N], c64, scale) <= tol(prec, K)
        assert float(big_c[:, N:].abs().max()) == 0.0  # untouched padding


def test_deterministic(cuda_device):
    for prec in PRECS:
        _, _, _, A, B, _ = make(1000, 4096, 1000, 0, 1, 3)
        c1 = ops.gemm(A, B, 1000, 4096, 1000, tb=True, precision=prec)
        c2 = ops.gemm(A, B, 1000, 4096, 1000, tb=True, precision=prec)
        torch.cuda.synchronize()
        assert torch.equal(c1, c2), prec


# ------------------------------------------------- parity with the oracles
@pytest.mark.parametrize("ta,tb", LAYOUTS)
def test_vs_cpu_oracle(cuda_device, ta, tb):
    """Against the NpArray restatement (oracle/np_oracle.c) on the same inputs."""
    M, K, N = 192, 320, 160
    for prec in PRECS:
        C, c64, scale, (a, b, _) = run_case(M, K, N, ta, tb, prec, seed=5, alpha=1.0)
        c_or = oracle.gemm(a, b, M, K, N, ta, tb, threads=oracle.default_threads())
        d = np.abs(C.cpu().numpy().astype(np.float64) - c_or.astype(np.float64))
        s = scale.cpu().numpy()
        assert float((d / np.where(s > 0, s, 1)).max()) <= 2 * tol(prec, K), prec


def _ref_gpu_lib():
    path = oracle.reference_gpu_lib_path()
    assert os.path.exists(path), f"reference GPU library missing: {path} (make -C oracle ref)"
    L = ctypes.CDLL(path)
    L.cublas_create_handle.restype = ctypes.c_void_p
    L.cuda_matmul.restype = ctypes.c_int
    L.cuda_matmul.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_float] * 2
    return L


@pytest.mark.parametrize("ta,tb", LAYOUTS)
@pytest.mark.parametrize("n", [512, 2048])
def test_vs_reference_cuda_matmul(cuda_device, n, ta, tb):
    """Against the reference's own cuda_matmul (cuBLAS FP32, built unmodified
    from moonxi-net-gpu/cuda/cuda_kernels.cu) on identical device inputs."""
    L = _ref_gpu_lib()
    h = L.cublas_create_handle()
    assert h
    M, K, N = n, n + 64, n - 32
    _, _, _, A, B, _ = make(M, K, N, ta, tb, 1)
    c_ref = torch.zeros((M, N), device="cuda")
    torch.cuda.synchronize()
    rc = L.cuda_matmul(h, A.data_ptr(), B.data_ptr(), c_ref.data_ptr(), M, K, N, ta, tb, 1.0, 0.0)
    torch.cuda.synchronize()
    assert rc == 0
    c64, scale = fp64_ref(A, B, M, K, N, ta, tb)
    for prec in PRECS:
        C = ops.gemm(A, B, M, K, N, ta=ta, tb=tb, precision=prec)
        torch.cuda.synchronize()
        assert rel_err(C, c_ref.double(), scale) <= 2 * tol(prec, K), prec
    assert rel_err(c_ref, c64, scale) <= tol("fp32", K)


# ------------------------------------------------------------- error paths
def test_invalid_arguments(cuda_device):
    L = _lib.lib()
    a = torch.zeros(16, device="cuda")
    assert L.moonbit_cuda_matmul(None, a.data_ptr(), a.data_ptr(), a.data_ptr(), -1, 2, 2, 0, 0,
                                 1.0, 0.0) == _lib.MX_ERR_INVALID
    assert L.mx_gemm_ex(None, a.data_ptr(), a.data_ptr(), a.data_ptr(), None, 4, 4, 4, 0, 0, 2, 0,
                        0, 1.0, 0.0, 0, None, 0) == _lib.MX_ERR_INVALID
    assert L.moonbit_cuda_matmul(None, None, a.data_ptr(), a.data_ptr(), 2, 2, 2, 0, 0, 1.0,
                                 0.0) == _lib.MX_ERR_INVALID
    # M == 0 or N == 0 is a no-op
    assert L.moonbit_cuda_matmul(None, a.data_ptr(), a.data_ptr(), a.data_ptr(), 0, 2, 2, 0, 0,
                                 1.0, 0.0) == 0


def test_status_word_clean(cuda_device):
    rc, where = ops.status()
    assert rc == 0, (rc, where)


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0)])
def test_tf32_large_ragged_direct(cuda_device, ta, tb):
    """Plain TF32 with the operands read in place (TMA-aligned: no rounded
    copies; the tensor cores use each fp32 value's TF32 part) on a large
    grid with ragged M and N: bias + ReLU and alpha/beta against fp64 at the
    TF32 tolerance, run to run bit-identical."""
    M, K, N = 4608 + 136, 1028, 4200
    C, c64, scale, _ = run_case(M, K, N, ta, tb, "tf32", seed=9, bias=True, relu=True)
    assert rel_err(C, c64, scale) <= tol("tf32", K)
    C2, _, _, _ = run_case(M, K, N, ta, tb, "tf32", seed=9, bias=True, relu=True)
    assert torch.equal(C, C2)
    C, c64, scale, _ = run_case(M, K, N, ta, tb, "tf32", seed=10, alpha=-0.5, beta=0.75)
    assert rel_err(C, c64, scale) <= tol("tf32", K)
