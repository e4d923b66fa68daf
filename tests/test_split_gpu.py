"""GPU tests of the split-form (3xTF32 operands kept as hi/lo copies) path:
mx_split_tf32, mx_gemm_split_ex in every operand majorness with the fused
ReLU-mask and split-output epilogue, and the split-form MLP step, which must
reproduce the per-call 3xTF32 step bit for bit."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from moonxi_net_b200 import nn, ops

pytestmark = pytest.mark.gpu


def _rna_tf32(x: torch.Tensor) -> torch.Tensor:
    """Round-to-nearest (ties away) to tf32, as cvt.rna.tf32.f32 (checker)."""
    b = x.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    r = (b + 0x1000) & 0xFFFFE000
    r = torch.where(r >= 2 ** 31, r - 2 ** 32, r).to(torch.int32)
    return r.view(torch.float32)


def test_split_tf32_matches_rounding_rule(cuda_device):
    x = torch.randn(300, 124, device="cuda") * 1e3
    hi = torch.empty_like(x)
    lo = torch.empty_like(x)
    ops.split_tf32(x, hi, lo)
    torch.cuda.synchronize()
    assert torch.equal(hi, _rna_tf32(x))
    assert torch.equal(lo, _rna_tf32(x - hi))
    # hi + lo carries x to about 2^-22 relative
    rel = ((hi.double() + lo.double() - x.double()).abs() / x.double().abs().clamp_min(1e-30))
    assert float(rel.max()) < 2.0 ** -20


def _split(t):
    # 64 readable floats past the last row, as the `padded` flag requires
    def padded_like(x):
        return torch.full((x.numel() + 64,), float("nan"), device="cuda")[:x.numel()].view(x.shape)
    hi, lo = padded_like(t), padded_like(t)
    ops.split_tf32(t, hi, lo)
    return hi, lo


@pytest.mark.parametrize("padded", [0, 3])
@pytest.mark.parametrize("a_k", [True, False])
@pytest.mark.parametrize("b_k", [True, False])
def test_gemm_split_all_majors_with_mask_and_split_out(cuda_device, a_k, b_k, padded):
    """M = 520 and N = 300 are not multiples of 32: MN-major operands take the
    per-chunk copies (padded = 0) or whole chunks reading the NaN padding past
    the last row (padded = 3), which must not reach any stored output."""
    M, K, N = 520, 392, 300
    g = torch.Generator("cuda").manual_seed(3)
    A = torch.randn(M, K, device="cuda", generator=g)          # logical A[m, k]
    B = torch.randn(K, N, device="cuda", generator=g)          # logical B[k, n]
    bias = torch.randn(N, device="cuda", generator=g)
    mask = torch.randn(M, N, device="cuda", generator=g)
    a_st = A.contiguous() if a_k else A.t().contiguous()       # stored per majorness
    b_st = B.t().contiguous() if b_k else B.contiguous()
    ah, al = _split(a_st)
    bh, bl = _split(b_st)
    c = torch.empty(M, N, device="cuda")
    ch, cl = torch.empty_like(c), torch.empty_like(c)
    ops.gemm_split(ah, al, K if a_k else M, a_k, bh, bl, K if b_k else N, b_k, M, K, N, c=c,
                   c_hi=ch, c_lo=cl, bias=bias, mask=mask, ldm=N, padded=padded)
    torch.cuda.synchronize()
    ref = (A.double() @ B.double() + bias.double()[None, :]) * (mask > 0)
    scale = A.double().abs() @ B.double().abs() + bias.double().abs()[None, :]
    err = float(((c.double() - ref).abs() / scale).max())
    assert err <= 1e-5 * math.sqrt(K)
    assert torch.equal(ch, _rna_tf32(c))
    assert torch.equal(cl, _rna_tf32(c - ch))


def _problem(dims, batch, seed):
    rng = np.random.default_rng(seed)
    ws = [((rng.random((dims[i], dims[i + 1]), dtype=np.float32) * 2 - 1) *
           np.float32(np.sqrt(6.0 / dims[i]))).astype(np.float32) for i in range(len(dims) - 1)]
    bs = [rng.standard_normal(dims[i + 1], dtype=np.float32) * np.float32(0.1)
          for i in range(len(dims) - 1)]
    x = rng.standard_normal((batch, dims[0]), dtype=np.float32)
    y = rng.integers(0, dims[-1], batch).astype(np.float32)
    return ws, bs, x, y


@pytest.mark.parametrize("layout", ["nn", "nt"])
def test_split_step_bit_identical_to_per_call_3xtf32(cuda_device, layout):
    dims = [1024, 512, 256, 128]
    ws, bs, x, y = _problem(dims, 384, 7)
    if layout == "nt":
        ws = [np.ascontiguousarray(w.T) for w in ws]
    X, Y = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    fused = nn.MLP(dims, ws, bs, layout=layout, precision="3xtf32")
    plain = nn.MLP(dims, ws, bs, layout=layout, precision="3xtf32", fused=False)
    assert fused.fused and not plain.fused
    for _ in range(3):
        lf = fused.step(X, Y).clone()
        lp = plain.step(X, Y).clone()
    torch.cuda.synchronize()
    assert torch.equal(lf, lp)
    assert torch.equal(fused.params, plain.params)
    assert torch.equal(fused.grads, plain.grads)
