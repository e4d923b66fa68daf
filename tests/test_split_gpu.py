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


@pytest.mark.parametrize("padded", [0, 3])
def test_gemm_split_colsum_is_the_bias_gradient(cuda_device, padded):
    """The fused column sums equal the fp64 column sums of the stored output
    (after bias, ReLU and mask, rows past M excluded), are bit-identical run
    to run, and leave the arrival counters ready for the next launch."""
    M, K, N = 1000, 392, 300   # partial tiles in both directions
    g = torch.Generator("cuda").manual_seed(4)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(K, N, device="cuda", generator=g)
    mask = torch.randn(M, N, device="cuda", generator=g)
    ah, al = _split(A.contiguous())
    bh, bl = _split(B.t().contiguous())
    c = torch.empty(M, N, device="cuda")
    scratch = torch.empty(ops.gemm_colsum_scratch_bytes(M, N) // 4, device="cuda")
    sums = []
    for _ in range(3):
        cs = torch.full((N,), float("nan"), device="cuda")
        ops.gemm_split(ah, al, K, True, bh, bl, K, True, M, K, N, c=c, mask=mask, ldm=N,
                       padded=padded, colsum=cs, colsum_scratch=scratch)
        sums.append(cs)
    torch.cuda.synchronize()
    want = c.double().sum(0)
    scale = c.double().abs().sum(0)
    err = float(((sums[0].double() - want).abs() / scale.clamp_min(1e-30)).max())
    assert err <= 1e-6 * math.sqrt(M), err
    assert torch.equal(sums[0], sums[1]) and torch.equal(sums[1], sums[2])


def test_softmax_ce_colsum_is_the_bias_gradient(cuda_device):
    B, C = 1000, 1000   # the last block and the last group are partial
    g = torch.Generator("cuda").manual_seed(5)
    logits = torch.randn(B, C, device="cuda", generator=g) * 3
    labels = torch.randint(0, C, (B,), device="cuda", generator=g).float()
    grad, gh, gl = (torch.empty(B, C, device="cuda") for _ in range(3))
    loss = torch.empty(1, device="cuda")
    scratch = torch.empty(ops.softmax_ce_colsum_scratch_bytes(B, C) // 4, device="cuda")
    out = []
    for _ in range(2):
        cs = torch.full((C,), float("nan"), device="cuda")
        ops.softmax_ce_labels_split(logits, labels, grad, gh, gl, loss, 4096, colsum=cs,
                                    colsum_scratch=scratch)
        out.append(cs)
    torch.cuda.synchronize()
    want = grad.double().sum(0)
    scale = grad.double().abs().sum(0)
    assert float(((out[0].double() - want).abs() / scale).max()) <= 1e-6 * math.sqrt(B)
    assert torch.equal(out[0], out[1])
    p = torch.softmax(logits.double(), 1)
    ref = (p - torch.nn.functional.one_hot(labels.long(), C).double()) / 4096
    assert float((grad.double() - ref).abs().max()) <= 1e-9
    assert ops.softmax_ce_colsum_scratch_bytes(B, 5000) == 0  # too wide to fuse


@pytest.mark.parametrize("layout", ["nn", "nt"])
def test_split_step_matches_per_call_3xtf32(cuda_device, layout):
    """The split-form step runs the same 3xTF32 GEMMs as the per-call path, so
    the loss and every weight gradient are bit-identical; its bias gradients
    come from the fused column sums (another fixed summation order than the
    separate reduction), so they agree to fp32 rounding of the column sums."""
    dims = [1024, 512, 256, 128]
    ws, bs, x, y = _problem(dims, 384, 7)
    if layout == "nt":
        ws = [np.ascontiguousarray(w.T) for w in ws]
    X, Y = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    fused = nn.MLP(dims, ws, bs, layout=layout, precision="3xtf32")
    plain = nn.MLP(dims, ws, bs, layout=layout, precision="3xtf32", fused=False)
    assert fused.fused and not plain.fused
    lf = fused.step(X, Y, update=False).clone()
    lp = plain.step(X, Y, update=False).clone()
    torch.cuda.synchronize()
    assert torch.equal(lf, lp)
    gbuf = plain._buffers(384)[1]
    for i in range(len(dims) - 1):
        assert torch.equal(fused.gw[i], plain.gw[i])
        dy = gbuf[i].double()
        want, scale = dy.sum(0), dy.abs().sum(0).clamp_min(1e-30)
        for m in (fused, plain):
            assert float(((m.gb[i].double() - want).abs() / scale).max()) <= 1e-6 * math.sqrt(384)
    # and the training runs stay together over several steps
    for _ in range(3):
        lf = fused.step(X, Y).clone()
        lp = plain.step(X, Y).clone()
    torch.cuda.synchronize()
    assert abs(float(lf) - float(lp)) <= 1e-6
    rel = float((fused.params - plain.params).norm() / plain.params.norm())
    assert rel <= 1e-6


@pytest.mark.parametrize("M,K,N,a_k,b_k", [
    (1024, 4096, 4096, True, True),    # 128 tiles on 148 SMs: whole tails, 7 per helper
    (4096, 1024, 4096, False, False),  # 3 full waves + 68 tiles: one piece per helper
    (1152, 2048, 2304, True, False),   # 81 tiles on 148 SMs: whole tails, 2 per helper
])
def test_tail_split_waves(cuda_device, M, K, N, a_k, b_k):
    """Shapes whose last wave of tiles is part-filled run the tail split (the
    remainder tiles' first k-blocks on their own CTAs, the rest on the idle
    ones, parts summed in k order by the last to finish): fp32-class against
    fp64, bit-identical run to run, with the fused column sums and mask."""
    g = torch.Generator("cuda").manual_seed(M + N)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(K, N, device="cuda", generator=g)
    mask = torch.randn(M, N, device="cuda", generator=g)
    bias = torch.randn(N, device="cuda", generator=g)
    ah, al = _split(A.contiguous() if a_k else A.t().contiguous())
    bh, bl = _split(B.t().contiguous() if b_k else B.contiguous())
    scratch = torch.empty(ops.gemm_colsum_scratch_bytes(M, N) // 4, device="cuda")
    outs = []
    for _ in range(2):
        c = torch.empty(M, N, device="cuda")
        cs = torch.empty(N, device="cuda")
        ops.gemm_split(ah, al, K if a_k else M, a_k, bh, bl, K if b_k else N, b_k, M, K, N, c=c,
                       bias=bias, mask=mask, ldm=N, padded=3, colsum=cs, colsum_scratch=scratch)
        outs.append((c, cs))
    torch.cuda.synchronize()
    (c, cs), (c2, cs2) = outs
    ref = (A.double() @ B.double() + bias.double()[None, :]) * (mask > 0)
    scale = A.double().abs() @ B.double().abs() + bias.double().abs()[None, :]
    assert float(((c.double() - ref).abs() / scale).max()) <= 1e-5 * math.sqrt(K)
    assert torch.equal(c, c2) and torch.equal(cs, cs2)
    want = c.double().sum(0)
    assert float(((cs.double() - want).abs() / c.double().abs().sum(0)).max()) <= \
        1e-6 * math.sqrt(M)
