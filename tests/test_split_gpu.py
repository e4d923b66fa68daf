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


@pytest.mark.parametrize("M,K,N,a_k,b_k,branch", [
    (1024, 16384, 4096, True, True, "tails"),    # 128 tiles on 148 SMs: 7 tails per helper
    (4096, 2048, 4096, False, False, "pieces"),  # 3 full waves + 68 tiles: one piece each
    (1152, 8192, 2304, True, False, "tails"),    # 81 tiles on 148 SMs: 2 tails per helper
])
def test_tail_split_waves(cuda_device, M, K, N, a_k, b_k, branch):
    """Shapes whose last wave of tiles is part-filled, with K deep enough
    for the split to pay, run the tail split (the remainder tiles' first
    k-blocks on their own CTAs, the rest on the idle ones, parts summed in k
    order by the last to finish): fp32-class against fp64, bit-identical run
    to run, with the fused column sums and mask."""
    plan = ops.split_plan(M, N, K)
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("tile counts chosen for 148 SMs")
    assert plan["mode"] == 2 and (plan["s"] > 0) == (branch == "pieces"), plan
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


def test_split_plan_skips_unprofitable_tails(cuda_device):
    """A part-filled last wave whose split would save fewer k-blocks than
    the partial tiles cost runs whole tiles: the 1024-row layers of the
    wide MLP (128 tiles of K = 4096 or 1000 on 148 SMs)."""
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("tile counts chosen for 148 SMs")
    for M, N, K in ((1024, 4096, 4096), (1024, 4096, 1000), (4096, 1000, 1024),
                    (4096, 4096, 1024)):
        assert ops.split_plan(M, N, K)["mode"] == 0, (M, N, K)


def _layer_backward(B, fi, fo, nt, seed):
    """Operands of one Linear layer's backward in split form, as the MLP step
    holds them: dY [B, fo], activation h [B, fi] (ReLU mask), weights
    (nn: [fi, fo], nt: [fo, fi]); the keyword arguments of the dX and dW
    GEMMs and their fp64 references."""
    g = torch.Generator("cuda").manual_seed(seed)
    dY = torch.randn(B, fo, device="cuda", generator=g)
    h = torch.randn(B, fi, device="cuda", generator=g)
    W = torch.randn(fo, fi, device="cuda", generator=g) if nt else \
        torch.randn(fi, fo, device="cuda", generator=g)
    gh, gl = _split(dY)
    hh, hl = _split(h)
    wh, wl = _split(W)
    out = dict(dx=torch.empty(B, fi, device="cuda"), dx_hi=torch.empty(B, fi, device="cuda"),
               dx_lo=torch.empty(B, fi, device="cuda"), cs=torch.empty(fi, device="cuda"),
               dw=torch.empty(*((fo, fi) if nt else (fi, fo)), device="cuda"),
               scratch=torch.empty(ops.gemm_colsum_scratch_bytes(B, fi) // 4, device="cuda"))
    dx_kw = dict(a_hi=gh, a_lo=gl, lda=fo, a_kmajor=True, b_hi=wh, b_lo=wl,
                 ldb=fi if nt else fo, b_kmajor=not nt, M=B, K=fo, N=fi, c=out["dx"],
                 c_hi=out["dx_hi"], c_lo=out["dx_lo"], mask=h, ldm=fi, colsum=out["cs"],
                 colsum_scratch=out["scratch"], padded=3)
    if nt:   # dW[out, in] = dY^T h
        dw_kw = dict(a_hi=gh, a_lo=gl, lda=fo, a_kmajor=False, b_hi=hh, b_lo=hl, ldb=fi,
                     b_kmajor=False, M=fo, K=B, N=fi, c=out["dw"], padded=3)
    else:    # dW[in, out] = h^T dY
        dw_kw = dict(a_hi=hh, a_lo=hl, lda=fi, a_kmajor=False, b_hi=gh, b_lo=gl, ldb=fo,
                     b_kmajor=False, M=fi, K=B, N=fo, c=out["dw"], padded=3)
    Wt = W.double() if nt else W.double().t()           # [fo, fi]
    dx_ref = (dY.double() @ Wt) * (h > 0)
    dx_scale = (dY.double().abs() @ Wt.abs())
    dw_ref = dY.double().t() @ h.double() if nt else h.double().t() @ dY.double()
    dw_scale = dY.double().abs().t() @ h.double().abs() if nt else \
        h.double().abs().t() @ dY.double().abs()
    return dx_kw, dw_kw, out, (dx_ref, dx_scale, dw_ref, dw_scale)


@pytest.mark.parametrize("B,fi,fo,nt", [
    (1024, 4096, 4096, False),   # the wide MLP's hidden layer at 8 GPUs (1024 rows each)
    (1024, 4096, 1000, False),   # ... and its output layer
    (8192, 1024, 512, False),    # dW with the longer tiles: it goes first
    (200, 300, 132, False),      # ragged: partial tiles in every dimension
    (200, 300, 132, True),
    (512, 1024, 1024, True),
])
def test_gemm_split_pair_matches_two_launches(cuda_device, B, fi, fo, nt):
    """mx_gemm_split_pair (a layer's dX and dW in one launch) against the
    same two GEMMs launched one by one: bit-identical when the single
    launches also run whole tiles, and fp32-class against fp64 always --
    the masked dX with its split copies and column sums, and dW."""
    dx_kw, dw_kw, out, (dx_ref, dx_scale, dw_ref, dw_scale) = _layer_backward(B, fi, fo, nt, B + fi)
    ops.gemm_split_pair(dx_kw, dw_kw)
    paired = {k: v.clone() for k, v in out.items() if k != "scratch"}
    ops.gemm_split(**dx_kw)
    ops.gemm_split(**dw_kw)
    torch.cuda.synchronize()
    assert ops.context_status(ops.context(0))[0] == 0
    whole = ops.split_plan(B, fi, fo)["mode"] == 0 and \
        ops.split_plan(dw_kw["M"], dw_kw["N"], B)["mode"] == 0
    if whole:
        for k, v in paired.items():
            assert torch.equal(v, out[k]), k
    tol = 1e-5
    assert float(((paired["dx"].double() - dx_ref).abs() / dx_scale.clamp_min(1e-30)).max()) \
        <= tol * math.sqrt(fo)
    assert float(((paired["dw"].double() - dw_ref).abs() / dw_scale).max()) <= tol * math.sqrt(B)
    assert torch.equal(paired["dx_hi"], _rna_tf32(paired["dx"]))
    assert torch.equal(paired["dx_lo"], _rna_tf32(paired["dx"] - paired["dx_hi"]))
    want = paired["dx"].double().sum(0)
    assert float(((paired["cs"].double() - want).abs() /
                  paired["dx"].double().abs().sum(0).clamp_min(1e-30)).max()) <= 1e-6 * math.sqrt(B)


def test_sm_budget_is_a_preference(cuda_device):
    """With 128 of 148 SMs preferred, a GEMM whose tiles make whole 128-SM
    waves keeps to the budget (whole tiles), while one that all SMs finish
    clearly sooner (512 tiles: 3 waves and a split instead of 4 waves) takes
    them, with its tail split."""
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("tile counts chosen for 148 SMs")
    ctx = ops.new_context(0)
    try:
        ops.set_sm_budget(ctx, 128)
        assert ops.split_plan(1024, 4096, 4096, ctx=ctx)["mode"] == 0
        assert ops.split_plan(4096, 4096, 4096, ctx=ctx)["mode"] == 2
        # and the GEMM computes the same either way
        M = K = N = 2048
        g = torch.Generator("cuda").manual_seed(5)
        A = torch.randn(M, K, device="cuda", generator=g)
        B = torch.randn(K, N, device="cuda", generator=g)
        ah, al = _split(A)
        bh, bl = _split(B)
        c = torch.empty(M, N, device="cuda")
        ops.gemm_split(ah, al, K, True, bh, bl, N, False, M, K, N, c=c, padded=3, ctx=ctx)
        torch.cuda.synchronize()
        assert ops.context_status(ctx)[0] == 0
        ref = A.double() @ B.double()
        scale = A.double().abs() @ B.double().abs()
        assert float(((c.double() - ref).abs() / scale).max()) <= 1e-5 * math.sqrt(K)
    finally:
        ops.destroy_context(ctx)


def test_sm_limit_is_hard(cuda_device):
    """mx_context_set_sm_limit caps the SMs whatever the cost model prefers:
    the 512-tile GEMM that takes all 148 SMs under a 128-SM preference runs
    four whole waves on 128 under a 128-SM limit, with the same result."""
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("tile counts chosen for 148 SMs")
    M = K = N = 4096
    g = torch.Generator("cuda").manual_seed(6)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(K, N, device="cuda", generator=g)
    ah, al = _split(A)
    bh, bl = _split(B)
    outs = []
    for limit in (0, 128):
        ctx = ops.new_context(0)
        try:
            ops.set_sm_budget(ctx, 128)
            ops.set_sm_limit(ctx, limit)
            assert ops.split_plan(M, N, K, ctx=ctx)["mode"] == (2 if limit == 0 else 0)
            c = torch.empty(M, N, device="cuda")
            ops.gemm_split(ah, al, K, True, bh, bl, N, False, M, K, N, c=c, padded=3, ctx=ctx)
            torch.cuda.synchronize()
            assert ops.context_status(ctx)[0] == 0
            outs.append(c)
        finally:
            ops.destroy_context(ctx)
    ref = A.double() @ B.double()
    scale = A.double().abs() @ B.double().abs()
    for c in outs:
        assert float(((c.double() - ref).abs() / scale).max()) <= 1e-5 * math.sqrt(K)
