"""Device ops of the matmul path, called through the C ABI.

torch is used only for device memory and streams: every function here takes
CUDA float32 tensors, passes their raw pointers and the current torch stream
to ``libmxgemm.so`` and lets the library's kernels do the work.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import PRECISIONS, check

_ctx_cache: dict[tuple, int] = {}


def context(device: int | None = None, mode: str = "default") -> int:
    """The library context (the ABI's ``handle``) for a device and precision
    mode, created once.  A context in "nparray" mode also runs the
    training-step ops in the NpArray CPU order (bit-identical results)."""
    if device is None:
        device = torch.cuda.current_device()
    key = (int(device), mode)
    h = _ctx_cache.get(key)
    if h is None:
        h = _lib.lib().mx_context_create(int(device))
        if not h:
            raise _lib.MXError(_lib.MX_ERR_NO_DEVICE, f"mx_context_create({device})")
        if mode != "default":
            check(_lib.lib().mx_context_set_precision(h, _prec(mode)), "mx_context_set_precision")
        _ctx_cache[key] = h
    return h


def new_context(device: int, mode: str = "default") -> int:
    """A context owned by the caller (not shared through `context`); free it
    with `destroy_context`."""
    h = _lib.lib().mx_context_create(int(device))
    if not h:
        raise _lib.MXError(_lib.MX_ERR_NO_DEVICE, f"mx_context_create({device})")
    if mode != "default":
        check(_lib.lib().mx_context_set_precision(h, _prec(mode)), "mx_context_set_precision")
    return h


def destroy_context(h) -> None:
    if h:
        _lib.lib().mx_context_destroy(h)


def set_sm_budget(ctx, sms: int) -> None:
    """SMs the context's tensor-core GEMMs prefer (0 = all); a launch takes
    every SM when that finishes it more than 3 % sooner."""
    check(_lib.lib().mx_context_set_sm_budget(ctx, int(sms)), "mx_context_set_sm_budget")


def set_sm_limit(ctx, sms: int) -> None:
    """Hard cap on the SMs of the context's tensor-core GEMMs (0 = none)."""
    check(_lib.lib().mx_context_set_sm_limit(ctx, int(sms)), "mx_context_set_sm_limit")


def _handle(ctx, t: torch.Tensor) -> int:
    return ctx if ctx is not None else context(t.device.index)


def _prec(precision) -> int:
    if isinstance(precision, str):
        return PRECISIONS[precision]
    return int(precision)


def _stream_ptr(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _check_tensor(t: torch.Tensor, name: str, numel: int | None = None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if numel is not None and t.numel() < numel:
        raise ValueError(f"{name} has {t.numel()} elements, needs {numel}")


def matmul(a: torch.Tensor, b: torch.Tensor, M: int, K: int, N: int, ta: bool = False,
           tb: bool = False, alpha: float = 1.0, beta: float = 0.0,
           out: torch.Tensor | None = None, precision="default", stream=None,
           ctx=None) -> torch.Tensor:
    """C[M,N] = alpha op(A) op(B) + beta C (the reference's cuda_matmul)."""
    _check_tensor(a, "a", M * K)
    _check_tensor(b, "b", K * N)
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=torch.float32)
    _check_tensor(out, "out", M * N)
    rc = _lib.lib().moonbit_cuda_matmul_ex(
        _handle(ctx, a), a.data_ptr(), b.data_ptr(), out.data_ptr(), M, K, N, int(ta),
        int(tb), float(alpha), float(beta), _stream_ptr(stream), _prec(precision))
    check(rc, "moonbit_cuda_matmul_ex")
    return out


def gemm(a: torch.Tensor, b: torch.Tensor, M: int, K: int, N: int, ta: bool = False,
         tb: bool = False, alpha: float = 1.0, beta: float = 0.0,
         bias: torch.Tensor | None = None, relu: bool = False,
         out: torch.Tensor | None = None, precision="default", stream=None,
         lda: int = 0, ldb: int = 0, ldc: int = 0, ctx=None) -> torch.Tensor:
    """C = act(alpha op(A) op(B) + beta C + bias) for any layout (mx_gemm_ex)."""
    _check_tensor(a, "a", M * K if not lda else 1)
    _check_tensor(b, "b", K * N if not ldb else 1)
    if bias is not None:
        _check_tensor(bias, "bias", N)
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=torch.float32)
    _check_tensor(out, "out", M * N if not ldc else 1)
    rc = _lib.lib().mx_gemm_ex(
        _handle(ctx, a), a.data_ptr(), b.data_ptr(), out.data_ptr(),
        bias.data_ptr() if bias is not None else None, M, K, N, int(ta), int(tb), int(lda),
        int(ldb), int(ldc), float(alpha), float(beta), int(relu), _stream_ptr(stream),
        _prec(precision))
    check(rc, "mx_gemm_ex")
    return out


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, relu: bool = False,
           transpose_w: bool = False, out: torch.Tensor | None = None, alpha: float = 1.0,
           precision="default", stream=None, ctx=None) -> torch.Tensor:
    """y = act(alpha x op(w) + bias): w is [K,N] (transpose_w=False) or [N,K]."""
    M, K = x.shape
    N = w.shape[0] if transpose_w else w.shape[1]
    _check_tensor(x, "x")
    _check_tensor(w, "w", K * N)
    if bias is not None:
        _check_tensor(bias, "bias", N)
    if out is None:
        out = torch.empty((M, N), device=x.device, dtype=torch.float32)
    _check_tensor(out, "out", M * N)
    rc = _lib.lib().moonbit_cuda_linear_fwd_ex(
        _handle(ctx, x), x.data_ptr(), w.data_ptr(),
        bias.data_ptr() if bias is not None else None, out.data_ptr(), M, K, N,
        int(transpose_w), int(relu), float(alpha), _stream_ptr(stream), _prec(precision))
    check(rc, "moonbit_cuda_linear_fwd_ex")
    return out


def linear_bias_first(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, relu: bool = True,
                      transpose_w: bool = True, out: torch.Tensor | None = None,
                      pre: torch.Tensor | None = None, stream=None, ctx=None):
    """The reference's fused_linear(_relu) (nparray/fused_ops.mbt:12-78): the
    sum starts from the bias, NpArray rounding order; returns (y, pre)."""
    M, K = x.shape
    N = w.shape[0] if transpose_w else w.shape[1]
    _check_tensor(x, "x")
    _check_tensor(w, "w", K * N)
    _check_tensor(bias, "bias", N)
    if out is None:
        out = torch.empty((M, N), device=x.device, dtype=torch.float32)
    _check_tensor(out, "out", M * N)
    if pre is not None:
        _check_tensor(pre, "pre", M * N)
    rc = _lib.lib().mx_linear_fwd_bias_first(
        _handle(ctx, x), x.data_ptr(), w.data_ptr(), bias.data_ptr(), out.data_ptr(),
        pre.data_ptr() if pre is not None else None, M, K, N, int(transpose_w), int(relu),
        _stream_ptr(stream))
    check(rc, "mx_linear_fwd_bias_first")
    return out, pre


def relu_backward(grad_out: torch.Tensor, saved: torch.Tensor, out: torch.Tensor | None = None,
                  stream=None, ctx=None) -> torch.Tensor:
    _check_tensor(grad_out, "grad_out")
    _check_tensor(saved, "saved", grad_out.numel())
    if out is None:
        out = torch.empty_like(grad_out)
    _check_tensor(out, "out", grad_out.numel())
    rc = _lib.lib().mx_relu_backward(_handle(ctx, grad_out), grad_out.data_ptr(),
                                     saved.data_ptr(), out.data_ptr(), grad_out.numel(),
                                     _stream_ptr(stream))
    check(rc, "mx_relu_backward")
    return out


def reduce_sum_leading(x: torch.Tensor, out: torch.Tensor | None = None,
                       stream=None, ctx=None) -> torch.Tensor:
    """Column sums of a [rows, cols] tensor (the bias gradient)."""
    rows, cols = x.shape
    _check_tensor(x, "x")
    if out is None:
        out = torch.empty((cols,), device=x.device, dtype=torch.float32)
    _check_tensor(out, "out", cols)
    rc = _lib.lib().mx_reduce_sum_leading(_handle(ctx, x), x.data_ptr(), out.data_ptr(),
                                          cols, rows, _stream_ptr(stream))
    check(rc, "mx_reduce_sum_leading")
    return out


def softmax_ce_labels(logits: torch.Tensor, labels: torch.Tensor, denom: int | None = None,
                      grad: torch.Tensor | None = None, loss: torch.Tensor | None = None,
                      want_grad: bool = True, stream=None, ctx=None):
    """(loss[1], dlogits) of mean cross-entropy with float class labels."""
    B, C = logits.shape
    _check_tensor(logits, "logits")
    _check_tensor(labels, "labels", B)
    if loss is None:
        loss = torch.empty((1,), device=logits.device, dtype=torch.float32)
    if want_grad and grad is None:
        grad = torch.empty_like(logits)
    rc = _lib.lib().mx_softmax_ce_labels(
        _handle(ctx, logits), logits.data_ptr(), labels.data_ptr(),
        grad.data_ptr() if want_grad else None, loss.data_ptr(), B, C,
        B if denom is None else int(denom), _stream_ptr(stream))
    check(rc, "mx_softmax_ce_labels")
    return loss, grad


def sgd_momentum_autoclip(params: torch.Tensor, grads: torch.Tensor, vels: torch.Tensor, lr: float,
                          momentum: float, weight_decay: float, max_grad_norm: float,
                          norm_out: torch.Tensor | None = None, n: int | None = None,
                          stream=None, ctx=None) -> None:
    n = params.numel() if n is None else n
    for t, name in ((params, "params"), (grads, "grads"), (vels, "vels")):
        _check_tensor(t, name, n)
    rc = _lib.lib().mx_sgd_momentum_autoclip(
        _handle(ctx, params), params.data_ptr(), grads.data_ptr(), vels.data_ptr(), n,
        float(lr), float(momentum), float(weight_decay), float(max_grad_norm),
        norm_out.data_ptr() if norm_out is not None else None, _stream_ptr(stream))
    check(rc, "mx_sgd_momentum_autoclip")


# ---------------------------------------------------------------- split form
def _ptr(t):
    return t.data_ptr() if t is not None else None


def split_tf32(src: torch.Tensor, hi: torch.Tensor, lo: torch.Tensor | None, ctx=None,
               stream=None) -> None:
    """hi/lo 3xTF32 split of a row-major 2-D (or flat, as one row) tensor."""
    _check_tensor(src, "src")
    rows, cols = (src.shape[0], src.shape[1]) if src.dim() == 2 else (1, src.numel())
    rc = _lib.lib().mx_split_tf32(_handle(ctx, src), src.data_ptr(), rows, cols, cols,
                                  hi.data_ptr(), _ptr(lo), cols, _stream_ptr(stream))
    check(rc, "mx_split_tf32")


def gemm_split(a_hi, a_lo, lda: int, a_kmajor: bool, b_hi, b_lo, ldb: int, b_kmajor: bool,
               M: int, K: int, N: int, c=None, c_hi=None, c_lo=None, ldc: int | None = None,
               alpha: float = 1.0, beta: float = 0.0, bias=None, relu: bool = False,
               mask=None, ldm: int = 0, passes: int = 3, padded: int = 0, ctx=None,
               stream=None, colsum=None, colsum_scratch=None) -> None:
    """tcgen05 GEMM on split operands (mx_gemm_split_ex); see the header.
    padded: bit 0 / bit 1 when A / B copies have 32 readable floats past
    their last row.  colsum: also write the column sums of the stored output
    (mx_gemm_split_colsum_ex; colsum_scratch holds colsum_scratch_bytes)."""
    ref = c if c is not None else c_hi
    args = (_handle(ctx, a_hi), a_hi.data_ptr(), _ptr(a_lo), lda, int(a_kmajor), b_hi.data_ptr(),
            _ptr(b_lo), ldb, int(b_kmajor), _ptr(c), _ptr(c_hi), _ptr(c_lo),
            N if ldc is None else ldc, M, K, N, float(alpha), float(beta), _ptr(bias), int(relu),
            _ptr(mask), ldm, passes, int(padded))
    if colsum is None:
        rc = _lib.lib().mx_gemm_split_ex(*args, _stream_ptr(stream))
        check(rc, "mx_gemm_split_ex")
    else:
        rc = _lib.lib().mx_gemm_split_colsum_ex(
            *args, colsum.data_ptr(), colsum_scratch.data_ptr(),
            colsum_scratch.numel() * colsum_scratch.element_size(), _stream_ptr(stream))
        check(rc, "mx_gemm_split_colsum_ex")
    return ref


def gemm_colsum_scratch_bytes(M: int, N: int) -> int:
    return int(_lib.lib().mx_gemm_colsum_scratch_bytes(M, N))


def _split_gemm(a_hi, a_lo, lda: int, a_kmajor: bool, b_hi, b_lo, ldb: int, b_kmajor: bool,
                M: int, K: int, N: int, c=None, c_hi=None, c_lo=None, ldc: int | None = None,
                alpha: float = 1.0, beta: float = 0.0, bias=None, relu: bool = False,
                mask=None, ldm: int = 0, padded: int = 0, colsum=None, colsum_scratch=None):
    g = _lib.SplitGemm()
    g.a_hi, g.a_lo, g.lda, g.a_kmajor = a_hi.data_ptr(), _ptr(a_lo), lda, int(a_kmajor)
    g.b_hi, g.b_lo, g.ldb, g.b_kmajor = b_hi.data_ptr(), _ptr(b_lo), ldb, int(b_kmajor)
    g.c, g.c_hi, g.c_lo = _ptr(c), _ptr(c_hi), _ptr(c_lo)
    g.ldc = N if ldc is None else ldc
    g.M, g.K, g.N, g.alpha, g.beta = M, K, N, float(alpha), float(beta)
    g.bias, g.relu, g.mask, g.ldm, g.flags = _ptr(bias), int(relu), _ptr(mask), ldm, int(padded)
    if colsum is not None:
        g.colsum, g.colsum_scratch = colsum.data_ptr(), colsum_scratch.data_ptr()
        g.colsum_scratch_bytes = colsum_scratch.numel() * colsum_scratch.element_size()
    return g


def gemm_split_pair(g0: dict, g1: dict, ctx=None, stream=None) -> None:
    """Two independent 3xTF32 split-operand GEMMs in one launch
    (mx_gemm_split_pair): each dict holds gemm_split's keyword arguments
    (a_hi ... colsum_scratch; passes is always 3)."""
    s0, s1 = _split_gemm(**g0), _split_gemm(**g1)
    rc = _lib.lib().mx_gemm_split_pair(_handle(ctx, g0["a_hi"]), ctypes.byref(s0),
                                       ctypes.byref(s1), _stream_ptr(stream))
    check(rc, "mx_gemm_split_pair")


def split_plan(M: int, N: int, K: int, passes: int = 3, ctx=None, device: int | None = None):
    """The work split the context's tcgen05 GEMM picks for M x N x K
    (mx_tc_split_plan): dict of mode (0 whole tiles, 1 stream-K, 2 tail
    split), tile0, r, kp, s, j."""
    out = (ctypes.c_int32 * 6)()
    h = ctx if ctx is not None else context(device)
    check(_lib.lib().mx_tc_split_plan(h, M, N, K, passes, out), "mx_tc_split_plan")
    return dict(zip(("mode", "tile0", "r", "kp", "s", "j"), (int(v) for v in out)))


def softmax_ce_colsum_scratch_bytes(batch: int, C: int) -> int:
    """0 when C is too large for the fused column sums."""
    return int(_lib.lib().mx_softmax_ce_colsum_scratch_bytes(batch, C))


def softmax_ce_labels_split(logits, labels, grad, g_hi, g_lo, loss, denom: int, ctx=None,
                            stream=None, colsum=None, colsum_scratch=None) -> None:
    """CE forward+backward writing the gradient and its split copy; with
    colsum, also the gradient's column sums (the output layer's bias
    gradient, mx_softmax_ce_labels_split_colsum)."""
    B, C = logits.shape
    if colsum is None:
        rc = _lib.lib().mx_softmax_ce_labels_split(
            _handle(ctx, logits), logits.data_ptr(), labels.data_ptr(), grad.data_ptr(),
            g_hi.data_ptr(), g_lo.data_ptr(), _ptr(loss), B, C, int(denom), _stream_ptr(stream))
        check(rc, "mx_softmax_ce_labels_split")
    else:
        rc = _lib.lib().mx_softmax_ce_labels_split_colsum(
            _handle(ctx, logits), logits.data_ptr(), labels.data_ptr(), grad.data_ptr(),
            g_hi.data_ptr(), g_lo.data_ptr(), _ptr(loss), B, C, int(denom), colsum.data_ptr(),
            colsum_scratch.data_ptr(), colsum_scratch.numel() * colsum_scratch.element_size(),
            _stream_ptr(stream))
        check(rc, "mx_softmax_ce_labels_split_colsum")


def sgd_momentum_autoclip_split(params, grads, vels, p_hi, p_lo, lr, momentum, weight_decay,
                                max_grad_norm, norm_out=None, ctx=None, stream=None) -> None:
    n = params.numel()
    rc = _lib.lib().mx_sgd_momentum_autoclip_split(
        _handle(ctx, params), params.data_ptr(), grads.data_ptr(), vels.data_ptr(), n,
        float(lr), float(momentum), float(weight_decay), float(max_grad_norm), _ptr(norm_out),
        p_hi.data_ptr(), p_lo.data_ptr(), _stream_ptr(stream))
    check(rc, "mx_sgd_momentum_autoclip_split")


def sum_squares(x, out, accumulate: bool = False, ctx=None, stream=None) -> None:
    """out[0] = (out[0] if accumulate else 0) + sum(x**2) (mx_sum_squares)."""
    rc = _lib.lib().mx_sum_squares(_handle(ctx, out), _ptr(x), x.numel(), out.data_ptr(),
                                   int(accumulate), _stream_ptr(stream))
    check(rc, "mx_sum_squares")


def sgd_momentum_clip(params, grads, vels, lr, momentum, weight_decay, max_grad_norm, norm_sq,
                      ctx=None, stream=None) -> None:
    """Momentum-SGD update of one range clipped by sqrt(norm_sq[0])
    (mx_sgd_momentum_clip)."""
    n = params.numel()
    rc = _lib.lib().mx_sgd_momentum_clip(
        _handle(ctx, params), params.data_ptr(), grads.data_ptr(), vels.data_ptr(), n,
        float(lr), float(momentum), float(weight_decay), float(max_grad_norm),
        norm_sq.data_ptr(), _stream_ptr(stream))
    check(rc, "mx_sgd_momentum_clip")


def status(device: int | None = None) -> tuple[int, int]:
    """(status, call site) of the device status word; synchronises, clears it."""
    return context_status(context(device))


def context_status(ctx) -> tuple[int, int]:
    """(status, call site) of one context's status word (mx_context_status):
    synchronises the context's device, clears the word."""
    where = ctypes.c_int32(0)
    rc = _lib.lib().mx_context_status(ctx, ctypes.byref(where))
    return rc, where.value


def reserve_workspace(nbytes: int, device: int | None = None) -> None:
    check(_lib.lib().mx_context_reserve_workspace(context(device), int(nbytes)),
          "mx_context_reserve_workspace")


def workspace_bytes(M: int, K: int, N: int, ta=False, tb=False, precision="default",
                    device: int | None = None) -> int:
    return int(_lib.lib().mx_matmul_workspace_bytes(context(device), M, K, N, int(ta), int(tb),
                                                    _prec(precision)))


def resolve_precision(M: int, K: int, N: int, precision="default",
                      device: int | None = None) -> str:
    p = _lib.lib().mx_matmul_resolve_precision(context(device), M, K, N, _prec(precision))
    return {v: k for k, v in PRECISIONS.items()}[p]
