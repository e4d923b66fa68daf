"""Failure detection on the GPU, without faulting it.

* A bounded in-kernel wait that runs out: a context whose wait limit is set
  to a few microseconds runs a GEMM whose first accumulator takes far longer
  than that to fill, so the epilogue's wait gives up.  The kernel records
  MX_ERR_TIMEOUT and the wait's call site in the context's status word, lets
  the copies and MMAs it already issued finish (under the separate drain
  limit), frees its tensor memory and returns.  The context stays usable: the
  next call with the normal limit is correct.  (The reference aborts the
  process on any failed call, moonxi-net-gpu/tensor/gpu_tensor.mbt:12-16.)
* A label outside [0, C) in the cross-entropy kernels is reported as
  MX_ERR_INVALID with a call site instead of being read out of bounds.
"""
from __future__ import annotations

import math

import pytest
import torch

from moonxi_net_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TC_WAIT_SITES = set(range(201, 209))


def _fresh_context(mode: str | None = None):
    h = _lib.lib().mx_context_create(0)
    assert h
    if mode is not None:
        assert _lib.lib().mx_context_set_precision(h, _lib.PRECISIONS[mode]) == 0
    return h


def _fp64_err(A, B, C):
    c64 = A.double() @ B.double()
    scale = A.double().abs() @ B.double().abs()
    return float(((C.double() - c64).abs() / scale).max())


def test_bounded_wait_times_out_and_context_recovers(cuda_device):
    h = _fresh_context("3xtf32")
    try:
        n = 4096
        g = torch.Generator("cuda").manual_seed(5)
        A = torch.randn((n, n), device="cuda", generator=g)
        B = torch.randn((n, n), device="cuda", generator=g)
        C = torch.zeros((n, n), device="cuda")
        assert _lib.lib().mx_context_set_timeout_ns(h, 5000) == 0  # 5 us
        rc = _lib.lib().moonbit_cuda_matmul_ex(h, A.data_ptr(), B.data_ptr(), C.data_ptr(), n, n,
                                               n, 0, 0, 1.0, 0.0, None, _lib.PREC_3XTF32)
        assert rc == 0  # the launch itself is fine; the wait gives up on the device
        st, where = ops.context_status(h)
        assert st == _lib.MX_ERR_TIMEOUT, st
        assert where in TC_WAIT_SITES, where
        # the word was cleared, the device and the context still work
        assert ops.context_status(h) == (0, 0)
        assert _lib.lib().mx_context_set_timeout_ns(h, 2_000_000_000) == 0
        rc = _lib.lib().moonbit_cuda_matmul_ex(h, A.data_ptr(), B.data_ptr(), C.data_ptr(), n, n,
                                               n, 0, 0, 1.0, 0.0, None, _lib.PREC_3XTF32)
        assert rc == 0
        assert ops.context_status(h) == (0, 0)
        assert _fp64_err(A, B, C) <= 1e-5 * math.sqrt(n)
    finally:
        _lib.lib().mx_context_destroy(h)


def test_zero_wait_limit_is_rejected(cuda_device):
    h = _fresh_context()
    try:
        assert _lib.lib().mx_context_set_timeout_ns(h, 0) == _lib.MX_ERR_INVALID
    finally:
        _lib.lib().mx_context_destroy(h)


@pytest.mark.parametrize("mode,site", [("3xtf32", 301), ("nparray", 302)])
def test_out_of_range_label_is_reported(cuda_device, mode, site):
    h = _fresh_context(mode)
    try:
        B, C = 64, 10
        g = torch.Generator("cuda").manual_seed(9)
        logits = torch.randn((B, C), device="cuda", generator=g)
        labels = torch.randint(0, C, (B,), device="cuda", generator=g).float()
        labels[5] = C        # one past the last class
        labels[17] = -1.0
        loss, grad = ops.softmax_ce_labels(logits, labels, ctx=h)
        st, where = ops.context_status(h)
        assert st == _lib.MX_ERR_INVALID and where == site, (st, where)
        assert math.isnan(float(loss.item()))
        # the valid rows still get the exact gradient (softmax - onehot) / B
        p = torch.softmax(logits.double(), dim=1)
        ok = torch.ones(B, dtype=torch.bool, device="cuda")
        ok[5] = ok[17] = False
        onehot = torch.zeros_like(p)
        onehot[ok] = torch.nn.functional.one_hot(labels[ok].long(), C).double()
        want = (p - onehot) / B
        assert float((grad.double()[ok] - want[ok]).abs().max()) <= 1e-6
        # good labels afterwards: no status
        labels[5], labels[17] = 1.0, 2.0
        loss, _ = ops.softmax_ce_labels(logits, labels, ctx=h)
        assert ops.context_status(h) == (0, 0)
        assert math.isfinite(float(loss.item()))
    finally:
        _lib.lib().mx_context_destroy(h)
