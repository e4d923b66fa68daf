"""TEST INFRASTRUCTURE ONLY: Python access to the CPU oracle.

This module wraps ``oracle/_build/libnporacle.so`` (the C restatement of the
moonxi-net NpArray ops, ``oracle/np_oracle.c``) and adds a tape-order mirror
of one MLP training step on top of it.  Only tests/, ``__graft_entry__.smoke``
and bench.py's CPU-baseline legs import it, and only to check or to time the
reference algorithm.  The product (``moonxi-net_b200``) never imports it.

The MLP step follows the reference autograd exactly:

* forward per layer: ``x.matmul(w).add(b)`` (``model/module.mbt:106-116``,
  weights stored ``[in, out]``) or ``x.matmul(w.transpose()).add(b)``
  (``model/mlp.mbt:16-23``, weights stored ``[out, in]``), then ``relu``
  between layers;
* loss: ``cross_entropy_with_labels`` (``nparray/image_impl.mbt:83-114``);
* backward: the closure tape of ``grad/grad.mbt:73-97`` replayed in reverse,
  with the matmul closures of ``grad/blas.mbt:23-39``, the add closures of
  ``grad/grad.mbt:163-174`` and the relu closure of ``grad/image.mbt:45-61``;
  the first layer's input has no gradient, so its dX GEMM never runs
  (``grad/grad.mbt:80-85``);
* update: ``batch_sgd_momentum_autoclip`` (``nparray/trait_impl.mbt:280-311``)
  over the parameters in ``[w1, b1, w2, b2, ...]`` order.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libnporacle.so")
_REF_LIB_PATH = os.path.join(_HERE, "_ref", "libref_cuda_kernels.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_lib = None


def build() -> str:
    """Compiles the C restatement (gcc, no fast-math) and returns the path."""
    subprocess.check_call(["make", "-s", "-C", _HERE, "all"])
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.np_matmul.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, ctypes.c_int]
        L.np_gemm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.c_int, ctypes.c_int,
                              ctypes.c_float, ctypes.c_float, ctypes.c_int]
        L.np_transpose.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.np_fused_linear.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.np_add_row_bias.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.np_relu.argtypes = [_f32p, _f32p, ctypes.c_int64]
        L.np_relu_backward.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64]
        L.np_reduce_sum_leading.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int]
        L.np_add_into.argtypes = [_f32p, _f32p, ctypes.c_int64]
        L.np_scale.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_float]
        L.np_ce_labels_forward.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int]
        L.np_ce_labels_forward.restype = ctypes.c_float
        L.np_ce_labels_backward.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int]
        L.np_sgd_momentum_autoclip.argtypes = [
            ctypes.POINTER(_f32p), ctypes.POINTER(_f32p), ctypes.POINTER(_f32p),
            ctypes.POINTER(ctypes.c_int64), ctypes.c_int, ctypes.c_float,
            ctypes.c_float, ctypes.c_float, ctypes.c_float]
        L.np_sgd_momentum_autoclip.restype = ctypes.c_float
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_f32p)


def default_threads() -> int:
    return max(1, os.cpu_count() or 1)


# --------------------------------------------------------------------------
# single ops (NpArray semantics)
# --------------------------------------------------------------------------
def matmul(a: np.ndarray, b: np.ndarray, threads: int = 1) -> np.ndarray:
    """NpArray::matmul (nparray/trait_impl.mbt:205-249)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    n, m = a.shape
    m2, p = b.shape
    assert m == m2
    c = np.empty((n, p), np.float32)
    lib().np_matmul(_p(a), _p(b), _p(c), n, m, p, threads)
    return c


def gemm(a, b, M, K, N, ta=0, tb=0, alpha=1.0, beta=0.0, c=None, threads=1):
    """cuda_matmul semantics (cuda_kernels.cu:1444-1499) in NpArray arithmetic."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    out = np.zeros((M, N), np.float32) if c is None else np.array(c, np.float32, copy=True)
    lib().np_gemm(_p(a), _p(b), _p(out), M, K, N, int(ta), int(tb),
                  float(alpha), float(beta), threads)
    return out


def fused_linear(x: np.ndarray, w: np.ndarray, bias: np.ndarray, relu: bool = True,
                 threads: int = 1):
    """fused_linear_relu / fused_linear (nparray/fused_ops.mbt:12-78): w is
    [out, in]; the sum starts from the bias.  Returns (out, pre_relu)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    bias = np.ascontiguousarray(bias, np.float32)
    n, m = x.shape
    p, m2 = w.shape
    assert m == m2 and bias.shape == (p,)
    out = np.empty((n, p), np.float32)
    pre = np.empty((n, p), np.float32)
    lib().np_fused_linear(_p(x), _p(w), _p(bias), _p(out), _p(pre), n, m, p, int(relu), threads)
    return out, pre


def transpose(x: np.ndarray) -> np.ndarray:
    """NpArray::transpose (nparray/trait_impl.mbt:252-261)."""
    x = np.ascontiguousarray(x, np.float32)
    n, m = x.shape
    out = np.empty((m, n), np.float32)
    lib().np_transpose(_p(x), _p(out), n, m)
    return out


def add_row_bias(x: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Broadcast add [rows, cols] + [cols] (nparray/nparray.mbt:32-98)."""
    x = np.ascontiguousarray(x, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    out = np.empty_like(x)
    lib().np_add_row_bias(_p(x), _p(b), _p(out), x.shape[0], x.shape[1])
    return out


def relu(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().np_relu(_p(x), _p(out), x.size)
    return out


def relu_backward(og, x):
    og = np.ascontiguousarray(og, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().np_relu_backward(_p(og), _p(x), _p(out), x.size)
    return out


def reduce_sum_leading(x, threads=1):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty((x.shape[1],), np.float32)
    lib().np_reduce_sum_leading(_p(x), _p(out), x.shape[0], x.shape[1], threads)
    return out


def ce_forward(logits, labels, denom=None):
    logits = np.ascontiguousarray(logits, np.float32)
    labels = np.ascontiguousarray(labels, np.float32)
    b, c = logits.shape
    return float(lib().np_ce_labels_forward(_p(logits), _p(labels), b, c,
                                            b if denom is None else denom))


def ce_backward(logits, labels, denom=None):
    logits = np.ascontiguousarray(logits, np.float32)
    labels = np.ascontiguousarray(labels, np.float32)
    b, c = logits.shape
    out = np.empty_like(logits)
    lib().np_ce_labels_backward(_p(logits), _p(labels), _p(out), b, c,
                                b if denom is None else denom)
    return out


def sgd_momentum_autoclip(params, grads, vels, lr, momentum, wd, max_norm):
    """In-place update of params / vels (lists of float32 arrays)."""
    n = len(params)
    P = (_f32p * n)(*[_p(x) for x in params])
    G = (_f32p * n)(*[_p(x) for x in grads])
    V = (_f32p * n)(*[_p(x) for x in vels])
    S = (ctypes.c_int64 * n)(*[x.size for x in params])
    return float(lib().np_sgd_momentum_autoclip(P, G, V, S, n, lr, momentum, wd,
                                                max_norm))


# --------------------------------------------------------------------------
# MLP training step, tape order of the reference autograd
# --------------------------------------------------------------------------
class MLPOracle:
    """Sequential MLP with ReLU between layers, trained with momentum SGD.

    ``layout="nn"``: weights ``[in, out]``, forward ``x.matmul(w)``
    (``Linear::as_module``).  ``layout="nt"``: weights ``[out, in]``, forward
    ``x.matmul(w.transpose())`` (``MLP::forward``).  Both give the same
    numbers for the same logical weights; the layout only changes which GEMM
    shapes run.
    """

    def __init__(self, weights, biases, layout="nn", lr=0.01, momentum=0.9,
                 weight_decay=1e-4, max_grad_norm=35.0, threads=1):
        self.w = [np.ascontiguousarray(w, np.float32).copy() for w in weights]
        self.b = [np.ascontiguousarray(b, np.float32).copy() for b in biases]
        self.layout = layout
        self.lr, self.momentum = np.float32(lr), np.float32(momentum)
        self.wd, self.max_norm = np.float32(weight_decay), np.float32(max_grad_norm)
        self.vw = [np.zeros_like(w) for w in self.w]
        self.vb = [np.zeros_like(b) for b in self.b]
        self.threads = threads

    def params(self):
        out = []
        for w, b in zip(self.w, self.b):
            out += [w, b]
        return out

    def forward(self, x):
        """Returns (logits, saved pre-activations, saved layer inputs)."""
        h = np.ascontiguousarray(x, np.float32)
        inputs, pre = [], []
        L = len(self.w)
        for i in range(L):
            inputs.append(h)
            wmat = self.w[i] if self.layout == "nn" else transpose(self.w[i])
            z = matmul(h, wmat, self.threads)
            a = add_row_bias(z, self.b[i])
            pre.append(a)
            h = relu(a) if i + 1 < L else a
        return h, pre, inputs

    def loss(self, x, labels, denom=None):
        logits, _, _ = self.forward(x)
        return ce_forward(logits, labels, denom)

    def grads(self, x, labels, denom=None):
        """Loss and parameter gradients (list aligned with params())."""
        logits, pre, inputs = self.forward(x)
        loss = ce_forward(logits, labels, denom)
        g = ce_backward(logits, labels, denom)
        g = np.ascontiguousarray(g * np.float32(1.0))  # raw.scale(og = 1.0)
        L = len(self.w)
        gw, gb = [None] * L, [None] * L
        for i in reversed(range(L)):
            # add closures (grad/grad.mbt:163-174): b <- reduce_sum_to(og)
            gb[i] = reduce_sum_leading(g, self.threads)
            # matmul closures (grad/blas.mbt:35,37): y first, then x
            wmat = self.w[i] if self.layout == "nn" else transpose(self.w[i])
            dw_in_out = matmul(transpose(inputs[i]), g, self.threads)
            gw[i] = dw_in_out if self.layout == "nn" else transpose(dw_in_out)
            if i > 0:
                dx = matmul(g, transpose(wmat), self.threads)
                # relu closure (grad/image.mbt:45-61)
                g = relu_backward(dx, pre[i - 1])
        out = []
        for i in range(L):
            out += [gw[i], gb[i]]
        return loss, out

    def step(self, x, labels, denom=None):
        loss, grads = self.grads(x, labels, denom)
        vels = []
        for vw, vb in zip(self.vw, self.vb):
            vels += [vw, vb]
        sgd_momentum_autoclip(self.params(), grads, vels, self.lr, self.momentum,
                              self.wd, self.max_norm)
        return loss


class MLPFloat64:
    """The same training step as MLPOracle evaluated in float64 with numpy
    (no fp32 rounding anywhere).  Used to measure how far the fp32 oracle's
    own loss curve drifts from exact arithmetic -- the conditioning floor for
    any fp32 implementation that does not reproduce NpArray's operation order."""

    def __init__(self, weights, biases, lr=0.01, momentum=0.9, weight_decay=1e-4,
                 max_grad_norm=35.0):
        self.w = [np.asarray(w, np.float64).copy() for w in weights]   # [in, out]
        self.b = [np.asarray(b, np.float64).copy() for b in biases]
        self.vw = [np.zeros_like(w) for w in self.w]
        self.vb = [np.zeros_like(b) for b in self.b]
        self.lr, self.m, self.wd, self.max_norm = lr, momentum, weight_decay, max_grad_norm

    def step(self, x, labels):
        B = x.shape[0]
        lab = np.asarray(labels).astype(np.int64)
        h, pre = [np.asarray(x, np.float64)], []
        L = len(self.w)
        for i in range(L):
            a = h[-1] @ self.w[i] + self.b[i]
            pre.append(a)
            h.append(np.maximum(a, 0.0) if i + 1 < L else a)
        z = h[-1]
        mx = z.max(1, keepdims=True)
        e = np.exp(z - mx)
        s = e.sum(1, keepdims=True)
        loss = float(np.mean(np.log(s[:, 0]) + mx[:, 0] - z[np.arange(B), lab]))
        g = e / s
        g[np.arange(B), lab] -= 1.0
        g /= B
        gw, gb = [None] * L, [None] * L
        for i in reversed(range(L)):
            gb[i] = g.sum(0)
            gw[i] = h[i].T @ g
            if i > 0:
                g = (g @ self.w[i].T) * (pre[i - 1] > 0)
        norm = np.sqrt(sum(float((q * q).sum()) for q in gw + gb))
        clip = self.max_norm / norm if norm > self.max_norm else 1.0
        for i in range(L):
            self.vw[i] = self.m * self.vw[i] + gw[i] * clip + self.wd * self.w[i]
            self.w[i] = self.w[i] - self.lr * self.vw[i]
            self.vb[i] = self.m * self.vb[i] + gb[i] * clip + self.wd * self.b[i]
            self.b[i] = self.b[i] - self.lr * self.vb[i]
        return loss


# --------------------------------------------------------------------------
# fp64 helpers for error bounds
# --------------------------------------------------------------------------
def op_mats(a, b, M, K, N, ta, tb):
    A = np.asarray(a, np.float64).reshape((K, M) if ta else (M, K))
    B = np.asarray(b, np.float64).reshape((N, K) if tb else (K, N))
    return (A.T if ta else A), (B.T if tb else B)


def gemm_fp64(a, b, M, K, N, ta=0, tb=0):
    A, B = op_mats(a, b, M, K, N, ta, tb)
    return A @ B


def abs_product_sum(a, b, M, K, N, ta=0, tb=0):
    """sum_k |a_ik * b_kj|: the scale of the componentwise error bound."""
    A, B = op_mats(a, b, M, K, N, ta, tb)
    return np.abs(A) @ np.abs(B)


def componentwise_rel_err(c, ref64, scale):
    """max |c - c64| / sum_k |a b| over all elements (0 where the scale is 0)."""
    c = np.asarray(c, np.float64)
    d = np.abs(c - ref64)
    s = np.where(scale > 0, scale, 1.0)
    r = np.where(scale > 0, d / s, d)
    return float(r.max()) if r.size else 0.0


def reference_gpu_lib_path() -> str:
    """Path of the reference's own cuda_kernels.cu built for sm_100a."""
    return _REF_LIB_PATH
