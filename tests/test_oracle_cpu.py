"""CPU tests of the oracle (oracle/np_oracle.c) -- pins the restatement of the
NpArray path against the reference's own known-answer tests and checks its
arithmetic properties.  No GPU."""
from __future__ import annotations

import json
import os
import struct

import numpy as np
import pytest

import oracle
from moonxi_net_b200 import synthetic

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def kats():
    with open(os.path.join(GOLDEN, "ref_kats.json")) as f:
        return json.load(f)


def test_kat_matmul(kats):
    k = kats["matmul_2x2"]
    c = oracle.matmul(np.array(k["a"], np.float32), np.array(k["b"], np.float32))
    assert c.ravel().tolist() == k["c"]


def test_kat_transpose(kats):
    k = kats["transpose_2x3"]
    y = oracle.transpose(np.array(k["x"], np.float32))
    assert y.shape == (3, 2) and y.ravel().tolist() == k["y"]


def test_kat_matmul_backward(kats):
    """dA = og . transpose(B), dB = transpose(A) . og (grad/blas.mbt:35,37)."""
    k = kats["matmul_backward_mean"]
    a, b, og = (np.array(k[n], np.float32) for n in ("a", "b", "og"))
    da = oracle.matmul(og, oracle.transpose(b))
    db = oracle.matmul(oracle.transpose(a), og)
    assert da.tolist() == k["da"] and db.tolist() == k["db"]
    # same through the cuda_matmul-semantics entry (NT and TN flags)
    assert oracle.gemm(og, b, 2, 2, 2, 0, 1).tolist() == k["da"]
    assert oracle.gemm(a, og, 2, 2, 2, 1, 0).tolist() == k["db"]


@pytest.mark.parametrize("name", ["linear_forward", "linear_forward_bias"])
def test_kat_linear(kats, name):
    k = kats[name]
    z = oracle.matmul(np.array(k["x"], np.float32), np.array(k["w"], np.float32))
    y = oracle.add_row_bias(z, np.array(k["b"], np.float32))
    assert np.allclose(y.ravel(), k["y"], atol=k["eps"], rtol=0)


def test_kat_sequential(kats):
    k = kats["sequential_two_linear"]
    h = oracle.add_row_bias(oracle.matmul(np.array(k["x"], np.float32),
                                          np.array(k["w1"], np.float32)),
                            np.array(k["b1"], np.float32))
    y = oracle.add_row_bias(oracle.matmul(h, np.array(k["w2"], np.float32)),
                            np.array(k["b2"], np.float32))
    assert np.allclose(y.ravel(), k["y"], atol=k["eps"], rtol=0)


def test_matmul_sequential_k_order():
    """Each element is the fp32 left-to-right sum of fp32 products."""
    rng = np.random.default_rng(11)
    a = rng.standard_normal((5, 37), dtype=np.float32)
    b = rng.standard_normal((37, 6), dtype=np.float32)
    c = oracle.matmul(a, b)
    for i in range(5):
        for j in range(6):
            s = np.float32(0.0)
            for k in range(37):
                s = np.float32(s + np.float32(a[i, k] * b[k, j]))
            assert c[i, j] == s


def test_matmul_threads_bit_identical():
    rng = np.random.default_rng(12)
    a = rng.standard_normal((333, 257), dtype=np.float32)
    b = rng.standard_normal((257, 190), dtype=np.float32)
    assert np.array_equal(oracle.matmul(a, b, 1), oracle.matmul(a, b, 8))


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gemm_layouts_against_fp64(ta, tb):
    M, K, N = 70, 129, 33
    a, b, _ = synthetic.gemm_problem(M, K, N, ta, tb, 3)
    c = oracle.gemm(a, b, M, K, N, ta, tb, alpha=0.5, beta=0.0)
    ref = 0.5 * oracle.gemm_fp64(a, b, M, K, N, ta, tb)
    scale = 0.5 * oracle.abs_product_sum(a, b, M, K, N, ta, tb)
    # sequential fp32 summation: error below K * 2^-24 of the scale
    assert oracle.componentwise_rel_err(c, ref, scale) <= K * 2.0 ** -24


def test_gemm_beta():
    rng = np.random.default_rng(2)
    a = rng.standard_normal((4, 3), dtype=np.float32)
    b = rng.standard_normal((3, 5), dtype=np.float32)
    c0 = rng.standard_normal((4, 5), dtype=np.float32)
    c = oracle.gemm(a, b, 4, 3, 5, 0, 0, 1.0, 2.0, c=c0)
    expect = (oracle.matmul(a, b) + np.float32(2.0) * c0).astype(np.float32)
    assert np.array_equal(c, expect)


def test_relu_and_backward():
    x = np.array([-1.0, 0.0, 2.0, np.nan], np.float32)
    assert oracle.relu(x)[:3].tolist() == [0.0, 0.0, 2.0] and oracle.relu(x)[3] == 0.0
    g = np.array([5.0, 6.0, 7.0, 8.0], np.float32)
    assert oracle.relu_backward(g, x).tolist() == [0.0, 0.0, 7.0, 0.0]


def test_reduce_sum_leading_order():
    x = np.array([[1e8, 1.0], [1.0, 2.0], [-1e8, 3.0]], np.float32)
    # sequential fp32: (1e8 + 1) + -1e8 = 0 in fp32
    assert oracle.reduce_sum_leading(x).tolist() == [0.0, 6.0]


def test_cross_entropy_matches_fp64_and_grad_sums_to_zero():
    rng = np.random.default_rng(5)
    logits = rng.standard_normal((16, 10), dtype=np.float32)
    labels = rng.integers(0, 10, 16).astype(np.float32)
    loss = oracle.ce_forward(logits, labels)
    l64 = logits.astype(np.float64)
    lse = np.log(np.exp(l64 - l64.max(1, keepdims=True)).sum(1)) + l64.max(1)
    ref = float(np.mean(lse - l64[np.arange(16), labels.astype(int)]))
    assert abs(loss - ref) <= 1e-5
    g = oracle.ce_backward(logits, labels)
    assert np.allclose(g.sum(1), 0.0, atol=1e-6)
    # denom scaling (data parallel shards use the global batch)
    assert np.allclose(oracle.ce_backward(logits, labels, denom=32), g / 2, rtol=1e-6)


def test_sgd_autoclip():
    p = [np.array([1.0, 2.0], np.float32)]
    g = [np.array([30.0, 40.0], np.float32)]  # norm 50 > 35 -> clip 0.7
    v = [np.zeros(2, np.float32)]
    norm = oracle.sgd_momentum_autoclip(p, g, v, 0.01, 0.9, 1e-4, 35.0)
    assert abs(norm - 50.0) < 1e-5
    clip = np.float32(35.0) / np.float32(50.0)
    v_exp = (np.float32(0.9) * 0 + g[0] * clip) + np.float32(1e-4) * np.array([1, 2], np.float32)
    assert np.allclose(v[0], v_exp, rtol=1e-7)
    assert np.allclose(p[0], np.array([1, 2], np.float32) - np.float32(0.01) * v_exp, rtol=1e-7)


def test_mlp_layouts_agree():
    """The nn and nt layouts describe the same model: identical numbers."""
    wn, bn, x, y = synthetic.mlp_problem("mlp784", layout="nn")
    wt, bt, _, _ = synthetic.mlp_problem("mlp784", layout="nt")
    ln, gn = oracle.MLPOracle(wn, bn, "nn", threads=8).grads(x, y)
    lt, gt = oracle.MLPOracle(wt, bt, "nt", threads=8).grads(x, y)
    assert ln == lt
    for i in range(0, len(gn), 2):
        assert np.array_equal(gn[i], gt[i].T)
        assert np.array_equal(gn[i + 1], gt[i + 1])


def test_mlp784_fixture():
    with open(os.path.join(GOLDEN, "mlp784_step.json")) as f:
        fx = json.load(f)
    w, b, x, y = synthetic.mlp_problem("mlp784")
    loss, grads = oracle.MLPOracle(w, b, threads=8).grads(x, y)
    assert struct.pack("<f", np.float32(loss)).hex() == fx["loss_hex"]
    for g, s in zip(grads, fx["grad_sum_abs"]):
        assert float(np.abs(g.astype(np.float64)).sum()) == s


def test_loss_curve_fixture_prefix():
    """The first steps of the committed 200-step curve reproduce bit-exactly."""
    with open(os.path.join(GOLDEN, "mlp3072_loss_curve.json")) as f:
        fx = json.load(f)
    w, b, x, y = synthetic.mlp_problem("mlp3072")
    m = oracle.MLPOracle(w, b, threads=oracle.default_threads())
    for s in range(2):
        assert struct.pack("<f", np.float32(m.step(x, y))).hex() == fx["loss_hex"][s]


def test_mlp_grads_against_fp64_autograd():
    """Oracle gradients against an independent fp64 derivation."""
    w, b, x, y = synthetic.mlp_problem("mlp784")
    loss, grads = oracle.MLPOracle(w, b, threads=8).grads(x, y)
    W = [wi.astype(np.float64) for wi in w]
    h0 = x.astype(np.float64)
    a1 = h0 @ W[0]
    h1 = np.maximum(a1, 0)
    a2 = h1 @ W[1]
    p = np.exp(a2 - a2.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    oh = np.zeros_like(p)
    oh[np.arange(len(y)), y.astype(int)] = 1
    g2 = (p - oh) / len(y)
    gw2 = h1.T @ g2
    g1 = (g2 @ W[1].T) * (a1 > 0)
    gw1 = h0.T @ g1
    for got, ref in ((grads[0], gw1), (grads[1], g1.sum(0)), (grads[2], gw2), (grads[3], g2.sum(0))):
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-4


def test_fused_linear_bias_first_order():
    """fused_linear(_relu) (nparray/fused_ops.mbt:12-78) starts every sum from
    the bias: a pure-Python loop of the same order agrees bit for bit, and the
    result differs from matmul -> add in the last bits on inputs chosen so
    the two orders round differently."""
    rng = np.random.default_rng(11)
    x = rng.standard_normal((5, 37), dtype=np.float32)
    w = rng.standard_normal((7, 37), dtype=np.float32)
    b = (rng.standard_normal(7) * 1e3).astype(np.float32)
    out, pre = oracle.fused_linear(x, w, b, relu=True, threads=3)
    for i in range(5):
        for j in range(7):
            s = np.float32(b[j])
            for k in range(37):
                s = np.float32(s + np.float32(x[i, k] * w[j, k]))
            assert pre[i, j] == s
            assert out[i, j] == (s if s > 0 else np.float32(0))
    out2, pre2 = oracle.fused_linear(x, w, b, relu=False)
    assert np.array_equal(out2, pre2) and np.array_equal(pre2, pre)
    later = oracle.add_row_bias(oracle.matmul(x, np.ascontiguousarray(w.T)), b)
    assert not np.array_equal(later, pre)  # the two rounding orders differ
    assert np.allclose(later, pre, rtol=1e-5, atol=1e-2)
