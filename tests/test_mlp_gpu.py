"""GPU parity of the Linear/MLP training step against the CPU oracle.

* one step of "MLP 784->256->10, batch 64, seed 0" (both weight layouts):
  loss, every gradient and the updated parameters against the NpArray
  restatement (norm-wise relative error <= 1e-5 * sqrt(K) of the widest GEMM);
* 200 steps of "MLP 3072->1024->1024->10, batch 512, seed 2": |loss_gpu -
  loss_oracle| <= 1e-4 at every step against the committed oracle curve;
* a CUDA-graph replay of the step is bit-identical to the eager step.
"""
from __future__ import annotations

import json
import math
import os
import struct

import numpy as np
import pytest
import torch

import oracle
from moonxi_net_b200 import nn, synthetic

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den > 0 else 1.0))


def _to_dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("layout", ["nn", "nt"])
@pytest.mark.parametrize("precision", ["fp32", "3xtf32"])
def test_mlp784_step_matches_oracle(cuda_device, layout, precision):
    w, b, x, y = synthetic.mlp_problem("mlp784", layout=layout)
    ref = oracle.MLPOracle(w, b, layout=layout, threads=oracle.default_threads())
    loss_ref, grads_ref = ref.grads(x, y)
    m = nn.MLP([784, 256, 10], w, b, layout=layout, precision=precision)
    loss = m.step(_to_dev(x), _to_dev(y), update=False)
    torch.cuda.synchronize()
    tol = 1e-5 * math.sqrt(784)
    assert abs(float(loss.item()) - loss_ref) <= 1e-5 * max(1.0, abs(loss_ref))
    for g, gr in zip(m.grads_numpy(), grads_ref):
        assert _rel(g, gr) <= tol
    # the update (fresh model so velocities start at zero on both sides)
    m2 = nn.MLP([784, 256, 10], w, b, layout=layout, precision=precision)
    m2.step(_to_dev(x), _to_dev(y))
    ref2 = oracle.MLPOracle(w, b, layout=layout, threads=oracle.default_threads())
    ref2.step(x, y)
    ws, bs = m2.weights_numpy()
    for a_, r_ in zip(ws + bs, ref2.w + ref2.b):
        assert _rel(a_, r_) <= 1e-6


def test_mlp784_step_matches_fixture(cuda_device):
    """Loss of one step against the committed oracle fixture."""
    with open(os.path.join(GOLDEN, "mlp784_step.json")) as f:
        fx = json.load(f)
    w, b, x, y = synthetic.mlp_problem("mlp784")
    m = nn.MLP([784, 256, 10], w, b, layout="nn")
    loss = float(m.step(_to_dev(x), _to_dev(y), update=False).item())
    ref = struct.unpack("<f", bytes.fromhex(fx["loss_hex"]))[0]
    assert abs(loss - ref) <= 1e-5
    sums = [float(np.abs(g.astype(np.float64)).sum()) for g in m.grads_numpy()]
    for s, r in zip(sums, fx["grad_sum_abs"]):
        assert abs(s - r) <= 1e-4 * max(1.0, abs(r))


@pytest.mark.parametrize("precision", ["default", "fp32"])
def test_mlp3072_loss_curve_200_steps(cuda_device, precision):
    with open(os.path.join(GOLDEN, "mlp3072_loss_curve.json")) as f:
        fx = json.load(f)
    ref = [struct.unpack("<f", bytes.fromhex(h))[0] for h in fx["loss_hex"]]
    w, b, x, y = synthetic.mlp_problem("mlp3072")
    m = nn.MLP([3072, 1024, 1024, 10], w, b, layout="nn", precision=precision)
    X, Y = _to_dev(x), _to_dev(y)
    losses = torch.empty(len(ref), device="cuda")
    for s in range(len(ref)):
        losses[s:s + 1].copy_(m.step(X, Y))
    got = losses.cpu().numpy().astype(np.float64)
    diff = np.abs(got - np.asarray(ref, np.float64))
    assert float(diff.max()) <= 1e-4, (int(diff.argmax()), float(diff.max()))


def test_graph_replay_bit_identical(cuda_device):
    w, b, x, y = synthetic.mlp_problem("mlp3072", batch=256)
    X, Y = _to_dev(x), _to_dev(y)
    eager = nn.MLP([3072, 1024, 1024, 10], w, b)
    graphed = nn.MLP([3072, 1024, 1024, 10], w, b)
    eager.step(X, Y)
    graphed.step(X, Y)  # sizes every workspace before capture
    graphed.capture(X, Y)
    for _ in range(3):
        l1 = eager.step(X, Y).clone()
        l2 = graphed.replay().clone()
    torch.cuda.synchronize()
    assert torch.equal(l1, l2)
    assert torch.equal(eager.params, graphed.params)
    graphed.release_graph()


def test_wide_mlp_small_batch_matches_oracle(cuda_device):
    """The bench architecture (4096^3 -> 1000) on 64 rows against the oracle."""
    w, b, x, y = synthetic.mlp_problem("wide", batch=64)
    ref = oracle.MLPOracle(w, b, threads=oracle.default_threads())
    loss_ref, grads_ref = ref.grads(x, y)
    m = nn.MLP([4096, 4096, 4096, 4096, 1000], w, b)
    loss = float(m.step(_to_dev(x), _to_dev(y), update=False).item())
    assert abs(loss - loss_ref) <= 1e-5 * max(1.0, abs(loss_ref))
    for g, gr in zip(m.grads_numpy(), grads_ref):
        assert _rel(g, gr) <= 1e-5 * math.sqrt(4096)
