"""Writes the committed golden fixtures of this directory.

* ``ref_kats.json`` -- known-answer vectors from the reference's own unit
  tests, transcribed from the test sources (each entry cites file:line).
  The reference is MoonBit and cannot run here, so these are the values its
  tests assert.
* ``mlp3072_loss_curve.json`` -- the loss curve of 200 momentum-SGD steps of
  configuration "MLP 3072->1024->1024->10, batch 512, seed 2" computed by the
  CPU oracle (oracle/np_oracle.c, a restatement of the NpArray path), same
  batch every step, Linear layout (w [in, out]).  Values are stored as fp32
  bit patterns (hex) so they round-trip exactly.
* ``mlp784_step.json`` -- loss and gradient checksums of one step of
  configuration "MLP 784->256->10, batch 64, seed 0" from the oracle.

The reference GPU step's curves in ``mlp3072_loss_curve.json`` are added by
``make_ref_gpu_curve.py`` (needs a GPU); rewriting the curve here drops them.

Run from the repository root:  python tests/golden/make_golden.py [--skip-curve]
"""
from __future__ import annotations

import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle  # noqa: E402
from moonxi_net_b200 import synthetic  # noqa: E402


def f32hex(x) -> str:
    return struct.pack("<f", np.float32(x)).hex()


# Values the reference's tests assert (paths relative to the moonxi-net root).
REF_KATS = {
    "matmul_2x2": {
        "source": "moonxi-net/nparray/nparray_wbtest.mbt:205-214",
        "a": [[1.0, 2.0], [3.0, 4.0]],
        "b": [[5.0, 6.0], [7.0, 8.0]],
        "c": [19.0, 22.0, 43.0, 50.0],
        "exact": True,
    },
    "transpose_2x3": {
        "source": "moonxi-net/nparray/nparray_wbtest.mbt:217-224",
        "x": [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]],
        "y": [1.0, 4.0, 2.0, 5.0, 3.0, 6.0],
        "exact": True,
    },
    "matmul_backward_mean": {
        "source": "moonxi-net/grad/grad_wbtest.mbt:104-134",
        "a": [[1.0, 2.0], [3.0, 4.0]],
        "b": [[5.0, 6.0], [7.0, 8.0]],
        "og": [[0.25, 0.25], [0.25, 0.25]],
        "da": [[2.75, 3.75], [2.75, 3.75]],
        "db": [[1.0, 1.0], [1.5, 1.5]],
        "exact": True,
    },
    "linear_forward": {
        "source": "moonxi-net/model/model_wbtest.mbt:11-29",
        "x": [[3.0, 5.0]],
        "w": [[1.0, 0.0, 1.0], [0.0, 1.0, 1.0]],
        "b": [0.0, 0.0, 0.0],
        "y": [3.0, 5.0, 8.0],
        "eps": 1e-4,
    },
    "linear_forward_bias": {
        "source": "moonxi-net/model/model_wbtest.mbt:32-44",
        "x": [[1.0, 1.0]],
        "w": [[2.0, 4.0], [3.0, 5.0]],
        "b": [10.0, 20.0],
        "y": [15.0, 29.0],
        "eps": 1e-4,
    },
    "sequential_two_linear": {
        "source": "moonxi-net/model/model_wbtest.mbt:63-97",
        "x": [[1.0, 2.0]],
        "w1": [[1.0, 0.0, 1.0], [0.0, 1.0, 1.0]],
        "b1": [0.0, 0.0, 0.0],
        "w2": [[1.0, 0.0], [0.0, 1.0], [0.0, 0.0]],
        "b2": [0.0, 0.0],
        "y": [1.0, 2.0],
        "eps": 1e-4,
    },
}


def write_kats():
    with open(os.path.join(HERE, "ref_kats.json"), "w") as f:
        json.dump(REF_KATS, f, indent=1)


def write_mlp784_step():
    w, b, x, y = synthetic.mlp_problem("mlp784")
    m = oracle.MLPOracle(w, b, layout="nn", threads=oracle.default_threads())
    loss, grads = m.grads(x, y)
    out = {
        "config": "mlp784 batch 64 seed 0, layout nn, one step",
        "loss_hex": f32hex(loss),
        "grad_sum_abs": [float(np.abs(g.astype(np.float64)).sum()) for g in grads],
        "grad_sum": [float(g.astype(np.float64).sum()) for g in grads],
    }
    with open(os.path.join(HERE, "mlp784_step.json"), "w") as f:
        json.dump(out, f, indent=1)


def write_loss_curve(steps=200):
    w, b, x, y = synthetic.mlp_problem("mlp3072")
    m = oracle.MLPOracle(w, b, layout="nn", threads=oracle.default_threads())
    m64 = oracle.MLPFloat64(w, b)
    losses, l64 = [], []
    for s in range(steps):
        losses.append(m.step(x, y))
        l64.append(m64.step(x, y))
        if s % 20 == 0:
            print(f"step {s}: loss {losses[-1]:.6f} fp64 {l64[-1]:.6f}", flush=True)
    dev = [abs(float(a) - b) for a, b in zip(losses, l64)]
    out = {
        "config": "mlp3072 batch 512 seed 2, layout nn, same batch each step, "
                  "momentum SGD lr 0.01 m 0.9 wd 1e-4 clip 35",
        "steps": steps,
        "loss_hex": [f32hex(v) for v in losses],
        # the same run in float64 (oracle.MLPFloat64): how far exact arithmetic
        # lands from the fp32 NpArray curve
        "loss_fp64": [repr(v) for v in l64],
        "max_abs_dev_fp64_vs_oracle": max(dev),
    }
    with open(os.path.join(HERE, "mlp3072_loss_curve.json"), "w") as f:
        json.dump(out, f, indent=0)


if __name__ == "__main__":
    oracle.build()
    write_kats()
    write_mlp784_step()
    if "--skip-curve" not in sys.argv:
        write_loss_curve()
