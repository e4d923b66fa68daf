"""Adds the reference GPU step's loss curves to ``mlp3072_loss_curve.json``.

The bound the fast kernels' loss curves are held to is measured on the
reference, not assumed.  The same 200 momentum-SGD steps of "MLP
3072->1024->1024->10, batch 512, seed 2" as the fixture's NpArray curve run
here on the GPU through the reference's own exported kernels, built
unmodified from moonxi-net-gpu/cuda/cuda_kernels.cu into ``oracle/_ref``:

* every GEMM through ``cuda_matmul`` (:1464-1499, cuBLAS with FP32 compute),
  along both of the reference's call paths: "tensor" -- as GpuTensor::matmul
  calls it (tensor/trait_impl.mbt:226-250), no transpose flags, on transposes
  materialised by ``cuda_transpose_2d`` (:1771); "flags" -- with the transpose
  flags, as the moonbit_cuda_matmul stub allows (cuda_stub.c:948-969);
* the loss and its gradient through ``cuda_softmax_ce_forward_labels`` /
  ``cuda_softmax_ce_backward_labels`` (:1283-1374, float exp, the loss summed
  with atomicAdd);
* the bias gradients through ``cuda_reduce_sum_leading`` (:1383-1406);
* the optimizer through ``cuda_mt_norm_sq_gpu_only`` (atomicAdd of block
  sums) and ``cuda_mt_sgd_momentum_autoclip`` (:1884-2029);
* ReLU forward/backward as exact max / mask (the reference calls cuDNN), and
  the bias add as a row broadcast (NpArray semantics: the reference's GPU add
  is not a broadcast -- it reads past the bias buffer -- so it cannot be run).

Each path runs RUNS times (the atomic sums make the reference's step
run-to-run nondeterministic).  The fixture records every curve (fp32 hex)
and ``max_abs_dev_ref_gpu_vs_oracle``: the largest distance of any of them
from the fp32 NpArray curve -- how far the reference's own GPU training
drifts from its CPU path.

Needs a GPU.  Run from the repository root:
    python tests/golden/make_ref_gpu_curve.py [--out PATH]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import torch  # noqa: E402

import oracle  # noqa: E402
from moonxi_net_b200 import synthetic  # noqa: E402

RUNS = 3
DIMS = [3072, 1024, 1024, 10]


def f32hex(x) -> str:
    return struct.pack("<f", float(x)).hex()


def load_reference():
    path = oracle.reference_gpu_lib_path()
    if not os.path.exists(path):
        raise SystemExit(f"reference GPU library missing: {path} (make -C oracle ref)")
    L = ctypes.CDLL(path)
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.cublas_create_handle.restype = vp
    sig = {
        "cuda_matmul": [vp] * 4 + [i] * 5 + [f] * 2,
        "cuda_transpose_2d": [vp, vp, i, i],
        "cuda_softmax_ce_forward_labels": [vp, vp, vp, i, i],
        "cuda_softmax_ce_backward_labels": [vp, vp, vp, i, i],
        "cuda_reduce_sum_leading": [vp, vp, i, i],
        "cuda_mt_norm_sq_gpu_only": [vp, vp, vp, i, i, vp],
        "cuda_mt_sgd_momentum_autoclip": [vp, vp, vp, vp, vp, i, i, f, f, f, vp, f],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.restype = i
        fn.argtypes = args
    return L


class ReferenceGpuStep:
    """The reference's GPU training step for a Linear stack (layout nn:
    w [in, out]), built from its exported kernels (module docstring)."""

    def __init__(self, L, weights, biases, path, lr=0.01, momentum=0.9, wd=1e-4, max_norm=35.0):
        self.L, self.path = L, path
        self.h = L.cublas_create_handle()
        assert self.h
        dev = "cuda"
        self.w = [torch.from_numpy(np.ascontiguousarray(w, np.float32)).to(dev) for w in weights]
        self.b = [torch.from_numpy(np.ascontiguousarray(b, np.float32)).to(dev) for b in biases]
        self.params = [t for pair in zip(self.w, self.b) for t in pair]
        self.grads = [torch.zeros_like(t) for t in self.params]
        self.vels = [torch.zeros_like(t) for t in self.params]
        self.lr, self.momentum, self.wd, self.max_norm = lr, momentum, wd, max_norm
        sizes = [t.numel() for t in self.params]
        blocks = [(n + 255) // 256 for n in sizes]
        offs = np.concatenate([[0], np.cumsum(blocks)[:-1]]).astype(np.int32)
        self.total_blocks = int(sum(blocks))
        self.d_sizes = torch.tensor(sizes, dtype=torch.int32, device=dev)
        self.d_offs = torch.from_numpy(offs).to(dev)
        ptrs = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=dev)
        self.d_p, self.d_g, self.d_v = ptrs(self.params), ptrs(self.grads), ptrs(self.vels)
        self.norm = torch.zeros(1, device=dev)
        self.loss = torch.zeros(1, device=dev)

    def mm(self, a, b, ta=False, tb=False):
        """op(a) @ op(b) through cuda_matmul on the chosen call path."""
        if self.path == "tensor" and (ta or tb):
            if ta:
                a = self.transpose(a)
            if tb:
                b = self.transpose(b)
            ta = tb = False
        M = a.shape[1] if ta else a.shape[0]
        K = a.shape[0] if ta else a.shape[1]
        N = b.shape[0] if tb else b.shape[1]
        c = torch.empty((M, N), device="cuda")
        rc = self.L.cuda_matmul(self.h, a.data_ptr(), b.data_ptr(), c.data_ptr(), M, K, N,
                                int(ta), int(tb), 1.0, 0.0)
        assert rc == 0, rc
        return c

    def transpose(self, x):
        n, m = x.shape
        out = torch.empty((m, n), device="cuda")
        assert self.L.cuda_transpose_2d(x.data_ptr(), out.data_ptr(), n, m) == 0
        return out

    def step(self, x, labels):
        B = x.shape[0]
        nl = len(self.w)
        hs, pre = [x], []
        h = x
        for i in range(nl):  # x.matmul(w).add(b), relu between layers
            z = self.mm(h, self.w[i]) + self.b[i][None, :]
            pre.append(z)
            h = torch.clamp_min(z, 0.0) if i + 1 < nl else z
            hs.append(h)
        logits = hs[-1].contiguous()
        C = logits.shape[1]
        assert self.L.cuda_softmax_ce_forward_labels(logits.data_ptr(), labels.data_ptr(),
                                                     self.loss.data_ptr(), B, C) == 0
        g = torch.empty_like(logits)
        assert self.L.cuda_softmax_ce_backward_labels(logits.data_ptr(), labels.data_ptr(),
                                                      g.data_ptr(), B, C) == 0
        for i in reversed(range(nl)):
            gb = self.grads[2 * i + 1]
            assert self.L.cuda_reduce_sum_leading(g.data_ptr(), gb.data_ptr(), g.shape[1], B) == 0
            self.grads[2 * i].copy_(self.mm(hs[i], g, ta=True))            # dW = X^T dY
            if i > 0:
                dx = self.mm(g, self.w[i], tb=True)                         # dX = dY W^T
                g = torch.where(pre[i - 1] > 0, dx, torch.zeros_like(dx))   # relu backward
        self.norm.zero_()
        assert self.L.cuda_mt_norm_sq_gpu_only(self.d_g.data_ptr(), self.d_sizes.data_ptr(),
                                               self.d_offs.data_ptr(), len(self.params),
                                               self.total_blocks, self.norm.data_ptr()) == 0
        assert self.L.cuda_mt_sgd_momentum_autoclip(
            self.d_p.data_ptr(), self.d_g.data_ptr(), self.d_v.data_ptr(),
            self.d_sizes.data_ptr(), self.d_offs.data_ptr(), len(self.params),
            self.total_blocks, self.lr, self.momentum, self.wd, self.norm.data_ptr(),
            self.max_norm) == 0
        return float(self.loss.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "mlp3072_loss_curve.json"))
    args = ap.parse_args()
    with open(os.path.join(HERE, "mlp3072_loss_curve.json")) as f:
        fx = json.load(f)
    cpu = np.array([struct.unpack("<f", bytes.fromhex(h))[0] for h in fx["loss_hex"]])
    torch.cuda.set_device(0)
    L = load_reference()
    w, b, x, y = synthetic.mlp_problem("mlp3072")
    X, Y = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    curves, devs = {}, {}
    for path in ("tensor", "flags"):
        for run in range(RUNS):
            m = ReferenceGpuStep(L, w, b, path)
            losses = np.array([m.step(X, Y) for _ in range(fx["steps"])])
            key = f"{path}_{run}"
            curves[key] = [f32hex(v) for v in losses]
            devs[key] = float(np.abs(losses - cpu).max())
            print(f"{key}: max |ref-gpu - cpu| = {devs[key]:.3e} at step "
                  f"{int(np.abs(losses - cpu).argmax())}", flush=True)
    for k in ("loss_ref_gpu_hex", "ref_gpu_note"):
        fx.pop(k, None)
    fx["ref_gpu_curves_hex"] = curves
    fx["ref_gpu_max_abs_dev"] = devs
    fx["max_abs_dev_ref_gpu_vs_oracle"] = max(devs.values())
    fx["ref_gpu_note"] = ("the reference's own GPU step from its exported kernels "
                          "(cuda_kernels.cu, built from source), both matmul call paths, "
                          f"{RUNS} runs each; tests/golden/make_ref_gpu_curve.py")
    with open(args.out, "w") as f:
        json.dump(fx, f, indent=0)
    print(f"bound: {fx['max_abs_dev_ref_gpu_vs_oracle']:.3e}")


if __name__ == "__main__":
    main()
