"""Seeded synthetic problems for the benchmark configurations.

No dataset is involved in this path: every configuration of the matmul
hot path is synthetic.  Inputs come from numpy's PCG64 generator with the
configuration's seed, in a fixed draw order (layer weights first, in layer
order, then inputs, then labels), so every implementation (the GPU path,
the CPU oracle, the tests) sees identical arrays.
"""
from __future__ import annotations

import numpy as np

# name -> (layer widths, batch, seed, input distribution)
MLP_CONFIGS = {
    # MLP 784->256->10, ReLU, batch 64, U[0,1) inputs, seed 0
    "mlp784": ([784, 256, 10], 64, 0, "uniform"),
    # MLP 3072->1024->1024->10, ReLU, batch 512, U[0,1) inputs, seed 2
    "mlp3072": ([3072, 1024, 1024, 10], 512, 2, "uniform"),
    # Wide MLP 4096->4096->4096->4096->1000, ReLU, global batch 8192, N(0,1), seed 3
    "wide": ([4096, 4096, 4096, 4096, 1000], 8192, 3, "normal"),
}


def kaiming_uniform(rng: np.random.Generator, fan_in: int, shape) -> np.ndarray:
    """U(-sqrt(6/fan_in), +sqrt(6/fan_in)) in float32."""
    bound = np.float32(np.sqrt(6.0 / fan_in))
    u = rng.random(shape, dtype=np.float32)
    return ((u * np.float32(2.0) - np.float32(1.0)) * bound).astype(np.float32)


def mlp_problem(name: str, layout: str = "nn", batch: int | None = None):
    """(weights, biases, x, labels) for a named MLP configuration.

    Weights are drawn as logical [in, out] matrices; layout "nn" stores them
    so (Linear::forward, w [in, out]), layout "nt" stores the transpose
    (MLP::forward, w [out, in]).  Biases are zero.  Labels are class indices
    stored as float32, as the reference's label tensors are.
    """
    dims, default_batch, seed, dist = MLP_CONFIGS[name]
    B = default_batch if batch is None else batch
    rng = np.random.default_rng(seed)
    weights, biases = [], []
    for i in range(len(dims) - 1):
        w = kaiming_uniform(rng, dims[i], (dims[i], dims[i + 1]))
        weights.append(np.ascontiguousarray(w if layout == "nn" else w.T))
        biases.append(np.zeros((dims[i + 1],), np.float32))
    if dist == "uniform":
        x = rng.random((B, dims[0]), dtype=np.float32)
    else:
        x = rng.standard_normal((B, dims[0]), dtype=np.float32)
    labels = rng.integers(0, dims[-1], size=B).astype(np.float32)
    return weights, biases, x, labels


def gemm_problem(M: int, K: int, N: int, ta: bool, tb: bool, seed: int, bias: bool = False):
    """A, B (stored per the transpose flags) and an optional bias, all N(0,1)."""
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((K, M) if ta else (M, K), dtype=np.float32)
    b = rng.standard_normal((N, K) if tb else (K, N), dtype=np.float32)
    bvec = rng.standard_normal((N,), dtype=np.float32) if bias else None
    return a, b, bvec


def gemm_sweep_sizes():
    """Square GEMM sweep of the reference configuration: M=N=K."""
    return [512, 1024, 2048, 4096, 8192]


def ragged_shapes():
    """Skinny / ragged GEMM shapes (tail-tile predication stress)."""
    return [(M, K, N) for M in (1, 7, 33, 127, 1000) for K in (512, 784, 3072, 4096)
            for N in (10, 100, 257, 1000)]
