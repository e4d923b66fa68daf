"""Data-parallel training step on 2 GPUs (NCCL), against one GPU.

Each rank runs the MLP step on its half of the batch with the loss scaled by
1/global_batch and all-reduces the per-layer gradient buckets; both replicas
must end bit-identical, and match a single-GPU run on the whole batch within
the fp32-class tolerance.  The step is also captured in a CUDA graph with its
all-reduces and replayed.  Three models: MLP 3072->1024->1024->10 (per-call
3xTF32 GEMMs, bucket all-reduce), a split-form model with the sharded update
(bucket reduce-scatter, each rank updates half the parameters, all-gather of
the new weights at the next step's start), and the same split-form model
with bucket all-reduces, its first-layer bucket reduced in row chunks as the
chunks are computed.  The collectives go through the library's NCCL stubs
(moonbit_nccl_*), and once more through torch.distributed for the last
model.  Needs two visible GPUs (skipped otherwise).
"""
from __future__ import annotations

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
pytestmark = pytest.mark.gpu
STEPS = 3
SPLIT_DIMS = [1024, 512, 256, 128]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(model):
    model = model.replace("_torch", "")
    import sys
    sys.path.insert(0, ROOT)
    from moonxi_net_b200 import synthetic
    if model == "mlp3072":
        w, b, x, y = synthetic.mlp_problem("mlp3072", batch=512)
        return [3072, 1024, 1024, 10], w, b, x, y
    rng = np.random.default_rng(9)
    d = SPLIT_DIMS
    w = [synthetic.kaiming_uniform(rng, d[i], (d[i], d[i + 1])) for i in range(len(d) - 1)]
    b = [np.zeros(d[i + 1], np.float32) for i in range(len(d) - 1)]
    x = rng.standard_normal((512, d[0]), dtype=np.float32)
    y = rng.integers(0, d[-1], 512).astype(np.float32)
    return d, w, b, x, y


def _flat_params(m):
    """Every weight and bias, concatenated (layout padding excluded: the
    sharded model pads its buckets to split evenly over the ranks)."""
    ws, bs = m.weights_numpy()
    return np.concatenate([a.ravel() for a in ws] + [a.ravel() for a in bs])


def _worker(rank, world, port, outdir, use_graph, model):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from moonxi_net_b200 import nn
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        dims, w, b, x, y = _problem(model)
        lo, hi = nn.shard_rows(512, rank, world)
        X = torch.from_numpy(x[lo:hi].copy()).to(dev)
        Y = torch.from_numpy(y[lo:hi].copy()).to(dev)
        torch_coll = model.endswith("_torch")
        model = model.replace("_torch", "")
        m = nn.MLP(dims, w, b, precision="3xtf32", process_group=dist.group.WORLD,
                   shard_update=(model != "split_allreduce"),
                   collectives="torch" if torch_coll else None)
        from moonxi_net_b200.collectives import NcclCollectives
        assert isinstance(m.coll, NcclCollectives) != torch_coll
        assert m.fused == (model != "mlp3072")
        assert m.sharded == (model == "split")
        m.last_bucket_chunks = 4  # exercise the chunked first-layer bucket
        losses = []
        if use_graph:
            losses.append(float(m.step(X, Y, 512).item()))
            m.capture(X, Y, 512)
            for _ in range(STEPS - 1):
                losses.append(float(m.replay().item()))
            m.release_graph()
        else:
            for _ in range(STEPS):
                losses.append(float(m.step(X, Y, 512).item()))
        m.sync_params()  # sharded update: gather every rank's pieces
        torch.cuda.synchronize()
        m.close()
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), params=_flat_params(m),
                 losses=np.array(losses))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(use_graph, model):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, d, use_graph, model))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            if p.is_alive():
                p.kill()
                pytest.fail("a rank did not finish")
        assert [p.exitcode for p in procs] == [0, 0]
        return [dict(np.load(os.path.join(d, f"rank{r}.npz"))) for r in range(2)]


@pytest.mark.parametrize("model", ["mlp3072", "split", "split_allreduce",
                                   "split_allreduce_torch"])
@pytest.mark.parametrize("use_graph", [False, True])
def test_dp2_matches_single_gpu(cuda_device, use_graph, model):
    from moonxi_net_b200 import nn
    r0, r1 = _run(use_graph, model)
    assert np.array_equal(r0["params"], r1["params"])       # identical replicas
    assert np.array_equal(r0["losses"], r1["losses"])
    dims, w, b, x, y = _problem(model)
    m = nn.MLP(dims, w, b, precision="3xtf32")
    X, Y = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    losses = [float(m.step(X, Y).item()) for _ in range(STEPS)]
    ref = _flat_params(m).astype(np.float64)
    got = r0["params"].astype(np.float64)
    assert np.linalg.norm(got - ref) <= 1e-5 * np.linalg.norm(ref)
    assert np.allclose(r0["losses"], losses, rtol=0, atol=1e-5)
