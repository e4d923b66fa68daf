"""Data-parallel host logic on CPU ranks (gloo, world size 2).

The GPU step shards the global batch by rows, scales the loss by
1/global_batch, all-reduces each layer's gradient bucket (FlatLayout) in
backward order and lets every replica apply the identical update.  Here the
same host logic runs on two gloo ranks with the CPU oracle doing the math,
and must reproduce the single-process step; a rank that leaves before the
collective must surface as an error on the other rank, not a hang.
"""
from __future__ import annotations

import datetime
import os
import socket
import sys
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_worker(rank, world, port, outdir, mode):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
    import oracle
    from moonxi_net_b200 import nn, synthetic
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        if mode == "leave" and rank == 1:
            return  # leaves without joining the collective
        w, b, x, y = synthetic.mlp_problem("mlp784")
        lay = nn.FlatLayout([784, 256, 10])
        lo, hi = nn.shard_rows(x.shape[0], rank, world)
        m = oracle.MLPOracle(w, b, threads=2)
        loss, grads = m.grads(x[lo:hi], y[lo:hi], denom=x.shape[0])
        buf = torch.zeros(lay.grads_buf_len)
        g = buf[64:]
        buf[0] = loss
        for i in range(lay.L):
            s, e = lay.w_range(i)
            g[s:e] = torch.from_numpy(grads[2 * i].ravel())
            s, e = lay.b_range(i)
            g[s:e] = torch.from_numpy(grads[2 * i + 1])
        try:
            for i in lay.reduce_order():
                s, e = lay.bucket(i)
                view = buf[s:e]
                dist.all_reduce(view)
        except Exception as exc:  # noqa: BLE001 -- any collective failure is "detected"
            with open(os.path.join(outdir, f"err{rank}.txt"), "w") as f:
                f.write(type(exc).__name__)
            return
        red = []
        for i in range(lay.L):
            s, e = lay.w_range(i)
            red.append(g[s:e].numpy().reshape(grads[2 * i].shape).copy())
            s, e = lay.b_range(i)
            red.append(g[s:e].numpy().copy())
        vels = [np.zeros_like(p) for p in m.params()]
        oracle.sgd_momentum_autoclip(m.params(), red, vels, m.lr, m.momentum, m.wd, m.max_norm)
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), loss=float(buf[0]), *red, *m.params())
    finally:
        if not (mode == "leave" and rank == 0):
            dist.destroy_process_group()


def _run(world, mode, outdir):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_dp_worker, args=(r, world, port, outdir, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    return [p.exitcode for p in procs]


def test_dp_two_ranks_match_single_process():
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
    import oracle
    from moonxi_net_b200 import synthetic
    with tempfile.TemporaryDirectory() as d:
        codes = _run(2, "ok", d)
        assert codes == [0, 0]
        r0 = np.load(os.path.join(d, "rank0.npz"))
        r1 = np.load(os.path.join(d, "rank1.npz"))
        keys = [k for k in r0.files if k.startswith("arr_")]
        for k in keys:  # every replica holds the identical gradients and update
            assert np.array_equal(r0[k], r1[k])
        assert r0["loss"] == r1["loss"]
        w, b, x, y = synthetic.mlp_problem("mlp784")
        m = oracle.MLPOracle(w, b, threads=4)
        loss, grads = m.grads(x, y)
        assert abs(float(r0["loss"]) - loss) <= 1e-6
        for i, gref in enumerate(grads):
            got = r0[f"arr_{i}"]
            assert np.linalg.norm(got - gref) <= 1e-6 * np.linalg.norm(gref) + 1e-9
        m.step(x, y)
        for j, pref in enumerate(m.params()):
            got = r0[f"arr_{len(grads) + j}"]
            assert np.linalg.norm(got - pref) <= 1e-6 * np.linalg.norm(pref) + 1e-9


def _shard_worker(rank, world, port, outdir):
    """The sharded update's host logic: reduce-scatter each bucket into this
    rank's piece, the global norm from per-rank partial sums, the update of
    the rank's own ranges, then the all-gather of the new parameters."""
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
    import oracle
    from moonxi_net_b200 import nn, synthetic
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        w, b, x, y = synthetic.mlp_problem("mlp784")
        lay = nn.FlatLayout([784, 256, 10], shard_world=world)
        plan = nn.ShardPlan(lay, world, rank)
        lo, hi = nn.shard_rows(x.shape[0], rank, world)
        m = oracle.MLPOracle(w, b, threads=2)
        loss, grads = m.grads(x[lo:hi], y[lo:hi], denom=x.shape[0])
        buf = torch.zeros(lay.grads_buf_len)
        pfull = torch.zeros(lay.grads_buf_len)
        vfull = torch.zeros(lay.grads_buf_len)
        for i in range(lay.L):
            s, e = lay.w_range(i)
            buf[64 + s:64 + e] = torch.from_numpy(grads[2 * i].ravel())
            pfull[64 + s:64 + e] = torch.from_numpy(np.asarray(w[i], np.float32).ravel())
            s, e = lay.b_range(i)
            buf[64 + s:64 + e] = torch.from_numpy(grads[2 * i + 1])
            pfull[64 + s:64 + e] = torch.from_numpy(np.asarray(b[i], np.float32))
        for i in lay.reduce_order():
            plan.reduce_scatter(buf, i, None, async_op=False)
        ranges = plan.update_ranges()
        norm_sq = torch.tensor([sum(float((buf[a:bb].double() ** 2).sum()) for a, bb in ranges)])
        dist.all_reduce(norm_sq)
        for a, bb in ranges:  # clip inactive here (asserted by the caller)
            oracle.sgd_momentum_autoclip([pfull[a:bb].numpy()], [buf[a:bb].numpy()],
                                         [vfull[a:bb].numpy()], m.lr, m.momentum, m.wd, 1e30)
        for i in range(lay.L):
            plan.all_gather(pfull, i, None, async_op=False)
        params = []
        for i in range(lay.L):
            s, e = lay.w_range(i)
            params.append(pfull[64 + s:64 + e].numpy().copy())
            s, e = lay.b_range(i)
            params.append(pfull[64 + s:64 + e].numpy().copy())
        np.savez(os.path.join(outdir, f"shard{rank}.npz"), norm_sq=float(norm_sq[0]),
                 ranges=np.array(ranges), *params)
    finally:
        dist.destroy_process_group()


def test_sharded_update_matches_replicated():
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
    import oracle
    from moonxi_net_b200 import nn, synthetic
    lay = nn.FlatLayout([784, 256, 10], shard_world=2)
    for i in range(lay.L):  # buckets split into 2 equal, 256-byte aligned pieces
        s, e = lay.bucket(i)
        assert (e - s) % 128 == 0
    # one rank: the unpadded layout ([w1, b1, w2, b2], 64-float blocks)
    assert nn.FlatLayout([784, 256, 10]).b_off == [784 * 256, 784 * 256 + 256 + 256 * 10]
    with tempfile.TemporaryDirectory() as d:
        port = _free_port()
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
                pytest.fail("a rank hung")
        assert [p.exitcode for p in procs] == [0, 0]
        r0 = np.load(os.path.join(d, "shard0.npz"))
        r1 = np.load(os.path.join(d, "shard1.npz"))
        # the two ranks own disjoint ranges that cover every parameter
        own = sorted([tuple(r) for r in r0["ranges"]] + [tuple(r) for r in r1["ranges"]])
        assert own[0][0] == 64 and own[-1][1] == lay.grads_buf_len
        assert all(own[k][1] == own[k + 1][0] for k in range(len(own) - 1))
        assert r0["norm_sq"] == r1["norm_sq"]
        keys = [k for k in r0.files if k.startswith("arr_")]
        for k in keys:  # identical replicas after the all-gather
            assert np.array_equal(r0[k], r1[k])
        w, b, x, y = synthetic.mlp_problem("mlp784")
        m = oracle.MLPOracle(w, b, threads=4)
        _, grads = m.grads(x, y)
        gn = float(np.sqrt(sum(float((g.astype(np.float64) ** 2).sum()) for g in grads)))
        assert gn < m.max_norm  # the replicated step does not clip either
        assert abs(np.sqrt(r0["norm_sq"]) - gn) <= 1e-5 * gn
        m.step(x, y)
        for j, pref in enumerate(m.params()):
            got = r0[f"arr_{j}"].reshape(pref.shape)
            assert np.linalg.norm(got - pref) <= 1e-6 * np.linalg.norm(pref) + 1e-9


def test_dp_rank_leaving_is_detected():
    with tempfile.TemporaryDirectory() as d:
        codes = _run(2, "leave", d)
        assert codes[1] == 0
        assert os.path.exists(os.path.join(d, "err0.txt")), "rank 0 did not see the failure"
