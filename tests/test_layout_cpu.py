"""Flat buffer layout and the sharded-update partition, for 1/2/4/8 ranks (CPU).

FlatLayout places [w1, b1, w2, b2, ...] in 256-byte blocks behind a 64-float
loss slot; with G ranks each layer's gradient bucket is padded to a multiple
of 64*G floats so that ShardPlan can split it into G equal, 256-byte aligned
pieces.  The pieces of all ranks must tile every bucket, and the ranks'
update ranges must cover every parameter exactly once.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, ROOT)

from moonxi_net_b200 import nn  # noqa: E402

MODELS = {
    "mlp784": [784, 256, 10],
    "mlp3072": [3072, 1024, 1024, 10],
    "wide": [4096, 4096, 4096, 4096, 1000],
    "odd": [33, 7, 1, 5],
}


@pytest.mark.parametrize("model", sorted(MODELS))
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_layout_blocks(model, world):
    dims = MODELS[model]
    lay = nn.FlatLayout(dims, shard_world=world)
    prev_end = 0
    for i in range(lay.L):
        ws, we = lay.w_range(i)
        bs, be = lay.b_range(i)
        assert ws % 64 == 0 and bs % 64 == 0          # 256-byte aligned blocks
        assert we - ws == dims[i] * dims[i + 1] and be - bs == dims[i + 1]
        assert ws >= prev_end and bs >= we             # in order, no overlap
        prev_end = be
    assert prev_end <= lay.n_flat
    assert lay.grads_buf_len == 64 + lay.n_flat
    # buckets tile the gradient buffer and split evenly over the ranks
    end = 0
    for i in range(lay.L):
        s, e = lay.bucket(i)
        assert s == end and (e - s) % (64 * world) == 0
        end = e
    assert end == lay.grads_buf_len


@pytest.mark.parametrize("model", sorted(MODELS))
def test_one_rank_layout_is_unpadded(model):
    dims = MODELS[model]
    lay = nn.FlatLayout(dims)
    off = 0
    for i in range(lay.L):
        assert lay.w_off[i] == off
        off += -(-dims[i] * dims[i + 1] // 64) * 64
        assert lay.b_off[i] == off
        off += -(-dims[i + 1] // 64) * 64
    assert lay.n_flat == off


@pytest.mark.parametrize("model", sorted(MODELS))
@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_plan_partitions(model, world):
    lay = nn.FlatLayout(MODELS[model], shard_world=world)
    plans = [nn.ShardPlan(lay, world, r) for r in range(world)]
    for i in range(lay.L):
        s, e = lay.bucket(i)
        pieces = sorted(p.pieces[i] for p in plans)
        assert pieces[0][0] == s and pieces[-1][1] == e
        for (a0, b0), (a1, _b1) in zip(pieces, pieces[1:]):
            assert b0 == a1
        assert len({b - a for a, b in pieces}) == 1   # equal sizes
        assert all(a % 64 == 0 for a, _ in pieces)
    ranges = sorted(r for p in plans for r in p.update_ranges())
    assert ranges[0][0] == 64 and ranges[-1][1] == lay.grads_buf_len
    for (a0, b0), (a1, _b1) in zip(ranges, ranges[1:]):
        assert b0 == a1                                # every parameter once


def test_shard_plan_rejects_unpadded_layout():
    with pytest.raises(ValueError):
        nn.ShardPlan(nn.FlatLayout([784, 256, 10]), 2, 0)
