"""Image-sharded sweep: shard bounds and the all-gather assembly, on gloo CPU ranks (no GPU)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rfdetr_training_throughput_b200 import sharded, workloads


def test_shard_bounds_cover_and_balance():
    for n, w in [(1024, 8), (13, 4), (3, 5), (0, 2)]:
        b = sharded.shard_bounds(n, w)
        assert len(b) == w and b[0][0] == 0 and b[-1][1] == n
        assert all(b[i][1] == b[i + 1][0] for i in range(w - 1))
        sizes = [e - s for s, e in b]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharded.shard_bounds(4, 0)


def _cpu_solver(logits, boxes, labels, tboxes, sizes, group_detr):
    """CPU stand-in for the device step: oracle cost + C LSAP, packed like match_packed."""
    from oracle import cost as ocost
    from oracle.matcher import solve_blocks

    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    lab = [labels[offs[i]:offs[i + 1]].numpy() for i in range(len(sizes))]
    bx = [tboxes[offs[i]:offs[i + 1]].numpy() for i in range(len(sizes))]
    cost = ocost.compact_cost(logits.numpy(), boxes.numpy(), lab, bx, **workloads.WEIGHTS)
    qs, ts = [], []
    for l in range(cost.shape[0]):
        for q, t in solve_blocks(cost[l], sizes, group_detr):
            qs.append(q)
            ts.append(t)
    q = np.concatenate(qs) if qs else np.zeros(0, np.int64)
    t = np.concatenate(ts) if ts else np.zeros(0, np.int64)
    return torch.from_numpy(np.stack([q, t]))


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wl = workloads.make("step", layers=2, images=5, group_detr=2)
        labels = torch.cat([t["labels"] for t in wl.targets])
        boxes = torch.cat([t["boxes"] for t in wl.targets])
        pairs, per = sharded.sharded_match(wl.pred_logits, wl.pred_boxes, labels, boxes, wl.sizes, wl.group_detr,
                                           local_solver=_cpu_solver)
        gathered, per2 = sharded.sharded_match(wl.pred_logits, wl.pred_boxes, labels, boxes, wl.sizes,
                                               wl.group_detr, local_solver=_cpu_solver, padded=True)
        # the padded result holds the same pairs: flat() and the per-image views of every layer
        flat = gathered.flat()
        views = [torch.cat([torch.stack([q, t]) for q, t in gathered.layer(l)], dim=1) for l in range(wl.layers)]
        if rank == 0:
            np.savez(result_path, pairs=pairs.numpy(), per=np.asarray(per), flat=flat.numpy(),
                     per2=np.asarray(per2), views=[v.numpy() for v in views])
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_match_on_two_gloo_ranks(tmp_path):
    path = str(tmp_path / "gathered.npz")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    got = np.load(path)
    wl = workloads.make("step", layers=2, images=5, group_detr=2)
    labels = torch.cat([t["labels"] for t in wl.targets])
    boxes = torch.cat([t["boxes"] for t in wl.targets])
    # single-process reference, reordered the way the shards concatenate: rank, then layer, then image
    bounds = sharded.shard_bounds(wl.images, 2)
    offs = np.concatenate([[0], np.cumsum(wl.sizes)])
    expect = []
    for a, b in bounds:
        expect.append(_cpu_solver(wl.pred_logits[:, a:b], wl.pred_boxes[:, a:b], labels[offs[a]:offs[b]],
                                  boxes[offs[a]:offs[b]], wl.sizes[a:b], wl.group_detr).numpy())
    expect = np.concatenate(expect, axis=1)
    assert np.array_equal(got["pairs"], expect)
    assert int(got["per"].sum()) == expect.shape[1]
    assert np.array_equal(got["flat"], expect) and np.array_equal(got["per2"], got["per"])
    # per-layer views: every rank's block of that layer, ranks in order (images in batch order)
    per = [int(c) for c in got["per"]]
    first_pair, first_count = 0, 0
    rank_blocks = []  # (pairs of the rank, its per-(layer, image) counts)
    for a, b in bounds:
        counts = per[first_count:first_count + (b - a) * wl.layers]
        rank_blocks.append((expect[:, first_pair:first_pair + sum(counts)], counts, b - a))
        first_pair += sum(counts)
        first_count += len(counts)
    for l in range(wl.layers):
        pieces = []
        for pairs_r, counts, n in rank_blocks:
            off = sum(counts[: l * n])
            pieces.append(pairs_r[:, off:off + sum(counts[l * n:(l + 1) * n])])
        assert np.array_equal(got["views"][l], np.concatenate(pieces, axis=1)), l


def test_exchange_layout():
    """Two [world, 2, width] int64 buffers, then the flag block on a 256-byte boundary."""
    for world, width in ((1, 0), (1, 7), (2, 100), (8, 13_000)):
        lay = sharded.exchange_layout(world, width)
        assert lay["parity_elems"] == world * 2 * width
        assert lay["flags"] % 256 == 0 and lay["flags"] >= 2 * lay["parity_elems"] * 8
        assert lay["epoch"] == lay["flags"] + 32 and lay["error"] == lay["flags"] + 36
        assert lay["bytes"] == lay["flags"] + 256
    for world in (0, 9):
        with pytest.raises(ValueError):
            sharded.exchange_layout(world, 4)
    with pytest.raises(ValueError):
        sharded.ShardedMatcher((3, 4), 1, 300, 2, 1, exchange="ring")
