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
        if rank == 0:
            np.savez(result_path, pairs=pairs.numpy(), per=np.asarray(per))
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
