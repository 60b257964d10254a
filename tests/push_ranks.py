"""Rank program of the two-GPU pushed-exchange test (run by torch.distributed.run, one process per
GPU; not collected by pytest).  ShardedMatcher with the pushed exchange must return exactly the
pairs of the NCCL all-gather, step after step with alternating inputs, and those of one GPU's
match_packed over the whole batch."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from rfdetr_training_throughput_b200 import matcher, sharded, workloads  # noqa: E402


def main() -> None:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    wl = workloads.make("sweep", images=int(os.environ.get("PUSH_IMAGES", "96")))
    lo, hi = sharded.shard_bounds(wl.images, world)[rank]
    sizes = tuple(wl.sizes)
    offs = [0]
    for s in sizes:
        offs.append(offs[-1] + s)
    labels = torch.cat([t["labels"] for t in wl.targets]).to(dev)
    tboxes = torch.cat([t["boxes"] for t in wl.targets]).to(dev)
    full = [(wl.pred_logits.to(dev), wl.pred_boxes.to(dev)),
            (wl.pred_logits.roll(7, dims=2).to(dev), wl.pred_boxes.roll(7, dims=2).to(dev))]
    packed = matcher.PackedTargets.from_list(wl.targets_on(dev), dev)
    expect = [matcher.match_packed(lg, bx, packed, wl.group_detr, weights=wl.weights).pairs for lg, bx in full]
    local_in = [(lg[:, lo:hi].contiguous(), bx[:, lo:hi].contiguous()) for lg, bx in full]
    lab, box = labels[offs[lo]:offs[hi]].contiguous(), tboxes[offs[lo]:offs[hi]].contiguous()
    kw = dict(weights=wl.weights, device=dev)
    nccl = sharded.ShardedMatcher(sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, **kw)
    push = sharded.ShardedMatcher(sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, exchange="push", **kw)
    try:
        for step in range(6):
            lg, bx = local_in[step % 2]
            a = nccl(lg, bx, lab, box)
            b = push(lg, bx, lab, box, padded=True)
            torch.cuda.synchronize()
            assert torch.equal(a, b.flat()), f"rank {rank} step {step}: pushed pairs differ from the all-gather"
            assert torch.equal(a, expect[step % 2]), f"rank {rank} step {step}: pairs differ from match_packed"
        push.check()
    finally:
        push.close()
        nccl.graph = None
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}/{world}: pushed exchange equals the all-gather", flush=True)


if __name__ == "__main__":
    main()
