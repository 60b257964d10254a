"""Image-sharded matcher sweep over several GPUs with an all-gather of the index pairs.

A large batch of images is split into contiguous, balanced image ranges, one per
rank (each image's ``layers x groups`` problems are independent, so there is no
exchange during matching).  Every rank matches its range with ``match_packed`` and
the packed int64 pairs of all ranks are then gathered with one
``all_gather_into_tensor`` (NCCL over NVLink on GPUs, gloo in the CPU tests), so
every rank ends with the whole batch's per-image ``(query_idx, target_idx)``.
Sizes are known on every host, so the gather needs no count exchange: each
rank's chunk is padded to the largest rank's pair count.
"""

from __future__ import annotations

from functools import lru_cache
from typing import Callable, Sequence

import numpy as np
import torch
import torch.distributed as dist


def shard_bounds(num_images: int, world: int) -> list[tuple[int, int]]:
    """Contiguous image ranges ``[start, end)`` per rank; sizes differ by at most one."""
    if world < 1:
        raise ValueError("world size must be >= 1")
    base, extra = divmod(num_images, world)
    bounds, start = [], 0
    for r in range(world):
        end = start + base + (1 if r < extra else 0)
        bounds.append((start, end))
        start = end
    return bounds


def pairs_per_image(sizes: Sequence[int], layers: int, queries: int, group_detr: int) -> np.ndarray:
    """Host-known pair count of every (layer, image): ``group_detr * min(Q/G, T_b)``."""
    qg = queries // group_detr
    per = group_detr * np.minimum(np.asarray(sizes, dtype=np.int64), qg)
    return np.tile(per, layers)


@lru_cache(maxsize=64)
def _layout(sizes: tuple[int, ...], layers: int, queries: int, group_detr: int, world: int):
    """Host-only split of a batch: image bounds, pair count per rank, per-(layer, image) counts."""
    bounds = shard_bounds(len(sizes), world)
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    counts, per = [], []
    for a, b in bounds:
        pi = pairs_per_image(sizes[a:b], layers, queries, group_detr)
        counts.append(int(pi.sum()))
        per.extend(int(x) for x in pi)
    return bounds, offsets, counts, per


def gather_pairs(local_pairs: torch.Tensor, counts: Sequence[int], group=None) -> torch.Tensor:
    """All-gather ``[2, counts[rank]]`` int64 chunks; returns ``[2, sum(counts)]`` in rank order."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    width = max(int(c) for c in counts) if counts else 0
    send = torch.zeros((2, width), dtype=local_pairs.dtype, device=local_pairs.device)
    n = int(counts[rank])
    if n:
        send[:, :n] = local_pairs[:, :n]
    recv = torch.empty((world, 2, width), dtype=local_pairs.dtype, device=local_pairs.device)
    dist.all_gather_into_tensor(recv, send.unsqueeze(0).contiguous(), group=group)
    return torch.cat([recv[r, :, : int(counts[r])] for r in range(world)], dim=1)


def sharded_match(pred_logits: torch.Tensor, pred_boxes: torch.Tensor, labels: torch.Tensor,
                  boxes: torch.Tensor, sizes: Sequence[int], group_detr: int, *,
                  weights: dict | None = None, group=None,
                  local_solver: Callable | None = None) -> tuple[torch.Tensor, list[int]]:
    """Match a batch split by image across the ranks of ``group``.

    ``pred_logits`` ``[L, B, Q, C]`` / ``pred_boxes`` ``[L, B, Q, 4]`` and the packed
    ``labels``/``boxes`` may hold the whole batch or only this rank's image range
    (detected from the leading image dimension).  Returns the gathered ``[2, total]``
    pairs (per rank, layer-major, images in order) and the per-(layer, image) pair
    counts in the same order.  ``local_solver(logits, boxes, labels, boxes, sizes,
    group_detr) -> [2, n]`` replaces the device step (used by CPU tests).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = tuple(int(s) for s in sizes)
    layers, nimg_in, queries, _ = pred_logits.shape
    bounds, offsets, counts, per = _layout(sizes, layers, queries, group_detr, world)
    lo, hi = bounds[rank]
    if nimg_in == len(sizes):  # whole batch given: slice this rank's images and targets
        pred_logits = pred_logits[:, lo:hi]
        pred_boxes = pred_boxes[:, lo:hi]
        labels = labels[offsets[lo]:offsets[hi]]
        boxes = boxes[offsets[lo]:offsets[hi]]
    elif nimg_in != hi - lo:
        raise ValueError(f"rank {rank} holds {nimg_in} images, its shard has {hi - lo}")
    local_sizes = sizes[lo:hi]
    if local_solver is None:
        from .matcher import PackedTargets, match_packed

        res = match_packed(pred_logits, pred_boxes, PackedTargets(labels, boxes, local_sizes), group_detr,
                           weights=weights)
        local = res.pairs
    else:
        local = local_solver(pred_logits, pred_boxes, labels, boxes, list(local_sizes), group_detr)
    return gather_pairs(local, counts, group), per
