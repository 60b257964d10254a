"""TEST INFRASTRUCTURE ONLY: the reference's CPU matching path, timed as the CPU baseline.

This is what RF-DETR runs when the matcher is left on the host (the configuration
the reference measures before its kernels): the unfused torch op chain of
``reference_matcher_cost`` (kernels_matcher.py:237-264) evaluated on CPU tensors
per image, then ``scipy.optimize.linear_sum_assignment`` per (image, group) block
on a thread pool, as the parallel_lap patch does (patches.py:186-232: a
``ThreadPoolExecutor`` of ``LAP_THREADS`` workers, serial below 8 problems).

rf-detr's ``box_ops`` is not vendored, so ``box_cxcywh_to_xyxy`` and
``generalized_box_iou`` are restated here with torch ops (the 1e-7 clamps of
kernels_matcher.py:121-127).  Only ``bench.py``'s CPU legs and the tests use it.
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch
import torch.nn.functional as F

FOCAL_GAMMA = 2.0
MIN_POOL_BATCH = 8


def box_cxcywh_to_xyxy(b: torch.Tensor) -> torch.Tensor:
    cx, cy, w, h = b.unbind(-1)
    return torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], dim=-1)


def generalized_box_iou(b1: torch.Tensor, b2: torch.Tensor) -> torch.Tensor:
    area1 = (b1[:, 2] - b1[:, 0]) * (b1[:, 3] - b1[:, 1])
    area2 = (b2[:, 2] - b2[:, 0]) * (b2[:, 3] - b2[:, 1])
    lt = torch.max(b1[:, None, :2], b2[:, :2])
    rb = torch.min(b1[:, None, 2:], b2[:, 2:])
    wh = (rb - lt).clamp(min=0)
    inter = wh[..., 0] * wh[..., 1]
    union = area1[:, None] + area2 - inter
    iou = inter / union.clamp(min=1e-7)
    lt2 = torch.min(b1[:, None, :2], b2[:, :2])
    rb2 = torch.max(b1[:, None, 2:], b2[:, 2:])
    wh2 = (rb2 - lt2).clamp(min=0)
    area = wh2[..., 0] * wh2[..., 1]
    return iou - (area - union) / area.clamp(min=1e-7)


def image_cost(logits: torch.Tensor, boxes: torch.Tensor, labels: torch.Tensor, tboxes: torch.Tensor,
               *, cost_class: float, cost_bbox: float, cost_giou: float, focal_alpha: float) -> torch.Tensor:
    """The reference op chain for one image: logits [Q,C], boxes [Q,4] vs labels [T], boxes [T,4]."""
    labels = labels.clamp(0, logits.shape[-1] - 1)
    target_logits = logits[:, labels]
    probabilities = target_logits.sigmoid()
    negative_cost = (1 - focal_alpha) * (probabilities**FOCAL_GAMMA) * (-F.logsigmoid(-target_logits))
    positive_cost = focal_alpha * ((1 - probabilities) ** FOCAL_GAMMA) * (-F.logsigmoid(target_logits))
    class_cost = positive_cost - negative_cost
    bbox_cost = torch.cdist(boxes, tboxes, p=1)
    giou_cost = -generalized_box_iou(box_cxcywh_to_xyxy(boxes), box_cxcywh_to_xyxy(tboxes))
    return cost_bbox * bbox_cost + cost_class * class_cost + cost_giou * giou_cost


def compact_cost(pred_logits: torch.Tensor, pred_boxes: torch.Tensor, targets, weights: dict) -> torch.Tensor:
    """[L, Q, sum T] compact cost from logits [L,B,Q,C] on the CPU (patches.py:149 layout)."""
    layers = pred_logits.shape[0]
    per_layer = []
    for l in range(layers):
        cols = [image_cost(pred_logits[l, b], pred_boxes[l, b], t["labels"], t["boxes"], **weights)
                for b, t in enumerate(targets) if t["labels"].shape[0]]
        per_layer.append(torch.cat(cols, dim=-1) if cols else pred_logits.new_zeros((pred_logits.shape[2], 0)))
    return torch.stack(per_layer)


class CpuMatcher:
    """torch-CPU cost chain + SciPy per (image, group) block on a thread pool.

    ``threads=1`` is the serial path: every block solved in turn in the calling
    thread, as the parallel_lap patch does below its pool threshold
    (patches.py:207-211) and as the unpatched matcher does always."""

    def __init__(self, threads: int | None = None):
        from scipy.optimize import linear_sum_assignment

        self._solve = linear_sum_assignment
        self.threads = int(threads or os.environ.get("LAP_THREADS", "8"))
        self.pool = ThreadPoolExecutor(max_workers=self.threads, thread_name_prefix="lap") if self.threads > 1 else None

    def close(self) -> None:
        if self.pool is not None:
            self.pool.shutdown(wait=True)

    def match(self, pred_logits: torch.Tensor, pred_boxes: torch.Tensor, targets, group_detr: int,
              weights: dict):
        cost = compact_cost(pred_logits, pred_boxes, targets, weights).numpy()
        sizes = [int(t["labels"].shape[0]) for t in targets]
        qg = cost.shape[1] // group_detr
        blocks, keys = [], []
        for l in range(cost.shape[0]):
            col = 0
            for b, t in enumerate(sizes):
                for g in range(group_detr if t else 0):
                    blocks.append(cost[l, g * qg:(g + 1) * qg, col:col + t])
                    keys.append((l, b, g))
                col += t
        if self.pool is None or len(blocks) < MIN_POOL_BATCH:
            solved = list(map(self._solve, blocks))
        else:
            solved = list(self.pool.map(self._solve, blocks))
        out = [[([], []) for _ in sizes] for _ in range(cost.shape[0])]
        for (l, b, g), (r, c) in zip(keys, solved):
            out[l][b][0].append(r + g * qg)
            out[l][b][1].append(c)
        return [[(np.concatenate(q) if q else np.zeros(0, np.int64), np.concatenate(t) if t else np.zeros(0, np.int64))
                 for q, t in layer] for layer in out]
