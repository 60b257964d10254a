"""TEST INFRASTRUCTURE ONLY: the whole ``HungarianMatcher.forward`` step on the CPU.

For every layer, image and query group it takes the ``[Q/G, T_b]`` block of the
numpy compact cost (``oracle.cost``) and solves it with the C restatement of
SciPy's ``rectangular_lsap`` (``oracle.lsap``), adding the group offset
``g * Q/G`` to the query indices and concatenating the groups in order -- the
per-(image, group) solve of rf-detr's matcher as the device path of patches.py
reproduces it (patches.py:371, 398, 406-418), in SciPy's row order.

``solve_blocks`` takes an already computed compact cost (for instance the one the
GPU produced) so that assignments can be compared on the same matrix.
"""

from __future__ import annotations

import numpy as np

from oracle import cost as ocost
from oracle.lsap import linear_sum_assignment


def solve_blocks(cost: np.ndarray, sizes, group_detr: int, solver=linear_sum_assignment):
    """Per-image ``(query_idx, target_idx)`` int64 arrays for one layer's compact cost [Q, sum T]."""
    queries = cost.shape[0]
    qg = queries // group_detr
    out = []
    col = 0
    for t in sizes:
        qs, ts = [], []
        if t:
            for g in range(group_detr):
                block = cost[g * qg:(g + 1) * qg, col:col + t]
                r, c = solver(block)
                qs.append(np.asarray(r, dtype=np.int64) + g * qg)
                ts.append(np.asarray(c, dtype=np.int64))
        col += t
        out.append((np.concatenate(qs) if qs else np.zeros(0, np.int64),
                    np.concatenate(ts) if ts else np.zeros(0, np.int64)))
    return out


def forward(pred_logits: np.ndarray, pred_boxes: np.ndarray, tgt_labels, tgt_boxes, group_detr: int,
            weights: dict):
    """Oracle matcher over logits [L,B,Q,C] / boxes [L,B,Q,4]; returns (per-layer pairs, compact cost)."""
    cost = ocost.compact_cost(pred_logits, pred_boxes, tgt_labels, tgt_boxes, **weights)
    sizes = [int(x.shape[0]) for x in tgt_labels]
    return [solve_blocks(cost[l], sizes, group_detr) for l in range(cost.shape[0])], cost
