"""Loading helpers for the fixtures under tests/golden (see make_golden.py)."""

from __future__ import annotations

import json
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def index() -> list[dict]:
    with open(os.path.join(GOLDEN, "index.json")) as f:
        return json.load(f)


def names(kind: str) -> list[str]:
    return [c["name"] for c in index() if c["kind"] == kind]


def load(name: str):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def matcher_case(name: str):
    """(logits [L,B,Q,C], boxes [L,B,Q,4], labels list, boxes list, group_detr, weights, cost, pairs)."""
    z = load(name)
    sizes = [int(s) for s in z["sizes"]]
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    labels = [z["labels"][offs[i]:offs[i + 1]] for i in range(len(sizes))]
    boxes = [z["tgt_boxes"][offs[i]:offs[i + 1]] for i in range(len(sizes))]
    weights = dict(zip(("cost_class", "cost_bbox", "cost_giou", "focal_alpha"), (float(x) for x in z["weights"])))
    layers = z["cost"].shape[0]
    pairs = [(z[f"q_{l}"], z[f"t_{l}"]) for l in range(layers)]
    return z["pred_logits"], z["pred_boxes"], labels, boxes, int(z["group_detr"]), weights, z["cost"], pairs


def lsap_case(name: str):
    """List of (matrix, result, rows, cols) with result in {"ok", "infeasible", "invalid"}."""
    z = load(name)
    out = []
    for i, res in enumerate(z["results"]):
        res = str(res)
        out.append((z[f"m_{i}"], res, z[f"r_{i}"] if res == "ok" else None, z[f"c_{i}"] if res == "ok" else None))
    return out


def to_targets(labels, boxes, device) -> list[dict]:
    return [{"labels": torch.as_tensor(l, dtype=torch.int64, device=device),
             "boxes": torch.as_tensor(b, dtype=torch.float32, device=device)} for l, b in zip(labels, boxes)]
