"""Generate the golden fixtures of tests/golden (run in a container with SciPy; CPU only).

``python tests/golden/make_golden.py`` rewrites every ``*.npz`` here.  Each
fixture holds the inputs of one small matcher case and the expected outputs
produced with the operators the reference's own CPU chain calls:

* cost: ``torch.gather``/``sigmoid``/``F.logsigmoid``/``torch.cdist(p=1)`` and a
  torch ``generalized_box_iou`` (kernels_matcher.py:237-264), evaluated in float32
  by torch on the CPU (``oracle.cpu_path.image_cost``);
* assignment: ``scipy.optimize.linear_sum_assignment`` (SciPy 1.18.1), the solver
  the reference verifies against (kernels_lap.py:370-379) and runs on its CPU path
  (patches.py:213-229), per (image, group) block.

LSAP-only fixtures (``lsap_*``) hold a batch of matrices, SciPy's (rows, cols)
for each, or the error SciPy raised.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch
from scipy.optimize import linear_sum_assignment

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.cpu_path import compact_cost  # noqa: E402
from rfdetr_training_throughput_b200 import workloads  # noqa: E402


def scipy_blocks(cost: np.ndarray, sizes, group_detr: int):
    qg = cost.shape[0] // group_detr
    qs, ts, col = [], [], 0
    for t in sizes:
        q_img, t_img = [], []
        for g in range(group_detr if t else 0):
            r, c = linear_sum_assignment(cost[g * qg:(g + 1) * qg, col:col + t])
            q_img.append(r + g * qg)
            t_img.append(c)
        qs.append(np.concatenate(q_img).astype(np.int64) if q_img else np.zeros(0, np.int64))
        ts.append(np.concatenate(t_img).astype(np.int64) if t_img else np.zeros(0, np.int64))
        col += t
    return qs, ts


def save_matcher_case(name: str, wl: workloads.Workload) -> dict:
    cost = compact_cost(wl.pred_logits, wl.pred_boxes, wl.targets, wl.weights).numpy()
    sizes = wl.sizes
    arrays = {
        "pred_logits": wl.pred_logits.numpy(),
        "pred_boxes": wl.pred_boxes.numpy(),
        "sizes": np.asarray(sizes, np.int64),
        "labels": np.concatenate([t["labels"].numpy() for t in wl.targets]) if sum(sizes) else np.zeros(0, np.int64),
        "tgt_boxes": np.concatenate([t["boxes"].numpy() for t in wl.targets]) if sum(sizes) else np.zeros((0, 4), np.float32),
        "group_detr": np.asarray(wl.group_detr),
        "weights": np.asarray([wl.weights[k] for k in ("cost_class", "cost_bbox", "cost_giou", "focal_alpha")], np.float64),
        "cost": cost,
    }
    for l in range(cost.shape[0]):
        qs, ts = scipy_blocks(cost[l], sizes, wl.group_detr)
        arrays[f"q_{l}"] = np.concatenate(qs) if qs else np.zeros(0, np.int64)
        arrays[f"t_{l}"] = np.concatenate(ts) if ts else np.zeros(0, np.int64)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    return {"name": name, "kind": "matcher", "layers": int(cost.shape[0]), "sizes": sizes,
            "queries": int(cost.shape[1]), "group_detr": wl.group_detr}


def save_lsap_case(name: str, mats: list[np.ndarray]) -> dict:
    arrays, results = {}, []
    for i, m in enumerate(mats):
        m = np.ascontiguousarray(m, dtype=np.float32)
        arrays[f"m_{i}"] = m
        try:
            r, c = linear_sum_assignment(m)
            arrays[f"r_{i}"] = r.astype(np.int64)
            arrays[f"c_{i}"] = c.astype(np.int64)
            results.append("ok")
        except ValueError as e:
            results.append("infeasible" if "infeasible" in str(e) else "invalid")
    arrays["results"] = np.asarray(results)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    return {"name": name, "kind": "lsap", "count": len(mats)}


def degenerate(wl: workloads.Workload) -> workloads.Workload:
    """Zero-area predicted and target boxes (kernels_matcher.py:310-320)."""
    wl.pred_boxes[..., 2:] = 0.0
    for t in wl.targets:
        t["boxes"][:, 2:] = 0.0
    return wl


def main() -> None:
    index = []
    index.append(save_matcher_case("cpu1", workloads.make("cpu1")))
    index.append(save_matcher_case("step_small", workloads.make("step", layers=2, images=2)))
    index.append(save_matcher_case("ties_small", workloads.make("ties", images=4, group_detr=2)))
    index.append(save_matcher_case("crowd_small", workloads.make("crowd", images=2, group_detr=1)))
    index.append(save_matcher_case("degenerate", degenerate(workloads.make("step", layers=1, images=3, group_detr=1))))

    rng = np.random.default_rng(20)
    quant = [(rng.integers(0, 4, (300, 10)) / 4) for _ in range(3)]
    quant += [(rng.integers(0, 2, (300, 6)) / 2), (rng.integers(0, 4, (40, 40)) / 4),
              (rng.integers(0, 3, (30, 30)).astype(np.float64)), (rng.integers(0, 4, (12, 50)) / 4)]
    index.append(save_lsap_case("lsap_ties", [np.full((300, 8), 1.5)] + quant + [np.zeros((5, 5))]))
    near = []
    for _ in range(4):
        base = rng.standard_normal((60, 7)).astype(np.float32)
        base[rng.integers(0, 60, 10), rng.integers(0, 7, 10)] += np.float32(1e-6)
        near.append(base)
    index.append(save_lsap_case("lsap_near_ties", near))
    inf_case = rng.standard_normal((20, 5))
    inf_case[:, 2] = np.inf
    feasible_inf = rng.standard_normal((20, 5))
    feasible_inf[3:, 1] = np.inf
    nan_case = rng.standard_normal((10, 4))
    nan_case[4, 2] = np.nan
    neg_inf = rng.standard_normal((6, 6))
    neg_inf[1, 1] = -np.inf
    index.append(save_lsap_case("lsap_special", [inf_case, feasible_inf, nan_case, neg_inf,
                                                 rng.standard_normal((1, 1)), rng.standard_normal((1, 300)),
                                                 rng.standard_normal((300, 1))]))
    with open(os.path.join(HERE, "index.json"), "w") as f:
        json.dump(index, f, indent=1)


if __name__ == "__main__":
    main()
