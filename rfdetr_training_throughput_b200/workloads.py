"""Seeded synthetic matcher inputs with the shapes and value distributions of the
five benchmark configurations of this path (no dataset is used; the reference's
production data is not available, so these stand in for it).

=====  ==========================================================================
name   what it is
=====  ==========================================================================
cpu1   1 image x 300 queries, 1 group, 2 classes, logits ~N(0, 1.5),
       T = 12 (the CPU-runnable single problem)
step   RF-DETR Medium matcher step: 5 decoder layers x 8 images x 13 groups of
       300 queries, 2 classes, logits ~N(-2, 1.5), T ~ Poisson(8) clipped to
       [1, 60] -> 520 problems
crowd  16 images x 13 groups x 300 queries, 91 classes, logits ~N(-3, 2),
       T ~ U[100, 300], target w/h ~ U(0.01, 0.2) -> 208 near-square problems
ties   8 images x 13 groups x 300 queries, 2 classes, boxes on a 1/16 grid, 30 %
       of queries exact duplicates of others, logits in {-2, 0, 2}, and images
       with T = 0, 1 and 300
sweep  1024 images x 13 groups x 300 queries, 2 classes, distributions as
       ``step`` -> 13,312 problems (the sharded throughput sweep)
=====  ==========================================================================

Predicted boxes are ``sigmoid(N(0, 1))`` per coordinate; target centres are
``U(0.1, 0.9)`` and sizes ``U(0.02, 0.5)`` unless stated.  Cost weights: class 2,
bbox 5, giou 2, focal alpha 0.25.  Everything is generated on the host with a
``torch.Generator`` seeded by the configuration index (plus an optional shard).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

WEIGHTS = {"cost_class": 2.0, "cost_bbox": 5.0, "cost_giou": 2.0, "focal_alpha": 0.25}
GROUP_WIDTH = 300


@dataclass
class Workload:
    name: str
    layers: int
    images: int
    group_detr: int
    classes: int
    pred_logits: torch.Tensor  # [L, B, Q, C] float32 (host)
    pred_boxes: torch.Tensor  # [L, B, Q, 4] float32 cxcywh (host)
    targets: list = field(default_factory=list)  # [{"labels": int64 [T], "boxes": float32 [T, 4]}]
    weights: dict = field(default_factory=lambda: dict(WEIGHTS))

    @property
    def queries(self) -> int:
        return self.pred_logits.shape[2]

    @property
    def sizes(self) -> list[int]:
        return [int(t["labels"].shape[0]) for t in self.targets]

    @property
    def num_problems(self) -> int:
        return self.layers * self.group_detr * sum(1 for s in self.sizes if s > 0)

    def outputs_list(self, device=None) -> list[dict]:
        lg = self.pred_logits if device is None else self.pred_logits.to(device)
        bx = self.pred_boxes if device is None else self.pred_boxes.to(device)
        return [{"pred_logits": lg[l], "pred_boxes": bx[l]} for l in range(self.layers)]

    def targets_on(self, device=None) -> list[dict]:
        if device is None:
            return self.targets
        return [{"labels": t["labels"].to(device), "boxes": t["boxes"].to(device)} for t in self.targets]


def _uniform(g: torch.Generator, shape, lo: float, hi: float) -> torch.Tensor:
    return torch.rand(shape, generator=g) * (hi - lo) + lo


def _targets(g: torch.Generator, sizes, classes: int, wh=(0.02, 0.5), quant: float | None = None):
    out = []
    for t in sizes:
        centers = _uniform(g, (t, 2), 0.1, 0.9)
        whs = _uniform(g, (t, 2), wh[0], wh[1])
        boxes = torch.cat([centers, whs], dim=-1)
        if quant:
            boxes = torch.round(boxes * quant) / quant
        labels = torch.randint(0, classes, (t,), generator=g, dtype=torch.int64)
        out.append({"labels": labels, "boxes": boxes.to(torch.float32).contiguous()})
    return out


def _poisson_sizes(g: torch.Generator, n: int, lam: float, lo: int, hi: int) -> list[int]:
    s = torch.poisson(torch.full((n,), float(lam)), generator=g).to(torch.int64).clamp(lo, hi)
    return [int(x) for x in s]


def make(name: str, *, shard: int = 0, images: int | None = None, layers: int | None = None,
         group_detr: int | None = None) -> Workload:
    """Build a named workload.  ``shard`` reseeds it (per-rank shards of the sweep);
    ``images``/``layers``/``group_detr`` shrink it for reduced test cases."""
    seeds = {"cpu1": 0, "step": 1, "crowd": 2, "ties": 3, "sweep": 4}
    if name not in seeds:
        raise KeyError(f"unknown workload {name!r}; choose from {sorted(seeds)}")
    g = torch.Generator().manual_seed(1000 * seeds[name] + 7919 * shard)
    if name == "cpu1":
        L, B, G, C = layers or 1, images or 1, 1, 2
        sizes = [12] * B
        mean, std = 0.0, 1.5
    elif name == "step":
        L, B, G, C = layers or 5, images or 8, 13, 2
        sizes = _poisson_sizes(g, B, 8.0, 1, 60)
        mean, std = -2.0, 1.5
    elif name == "crowd":
        L, B, G, C = layers or 1, images or 16, 13, 91
        sizes = [int(x) for x in torch.randint(100, 301, (B,), generator=g)]
        mean, std = -3.0, 2.0
    elif name == "ties":
        L, B, G, C = layers or 1, images or 8, 13, 2
        fixed = [0, 1, 300]
        rest = [int(x) for x in torch.randint(2, 41, (max(B - 3, 0),), generator=g)]
        sizes = (fixed + rest)[:B]
        mean, std = 0.0, 0.0
    else:  # sweep
        L, B, G, C = layers or 1, images or 1024, 13, 2
        sizes = _poisson_sizes(g, B, 8.0, 1, 60)
        mean, std = -2.0, 1.5
    G = group_detr or G
    Q = G * GROUP_WIDTH

    if name == "ties":
        logits = (torch.randint(0, 3, (L, B, Q, C), generator=g) * 2 - 2).to(torch.float32)
        boxes = torch.sigmoid(torch.randn((L, B, Q, 4), generator=g))
        boxes = torch.round(boxes * 16) / 16
        ndup = int(0.3 * Q)
        for l in range(L):
            for b in range(B):
                dst = torch.randperm(Q, generator=g)[:ndup]
                src = torch.randint(0, Q, (ndup,), generator=g)
                logits[l, b, dst] = logits[l, b, src]
                boxes[l, b, dst] = boxes[l, b, src]
        targets = _targets(g, sizes, C, quant=16.0)
    else:
        logits = torch.randn((L, B, Q, C), generator=g) * std + mean
        boxes = torch.sigmoid(torch.randn((L, B, Q, 4), generator=g))
        wh = (0.01, 0.2) if name == "crowd" else (0.02, 0.5)
        targets = _targets(g, sizes, C, wh=wh)
    return Workload(name, L, B, G, C, logits.to(torch.float32).contiguous(),
                    boxes.to(torch.float32).contiguous(), targets)
