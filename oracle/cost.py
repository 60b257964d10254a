"""TEST INFRASTRUCTURE ONLY: numpy float32 restatement of RF-DETR's matcher cost.

This is the parity oracle for the CUDA cost kernel.  It follows the reference's
unfused op chain ``reference_matcher_cost`` (kernels_matcher.py:237-264) term by
term and in the same order of float32 operations:

* class gather of the logit at the (clamped, kernels_matcher.py:133-134) label;
* ``p = sigmoid(x)``; focal cost with gamma 2 (kernels_matcher.py:49-50):
  ``alpha * (1-p)**2 * -logsigmoid(x)  -  (1-alpha) * p**2 * -logsigmoid(-x)``
  (kernels_matcher.py:257-260);
* ``torch.cdist(p=1)`` on cxcywh boxes (kernels_matcher.py:262);
* cxcywh -> xyxy, then GIoU with the union and enclosing area clamped at 1e-7
  (kernels_matcher.py:105-127, the formulation the reference kernel documents as
  upstream's ``generalized_box_iou``);
* ``cost_bbox * l1 + cost_class * class + cost_giou * (-giou)``
  (kernels_matcher.py:264).

rf-detr's own ``box_ops`` is not vendored in the reference, so the box formulas
are restated here from the math above; ``tests/golden`` pins this module against
fixtures produced with torch's own operators (the ones the reference chain calls).

The compact layout is the one ``patches.py:149`` builds: row ``q`` of the
``[Q, sum T]`` matrix holds image ``b``'s targets in columns ``off[b]:off[b+1]``.

Only tests, ``__graft_entry__.smoke`` and the benchmark's CPU-baseline leg use it.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
BOX_EPS = F32(1e-7)


def _logsigmoid(x: np.ndarray) -> np.ndarray:
    """``min(x, 0) - log1p(exp(-|x|))`` in float32 (the stable logsigmoid)."""
    x = x.astype(F32, copy=False)
    return (np.minimum(x, F32(0)) - np.log1p(np.exp(-np.abs(x)))).astype(F32)


def _sigmoid(x: np.ndarray) -> np.ndarray:
    x = x.astype(F32, copy=False)
    return (F32(1) / (F32(1) + np.exp(-x))).astype(F32)


def focal_cost(logit: np.ndarray, alpha: float) -> np.ndarray:
    """Focal classification cost of a gathered logit (kernels_matcher.py:257-260)."""
    x = logit.astype(F32)
    p = _sigmoid(x)
    a = F32(alpha)
    # torch multiplies by the Python scalar (1 - alpha), rounded once to float32
    neg = F32(1.0 - alpha) * (p * p) * (-_logsigmoid(-x))
    pos = a * ((F32(1) - p) * (F32(1) - p)) * (-_logsigmoid(x))
    return (pos - neg).astype(F32)


def cxcywh_to_xyxy(b: np.ndarray) -> np.ndarray:
    cx, cy, w, h = (b[..., k].astype(F32) for k in range(4))
    half = F32(0.5)
    return np.stack([cx - half * w, cy - half * h, cx + half * w, cy + half * h], axis=-1).astype(F32)


def giou_pairwise(pred_xyxy: np.ndarray, tgt_xyxy: np.ndarray) -> np.ndarray:
    """GIoU of every pred [Q,4] against every target [T,4] (kernels_matcher.py:115-127)."""
    p = pred_xyxy[:, None, :]
    t = tgt_xyxy[None, :, :]
    area_p = (p[..., 2] - p[..., 0]) * (p[..., 3] - p[..., 1])
    area_t = (t[..., 2] - t[..., 0]) * (t[..., 3] - t[..., 1])
    inter_w = np.minimum(p[..., 2], t[..., 2]) - np.maximum(p[..., 0], t[..., 0])
    inter_h = np.minimum(p[..., 3], t[..., 3]) - np.maximum(p[..., 1], t[..., 1])
    inter = np.maximum(inter_w, F32(0)) * np.maximum(inter_h, F32(0))
    union = (area_p + area_t) - inter
    iou = inter / np.maximum(union, BOX_EPS)
    enc_w = np.maximum(p[..., 2], t[..., 2]) - np.minimum(p[..., 0], t[..., 0])
    enc_h = np.maximum(p[..., 3], t[..., 3]) - np.minimum(p[..., 1], t[..., 1])
    enclose = np.maximum(enc_w, F32(0)) * np.maximum(enc_h, F32(0))
    return (iou - (enclose - union) / np.maximum(enclose, BOX_EPS)).astype(F32)


def l1_pairwise(pred: np.ndarray, tgt: np.ndarray) -> np.ndarray:
    """``torch.cdist(pred, tgt, p=1)`` for 4-wide boxes, summed in feature order."""
    d = np.abs(pred[:, None, :].astype(F32) - tgt[None, :, :].astype(F32))
    return (((d[..., 0] + d[..., 1]) + d[..., 2]) + d[..., 3]).astype(F32)


def image_cost(
    pred_logits: np.ndarray,
    pred_boxes: np.ndarray,
    tgt_labels: np.ndarray,
    tgt_boxes: np.ndarray,
    *,
    cost_class: float,
    cost_bbox: float,
    cost_giou: float,
    focal_alpha: float,
) -> np.ndarray:
    """Cost ``[Q, T]`` of one image: logits [Q,C], boxes [Q,4], labels [T], boxes [T,4]."""
    q, c = pred_logits.shape
    t = tgt_labels.shape[0]
    if t == 0:
        return np.zeros((q, 0), dtype=F32)
    labels = np.clip(tgt_labels.astype(np.int64), 0, c - 1)
    gathered = pred_logits.astype(F32)[:, labels]
    class_cost = focal_cost(gathered, focal_alpha)
    l1 = l1_pairwise(pred_boxes, tgt_boxes)
    giou = giou_pairwise(cxcywh_to_xyxy(pred_boxes), cxcywh_to_xyxy(tgt_boxes))
    out = F32(cost_bbox) * l1 + F32(cost_class) * class_cost + F32(cost_giou) * (-giou)
    return out.astype(F32)


def compact_cost(
    pred_logits: np.ndarray,
    pred_boxes: np.ndarray,
    tgt_labels: list[np.ndarray],
    tgt_boxes: list[np.ndarray],
    *,
    cost_class: float,
    cost_bbox: float,
    cost_giou: float,
    focal_alpha: float,
) -> np.ndarray:
    """Compact cost ``[L, Q, sum T]`` for logits [L,B,Q,C] / boxes [L,B,Q,4] (patches.py:149)."""
    layers, images, queries, _ = pred_logits.shape
    sizes = [int(x.shape[0]) for x in tgt_labels]
    out = np.zeros((layers, queries, sum(sizes)), dtype=F32)
    for layer in range(layers):
        col = 0
        for b in range(images):
            t = sizes[b]
            if t:
                out[layer, :, col : col + t] = image_cost(
                    pred_logits[layer, b],
                    pred_boxes[layer, b],
                    tgt_labels[b],
                    tgt_boxes[b],
                    cost_class=cost_class,
                    cost_bbox=cost_bbox,
                    cost_giou=cost_giou,
                    focal_alpha=focal_alpha,
                )
            col += t
    return out
