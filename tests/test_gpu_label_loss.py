"""rfm_label_loss_forward / _backward against torch fp32 autograd restatements of the two
classification losses of the DETR-family criterion's loss_labels, evaluated on the pairs the device
matcher produced: Deformable DETR's sigmoid focal loss (one-hot targets at the matched classes) and
the IoU-aware BCE of LW-DETR / RF-DETR (soft target t = max(p^alpha u^(1-alpha), 0.01), detached).
rf-detr's criterion is not vendored, so the restatements follow those published formulas.

Tolerances: loss sums within 1e-5 relative; gradients within 1e-5 of the largest gradient
magnitude (elementwise float32 terms, different summation order).  The tie configuration has
matched pairs whose boxes both have zero area: their IoU is 0/0 = NaN and the IoU-aware loss of
that layer is NaN in both, with NaN gradients at exactly the same elements."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from rfdetr_training_throughput_b200 import matcher, workloads
from rfdetr_training_throughput_b200.loss import criterion_loss_labels, matched_label_losses

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _xyxy(b):
    cx, cy, w, h = b.unbind(-1)
    return torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], dim=-1)


def _pair_iou(p, t):
    """Diagonal of box_iou(xyxy(p), xyxy(t)): inter / union, no clamp."""
    a, b = _xyxy(p), _xyxy(t)
    area_a = (a[:, 2] - a[:, 0]) * (a[:, 3] - a[:, 1])
    area_b = (b[:, 2] - b[:, 0]) * (b[:, 3] - b[:, 1])
    wh = (torch.min(a[:, 2:], b[:, 2:]) - torch.max(a[:, :2], b[:, :2])).clamp(min=0)
    inter = wh[:, 0] * wh[:, 1]
    return inter / (area_a + area_b - inter)


def _positives(wl, res, layer):
    """(batch idx, query idx, class, target box, matched pred slot) of one layer's pairs."""
    bi, qi, cls, tbox = [], [], [], []
    for b, (q, t) in enumerate(res.layer(layer)):
        bi.append(torch.full_like(q, b))
        qi.append(q)
        cls.append(wl.targets[b]["labels"].to(DEV)[t])
        tbox.append(wl.targets[b]["boxes"].to(DEV)[t])
    return torch.cat(bi), torch.cat(qi), torch.cat(cls), torch.cat(tbox)


def _torch_loss(x, boxes, wl, res, mode, alpha):
    """Sum over layers of the restated loss; x [L, B, Q, C] requires grad."""
    total = []
    for l in range(x.shape[0]):
        bi, qi, cls, tbox = _positives(wl, res, l)
        src = x[l]
        if mode == "focal":
            y = torch.zeros_like(src)
            y[bi, qi, cls] = 1.0
            prob = src.sigmoid()
            ce = F.binary_cross_entropy_with_logits(src, y, reduction="none")
            p_t = prob * y + (1 - prob) * (1 - y)
            loss = ce * ((1 - p_t) ** 2)
            loss = (alpha * y + (1 - alpha) * (1 - y)) * loss
        else:
            iou = _pair_iou(boxes[l][bi, qi].detach(), tbox)
            prob = src.sigmoid()
            pos_w = torch.zeros_like(src)
            neg_w = prob ** 2
            t = (prob[bi, qi, cls].pow(alpha) * iou.pow(1 - alpha)).clamp(min=0.01).detach()
            pos_w[bi, qi, cls] = t
            neg_w[bi, qi, cls] = 1 - t
            loss = neg_w * src - F.logsigmoid(src) * (pos_w + neg_w)
        total.append(loss.sum())
    return torch.stack(total)


def _case(name, **kw):
    wl = workloads.make(name, **kw)
    logits, boxes = wl.pred_logits.to(DEV), wl.pred_boxes.to(DEV)
    packed = matcher.PackedTargets.from_list(wl.targets_on(DEV), DEV)
    res = matcher.match_packed(logits, boxes, packed, wl.group_detr, weights=wl.weights)
    return wl, logits, boxes, packed, res


@pytest.mark.parametrize("mode", ["focal", "ia_bce"])
@pytest.mark.parametrize("name,kw", [("step", {}), ("crowd", {"images": 2}), ("ties", {})])
def test_label_loss_matches_torch_autograd(mode, name, kw):
    wl, logits, boxes, packed, res = _case(name, **kw)
    x = logits.clone().requires_grad_(True)
    loss, correct = matched_label_losses(x, boxes, packed, res, mode=mode, focal_alpha=0.25)
    gw = torch.linspace(0.5, 1.5, wl.layers, device=DEV)
    (loss * gw).sum().backward()
    xr = logits.clone().requires_grad_(True)
    ref = _torch_loss(xr, boxes, wl, res, mode, 0.25)
    (ref * gw).sum().backward()
    torch.cuda.synchronize()
    assert torch.allclose(loss.detach(), ref.detach(), rtol=1e-5, atol=0.0, equal_nan=True), (loss, ref)
    assert torch.equal(torch.isnan(x.grad), torch.isnan(xr.grad))
    finite = torch.isfinite(xr.grad)
    scale = float(xr.grad[finite].abs().max())
    assert float((x.grad[finite] - xr.grad[finite]).abs().max()) <= 1e-5 * scale
    # top-1 accuracy of the matched queries (smallest index among equal maxima)
    for l in range(wl.layers):
        bi, qi, cls, _t = _positives(wl, res, l)
        rows = logits[l][bi, qi]
        best = torch.tensor([int(np.argmax(r)) for r in rows.cpu().numpy()], device=DEV)
        assert int(correct[l]) == int((best == cls).sum())


def test_criterion_contract_and_class_error():
    wl, logits, boxes, packed, res = _case("step", layers=1)
    idx = res.layer(0)
    targets = wl.targets_on(DEV)
    out = criterion_loss_labels({"pred_logits": logits[0], "pred_boxes": boxes[0]}, targets, idx, 7.0,
                                mode="ia_bce", focal_alpha=0.25)
    xr = logits.clone().requires_grad_(True)
    ref = _torch_loss(xr, boxes, wl, res, "ia_bce", 0.25)[0] / 7.0
    assert torch.allclose(out["loss_ce"], ref.detach(), rtol=1e-5)
    bi, qi, cls, _t = _positives(wl, res, 0)
    acc = 100.0 * float((logits[0][bi, qi].argmax(-1) == cls).float().mean())
    assert abs(float(out["class_error"]) - (100.0 - acc)) < 1e-3
    # nothing matched: the loss is all negatives and class_error is 100
    empty = [(torch.zeros(0, dtype=torch.int64, device=DEV),) * 2 for _ in targets]
    out = criterion_loss_labels({"pred_logits": logits[0], "pred_boxes": boxes[0]}, targets, empty, 1.0, mode="focal")
    assert float(out["class_error"]) == 100.0 and float(out["loss_ce"]) > 0
