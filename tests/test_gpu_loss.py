"""matched_box_losses (rfm_box_loss_forward / _backward) against a plain torch fp32 reference of
the DETR-family loss_boxes on the same matched pairs: gather the matched boxes, L1 of the cxcywh
coordinates, 1 - diag(generalized_box_iou) of the xyxy boxes, torch autograd for the gradient.

Tolerances: per-layer sums within 1e-5 relative (fp32 sums of the same terms in a different
order); gradients within 1e-4 relative + 1e-5 absolute of torch's (the GIoU gradient is a
different but equivalent expression of the same derivative)."""

import numpy as np
import pytest
import torch

from rfdetr_training_throughput_b200 import matcher, workloads
from rfdetr_training_throughput_b200.loss import matched_box_losses

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _xyxy(b):
    cx, cy, w, h = b.unbind(-1)
    return torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], dim=-1)


def _area(b):
    return (b[:, 2] - b[:, 0]) * (b[:, 3] - b[:, 1])


def _generalized_box_iou(b1, b2):
    """The pairwise GIoU matrix of the DETR box ops (no clamps besides wh >= 0)."""
    a1, a2 = _area(b1), _area(b2)
    lt = torch.max(b1[:, None, :2], b2[:, :2])
    rb = torch.min(b1[:, None, 2:], b2[:, 2:])
    wh = (rb - lt).clamp(min=0)
    inter = wh[:, :, 0] * wh[:, :, 1]
    union = a1[:, None] + a2 - inter
    iou = inter / union
    lt = torch.min(b1[:, None, :2], b2[:, :2])
    rb = torch.max(b1[:, None, 2:], b2[:, 2:])
    wh = (rb - lt).clamp(min=0)
    area = wh[:, :, 0] * wh[:, :, 1]
    return iou - (area - union) / area


def _reference(pred, tgt_list, res):
    """Per-layer (sum L1, sum 1 - GIoU) and d(sum of both)/d pred, torch fp32 on the CPU."""
    pred = pred.detach().cpu().requires_grad_(True)
    l1s, gious = [], []
    for l in range(res.layers):
        pairs = res.layer(l)
        src = torch.cat([pred[l, b, q.cpu()] for b, (q, _t) in enumerate(pairs)])
        tgt = torch.cat([tgt_list[b][t.cpu()] for b, (_q, t) in enumerate(pairs)])
        l1s.append(torch.nn.functional.l1_loss(src, tgt, reduction="none").sum())
        gious.append((1 - torch.diag(_generalized_box_iou(_xyxy(src), _xyxy(tgt)))).sum())
    l1, giou = torch.stack(l1s), torch.stack(gious)
    w = torch.arange(1, res.layers + 1, dtype=torch.float32)  # distinct upstream weights per layer
    ((w * l1).sum() + (0.5 * w * giou).sum()).backward()
    return l1.detach(), giou.detach(), pred.grad


@pytest.mark.parametrize("name,kw", [("step", {}), ("sweep", {"images": 64}), ("crowd", {"images": 2})])
def test_box_losses_and_gradients_match_torch(name, kw):
    wl = workloads.make(name, **kw)
    packed = matcher.PackedTargets.from_list(wl.targets_on(DEV), DEV)
    pred = wl.pred_boxes.to(DEV)
    res = matcher.match_packed(wl.pred_logits.to(DEV), pred, packed, wl.group_detr, weights=wl.weights)
    x = pred.clone().requires_grad_(True)
    l1, giou = matched_box_losses(x, packed, res)
    w = torch.arange(1, wl.layers + 1, dtype=torch.float32, device=DEV)
    ((w * l1).sum() + (0.5 * w * giou).sum()).backward()
    torch.cuda.synchronize()
    r_l1, r_giou, r_grad = _reference(pred, [t["boxes"] for t in wl.targets], res)
    np.testing.assert_allclose(l1.detach().cpu().numpy(), r_l1.numpy(), rtol=1e-5)
    np.testing.assert_allclose(giou.detach().cpu().numpy(), r_giou.numpy(), rtol=1e-5)
    np.testing.assert_allclose(x.grad.cpu().numpy(), r_grad.numpy(), rtol=1e-4, atol=1e-5)
    # unmatched queries get no gradient
    matched = torch.zeros(pred.shape[:3], dtype=torch.bool)
    for l in range(wl.layers):
        for b, (q, _t) in enumerate(res.layer(l)):
            matched[l, b, q.cpu()] = True
    assert bool((x.grad.cpu()[~matched] == 0).all())


def test_box_losses_are_deterministic_and_sync_free():
    wl = workloads.make("sweep", images=128)
    packed = matcher.PackedTargets.from_list(wl.targets_on(DEV), DEV)
    pred = wl.pred_boxes.to(DEV)
    res = matcher.match_packed(wl.pred_logits.to(DEV), pred, packed, wl.group_detr, weights=wl.weights)
    torch.cuda.synchronize()
    first = matched_box_losses(pred, packed, res)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        again = [matched_box_losses(pred, packed, res) for _ in range(3)]
    finally:
        torch.cuda.set_sync_debug_mode(0)
    torch.cuda.synchronize()
    for l1, giou in again:
        assert torch.equal(l1, first[0]) and torch.equal(giou, first[1])


def test_criterion_contract_on_index_lists():
    """criterion_loss_boxes (the box_loss patch): DETR's loss_boxes(outputs, targets, indices,
    num_boxes) on one layer's per-image index tuples, against the torch reference."""
    from rfdetr_training_throughput_b200.loss import criterion_loss_boxes

    wl = workloads.make("step", layers=1)
    targets = wl.targets_on(DEV)
    outputs = wl.outputs_list(DEV)[0]
    indices = matcher.match_layers([outputs], targets, wl.group_detr, weights=wl.weights)[0]
    x = outputs["pred_boxes"].clone().requires_grad_(True)
    num_boxes = 17.0
    losses = criterion_loss_boxes({"pred_boxes": x}, targets, indices, num_boxes)
    (losses["loss_bbox"] + 2.0 * losses["loss_giou"]).backward()
    torch.cuda.synchronize()
    ref = x.detach().cpu().requires_grad_(True)
    src = torch.cat([ref[b, q.cpu()] for b, (q, _t) in enumerate(indices)])
    tgt = torch.cat([targets[b]["boxes"].cpu()[t.cpu()] for b, (_q, t) in enumerate(indices)])
    r_bbox = torch.nn.functional.l1_loss(src, tgt, reduction="none").sum() / num_boxes
    r_giou = (1 - torch.diag(_generalized_box_iou(_xyxy(src), _xyxy(tgt)))).sum() / num_boxes
    (r_bbox + 2.0 * r_giou).backward()
    np.testing.assert_allclose(losses["loss_bbox"].item(), r_bbox.item(), rtol=1e-5)
    np.testing.assert_allclose(losses["loss_giou"].item(), r_giou.item(), rtol=1e-5)
    np.testing.assert_allclose(x.grad.cpu().numpy(), ref.grad.numpy(), rtol=1e-4, atol=1e-6)
