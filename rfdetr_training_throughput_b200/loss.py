"""The criterion's consumers of the matcher's pairs, with autograd, on the device: the matched-box
losses (L1 and GIoU) and the classification loss over every logit with the matched classes as
positives.

The DETR-family criterion's ``loss_boxes`` gathers the matched prediction boxes
and target boxes with the matcher's index tensors (criterion.py:904/906, cited at
patches.py:339-341), then takes the L1 of their cxcywh coordinates and the
diagonal of an N x N generalized-IoU matrix, normalised by the number of boxes.
``matched_box_losses`` computes the same two sums per decoder layer straight from
a ``MatchResult`` (``rfm_box_loss_forward``), and its backward writes each matched
query's box gradient in place (``rfm_box_loss_backward``): no gathers, no index
tensors, no N x N matrix, no host synchronisation.  Normalisation (the criterion's
``num_boxes``, which rf-detr averages over ranks) is left to the caller.

``matched_label_losses`` is the criterion's ``loss_labels`` (the target-class scatter at
criterion.py:562, cited at patches.py:339-341): the matched queries' target classes are the
positives of a sigmoid loss over all ``[L, B, Q, C]`` logits -- Deformable DETR's focal loss or
the IoU-aware BCE of LW-DETR / RF-DETR -- evaluated by ``rfm_label_loss_forward`` straight from
the packed pairs (no class map, no one-hot tensor), its gradient written by
``rfm_label_loss_backward``.
"""

from __future__ import annotations

import ctypes
from functools import lru_cache

import numpy as np
import torch

from . import _lib
from .matcher import MatchResult, PackedTargets


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


@lru_cache(maxsize=64)
def _offsets_cached(counts: tuple[int, ...], device: str) -> torch.Tensor:
    off = np.zeros(len(counts) + 1, dtype=np.int32)
    off[1:] = np.cumsum(counts)
    return torch.from_numpy(off).to(device)


_BY_ID: dict = {}


def _offsets_on(counts: tuple[int, ...], device: str) -> torch.Tensor:
    """Exclusive prefix sums of ``counts`` as a device int32 array, cached per counts tuple and,
    for the tuples a training loop reuses every step, by the tuple object itself."""
    key = (id(counts), device)
    hit = _BY_ID.get(key)
    if hit is not None and hit[0] is counts:
        return hit[1]
    t = _offsets_cached(counts, device)
    if len(_BY_ID) >= 64:
        _BY_ID.clear()
    _BY_ID[key] = (counts, t)
    return t


class _MatchedBoxLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred_boxes, tgt_boxes, tgt_offsets, pairs, pair_offsets, layers, images):
        queries = pred_boxes.shape[2]
        parts = torch.empty((2, layers * images), dtype=torch.float32, device=pred_boxes.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(pred_boxes.device).cuda_stream)
        _lib.check("rfm_box_loss_forward", _lib.load().rfm_box_loss_forward(
            _ptr(pred_boxes), _ptr(tgt_boxes), _ptr(tgt_offsets), _ptr(pairs[0]), _ptr(pairs[1]),
            _ptr(pair_offsets), layers, images, queries, tgt_boxes.shape[0], _ptr(parts[0]), _ptr(parts[1]),
            stream))
        ctx.save_for_backward(pred_boxes, tgt_boxes, tgt_offsets, pairs, pair_offsets)
        ctx.layers, ctx.images = layers, images
        sums = parts.view(2, layers, images).sum(dim=2)
        return sums[0], sums[1]

    @staticmethod
    def backward(ctx, grad_l1, grad_giou):
        pred_boxes, tgt_boxes, tgt_offsets, pairs, pair_offsets = ctx.saved_tensors
        grad = torch.zeros_like(pred_boxes)
        g1 = (torch.zeros(ctx.layers, device=pred_boxes.device) if grad_l1 is None else grad_l1).float().contiguous()
        g2 = (torch.zeros(ctx.layers, device=pred_boxes.device) if grad_giou is None else grad_giou).float().contiguous()
        stream = ctypes.c_void_p(torch.cuda.current_stream(pred_boxes.device).cuda_stream)
        _lib.check("rfm_box_loss_backward", _lib.load().rfm_box_loss_backward(
            _ptr(pred_boxes), _ptr(tgt_boxes), _ptr(tgt_offsets), _ptr(pairs[0]), _ptr(pairs[1]),
            _ptr(pair_offsets), ctx.layers, ctx.images, pred_boxes.shape[2], tgt_boxes.shape[0], _ptr(g1),
            _ptr(g2), _ptr(grad), stream))
        return grad, None, None, None, None, None, None


def box_losses(pred_boxes: torch.Tensor, tgt_boxes: torch.Tensor, sizes: tuple[int, ...], pairs: torch.Tensor,
               per_image: tuple[int, ...]) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-layer ``(sum of L1, sum of 1 - GIoU)`` over index pairs, differentiable in ``pred_boxes``.

    ``pred_boxes`` ``[L, B, Q, 4]`` cxcywh; ``tgt_boxes`` ``[S, 4]`` packed, image ``b`` owning
    ``sizes[b]`` rows; ``pairs`` int64 ``[2, N]`` (query index, target index within its image) in
    ``L * B`` consecutive chunks of ``per_image`` pairs (layer-major).  Pairs holding -1 are skipped.
    """
    if not pred_boxes.is_cuda:
        raise ValueError("pred_boxes must be a CUDA tensor (this loss has no CPU path)")
    if pred_boxes.dim() != 4 or pred_boxes.shape[-1] != 4:
        raise ValueError("expected pred_boxes [L, B, Q, 4]")
    layers, images = pred_boxes.shape[0], pred_boxes.shape[1]
    if len(sizes) != images or len(per_image) != layers * images:
        raise ValueError("sizes / per_image do not match pred_boxes' layers and images")
    if pairs.dtype != torch.int64 or pairs.dim() != 2 or pairs.shape[0] != 2 or pairs.stride(1) != 1:
        raise ValueError("pairs must be int64 [2, N] with contiguous rows")
    pred = pred_boxes if pred_boxes.dtype == torch.float32 else pred_boxes.float()
    pred = pred.contiguous()
    if pred.data_ptr() % 16:
        pred = pred.clone()
    tgt = tgt_boxes.float().contiguous()
    if tgt.data_ptr() % 16:
        tgt = tgt.clone()
    device = str(pred.device)
    return _MatchedBoxLoss.apply(pred, tgt, _offsets_on(sizes, device), pairs, _offsets_on(per_image, device),
                                 layers, images)


def matched_box_losses(pred_boxes: torch.Tensor, targets: PackedTargets,
                       match: MatchResult) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-layer ``(sum of L1, sum of 1 - GIoU)`` over a ``MatchResult``'s pairs, differentiable in
    ``pred_boxes`` ``[L, B, Q, 4]`` (cxcywh float32, the boxes the pairs were matched on)."""
    if (match.layers, match.images) != tuple(pred_boxes.shape[:2]) or len(targets.sizes) != pred_boxes.shape[1]:
        raise ValueError("match, targets and pred_boxes disagree on layers or images")
    tg = targets.checked()
    return box_losses(pred_boxes, tg.boxes, tg.sizes, match.pairs, match.per_image_key)


def criterion_loss_boxes(outputs: dict, targets, indices, num_boxes) -> dict:
    """DETR's ``SetCriterion.loss_boxes(outputs, targets, indices, num_boxes)`` contract on one
    layer: ``{"loss_bbox": sum L1 / num_boxes, "loss_giou": sum (1 - GIoU) / num_boxes}`` over
    ``indices`` (one ``(query_idx, target_idx)`` pair of int64 tensors per image)."""
    pred = outputs["pred_boxes"]
    if len(indices) != pred.shape[0] or len(targets) != pred.shape[0]:
        raise ValueError("one (query_idx, target_idx) pair and one target dict per image expected")
    counts = tuple(int(q.shape[0]) for q, _t in indices)  # host-known shapes: no synchronisation
    device = pred.device
    if sum(counts):
        pairs = torch.stack([torch.cat([q.to(device, torch.int64) for q, _t in indices]),
                             torch.cat([t.to(device, torch.int64) for _q, t in indices])])
    else:
        pairs = torch.zeros((2, 0), dtype=torch.int64, device=device)
    sizes = tuple(int(t["boxes"].shape[0]) for t in targets)
    tgt = torch.cat([t["boxes"].reshape(-1, 4) for t in targets]).to(device) if targets else \
        torch.zeros((0, 4), device=device)
    l1, giou = box_losses(pred.unsqueeze(0), tgt, sizes, pairs, counts)
    return {"loss_bbox": l1[0] / num_boxes, "loss_giou": giou[0] / num_boxes}


# --------------------------------------------------------------------------- classification loss

#: ``mode`` values of the classification loss (RFM_LABEL_LOSS_* in include/rfm.h).
LABEL_LOSS_MODES = {"focal": 0, "ia_bce": 1}


class _MatchedLabelLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, pred_boxes, labels, tgt_boxes, tgt_offsets, pairs, pair_offsets, mode, alpha):
        layers, images, queries, classes = logits.shape
        lib = _lib.load()
        nparts = int(lib.rfm_label_loss_parts(layers, images, queries, classes))
        if nparts < 0:
            raise _lib.RfmError("rfm_label_loss_parts", -nparts)
        loss_part = torch.empty(nparts, dtype=torch.float32, device=logits.device)
        correct_part = torch.empty(nparts, dtype=torch.int32, device=logits.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(logits.device).cuda_stream)
        _lib.check("rfm_label_loss_forward", lib.rfm_label_loss_forward(
            _ptr(logits), _ptr(pred_boxes), _ptr(labels), _ptr(tgt_boxes), _ptr(tgt_offsets), _ptr(pairs[0]),
            _ptr(pairs[1]), _ptr(pair_offsets), layers, images, queries, classes, labels.shape[0], mode, alpha,
            _ptr(loss_part), _ptr(correct_part), stream))
        ctx.save_for_backward(logits, pred_boxes, labels, tgt_boxes, tgt_offsets, pairs, pair_offsets)
        ctx.mode, ctx.alpha = mode, alpha
        correct = correct_part.view(layers, -1).sum(dim=1)
        ctx.mark_non_differentiable(correct)
        return loss_part.view(layers, -1).sum(dim=1), correct

    @staticmethod
    def backward(ctx, grad_loss, _grad_correct):
        logits, pred_boxes, labels, tgt_boxes, tgt_offsets, pairs, pair_offsets = ctx.saved_tensors
        layers, images, queries, classes = logits.shape
        g = (torch.zeros(layers, device=logits.device) if grad_loss is None else grad_loss).float().contiguous()
        grad = torch.empty_like(logits)
        stream = ctypes.c_void_p(torch.cuda.current_stream(logits.device).cuda_stream)
        _lib.check("rfm_label_loss_backward", _lib.load().rfm_label_loss_backward(
            _ptr(logits), _ptr(pred_boxes), _ptr(labels), _ptr(tgt_boxes), _ptr(tgt_offsets), _ptr(pairs[0]),
            _ptr(pairs[1]), _ptr(pair_offsets), layers, images, queries, classes, labels.shape[0], ctx.mode,
            ctx.alpha, _ptr(g), _ptr(grad), stream))
        return grad, None, None, None, None, None, None, None, None


def label_losses(pred_logits: torch.Tensor, pred_boxes: torch.Tensor, labels: torch.Tensor, tgt_boxes: torch.Tensor,
                 sizes: tuple[int, ...], pairs: torch.Tensor, per_image: tuple[int, ...], *, mode: str = "ia_bce",
                 focal_alpha: float = 0.25) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-layer ``(sum of the classification loss, matched queries whose top logit is their class)``
    over index pairs, differentiable in ``pred_logits``.

    ``pred_logits`` ``[L, B, Q, C]`` and ``pred_boxes`` ``[L, B, Q, 4]`` (cxcywh, read by the IoU-aware
    loss only, no gradient); ``labels`` ``[S]`` and ``tgt_boxes`` ``[S, 4]`` packed, image ``b`` owning
    ``sizes[b]`` rows; ``pairs`` int64 ``[2, N]`` (query index, target index within its image) in
    ``L * B`` consecutive chunks of ``per_image`` pairs (layer-major).  ``mode`` is ``"focal"``
    (Deformable DETR's sigmoid focal loss) or ``"ia_bce"`` (the IoU-aware BCE of LW-DETR / RF-DETR).
    """
    if mode not in LABEL_LOSS_MODES:
        raise ValueError(f"mode must be one of {sorted(LABEL_LOSS_MODES)}")
    if not pred_logits.is_cuda:
        raise ValueError("pred_logits must be a CUDA tensor (this loss has no CPU path)")
    if pred_logits.dim() != 4 or pred_boxes.dim() != 4 or pred_boxes.shape[:3] != pred_logits.shape[:3]:
        raise ValueError("expected pred_logits [L, B, Q, C] and pred_boxes [L, B, Q, 4]")
    layers, images = pred_logits.shape[0], pred_logits.shape[1]
    if len(sizes) != images or len(per_image) != layers * images:
        raise ValueError("sizes / per_image do not match pred_logits' layers and images")
    if pairs.dtype != torch.int64 or pairs.dim() != 2 or pairs.shape[0] != 2 or pairs.stride(1) != 1:
        raise ValueError("pairs must be int64 [2, N] with contiguous rows")
    logits = pred_logits if pred_logits.dtype == torch.float32 else pred_logits.float()
    logits = logits.contiguous()
    boxes = pred_boxes.detach().float().contiguous()
    if boxes.data_ptr() % 16:
        boxes = boxes.clone()
    tgt = tgt_boxes.float().contiguous()
    if tgt.data_ptr() % 16:
        tgt = tgt.clone()
    lab = labels.to(torch.int64).contiguous()
    device = str(logits.device)
    return _MatchedLabelLoss.apply(logits, boxes, lab, tgt, _offsets_on(sizes, device), pairs,
                                   _offsets_on(per_image, device), LABEL_LOSS_MODES[mode], float(focal_alpha))


def matched_label_losses(pred_logits: torch.Tensor, pred_boxes: torch.Tensor, targets: PackedTargets,
                         match: MatchResult, *, mode: str = "ia_bce",
                         focal_alpha: float = 0.25) -> tuple[torch.Tensor, torch.Tensor]:
    """``label_losses`` over a ``MatchResult``'s pairs (the predictions it was matched on)."""
    if (match.layers, match.images) != tuple(pred_logits.shape[:2]) or len(targets.sizes) != pred_logits.shape[1]:
        raise ValueError("match, targets and pred_logits disagree on layers or images")
    tg = targets.checked()
    return label_losses(pred_logits, pred_boxes, tg.labels, tg.boxes, tg.sizes, match.pairs, match.per_image_key,
                        mode=mode, focal_alpha=focal_alpha)


def criterion_loss_labels(outputs: dict, targets, indices, num_boxes, log: bool = True, *, mode: str = "ia_bce",
                          focal_alpha: float = 0.25) -> dict:
    """DETR's ``SetCriterion.loss_labels(outputs, targets, indices, num_boxes, log)`` contract on one
    layer: ``{"loss_ce": sum / num_boxes}`` plus, with ``log``, ``"class_error"`` (100 minus the top-1
    accuracy in percent of the matched queries, 100 when nothing is matched)."""
    logits = outputs["pred_logits"]
    boxes = outputs["pred_boxes"]
    if len(indices) != logits.shape[0] or len(targets) != logits.shape[0]:
        raise ValueError("one (query_idx, target_idx) pair and one target dict per image expected")
    counts = tuple(int(q.shape[0]) for q, _t in indices)  # host-known shapes: no synchronisation
    device = logits.device
    if sum(counts):
        pairs = torch.stack([torch.cat([q.to(device, torch.int64) for q, _t in indices]),
                             torch.cat([t.to(device, torch.int64) for _q, t in indices])])
    else:
        pairs = torch.zeros((2, 0), dtype=torch.int64, device=device)
    sizes = tuple(int(t["labels"].shape[0]) for t in targets)
    if targets:
        labels = torch.cat([t["labels"].reshape(-1) for t in targets]).to(device)
        tgt = torch.cat([t["boxes"].reshape(-1, 4) for t in targets]).to(device)
    else:
        labels = torch.zeros(0, dtype=torch.int64, device=device)
        tgt = torch.zeros((0, 4), device=device)
    loss, correct = label_losses(logits.unsqueeze(0), boxes.unsqueeze(0), labels, tgt, sizes, pairs, counts,
                                 mode=mode, focal_alpha=focal_alpha)
    out = {"loss_ce": loss[0] / num_boxes}
    if log:
        matched = sum(counts)
        out["class_error"] = (100.0 - 100.0 * correct[0].float() / matched) if matched else \
            torch.full((), 100.0, device=device)
    return out
