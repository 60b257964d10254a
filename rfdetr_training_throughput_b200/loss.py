"""Matched-box losses (L1 and GIoU over the matcher's pairs) with autograd, on the device.

The DETR-family criterion's ``loss_boxes`` gathers the matched prediction boxes
and target boxes with the matcher's index tensors (criterion.py:904/906, cited at
patches.py:339-341), then takes the L1 of their cxcywh coordinates and the
diagonal of an N x N generalized-IoU matrix, normalised by the number of boxes.
``matched_box_losses`` computes the same two sums per decoder layer straight from
a ``MatchResult`` (``rfm_box_loss_forward``), and its backward writes each matched
query's box gradient in place (``rfm_box_loss_backward``): no gathers, no index
tensors, no N x N matrix, no host synchronisation.  Normalisation (the criterion's
``num_boxes``, which rf-detr averages over ranks) is left to the caller.
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
