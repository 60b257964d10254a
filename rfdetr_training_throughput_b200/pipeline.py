"""Matching batches that arrive in host memory, with the upload of the next batch overlapping the
matching of the current one.

A training step's predictions are on the device already; a consumer that feeds the matcher from
the host (an evaluation or labelling pipeline, a process that receives detections over the network)
pays one host-to-device copy per batch, which over PCIe takes far longer than the match itself.
``PrefetchingMatcher`` issues each batch's copy on its own stream into freshly allocated device
buffers (``prefetch``) and lets ``match`` wait for exactly that copy before launching the two
matcher kernels on the caller's stream, so copy k+1 runs while batch k is matched and its pairs are
read back.  Buffers are handed to the caching allocator with ``record_stream`` so they are not
reused before the match that reads them has run.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

from .matcher import DEFAULT_WEIGHTS, MatchResult, PackedTargets, match_packed


@dataclass
class PrefetchedBatch:
    """One batch's device copies and the event that marks them complete."""

    logits: torch.Tensor
    boxes: torch.Tensor
    targets: PackedTargets
    ready: torch.cuda.Event


class PrefetchingMatcher:
    """``match_packed`` over host batches with the next batch's upload in flight."""

    def __init__(self, group_detr: int, *, weights: dict | None = None, device: torch.device | None = None):
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.group_detr = group_detr
        self.weights = dict(DEFAULT_WEIGHTS if weights is None else weights)
        self.copy_stream = torch.cuda.Stream(self.device)

    def prefetch(self, pred_logits: torch.Tensor, pred_boxes: torch.Tensor, labels: torch.Tensor,
                 tgt_boxes: torch.Tensor, sizes: Sequence[int]) -> PrefetchedBatch:
        """Start copying one host batch (pinned memory for a true asynchronous copy): logits
        ``[L, B, Q, C]``, boxes ``[L, B, Q, 4]``, packed labels ``[S]`` and boxes ``[S, 4]``."""
        # The destinations are fresh allocations (record_stream in match() keeps them alive until
        # the match that reads them has run), so the copy waits for nothing on the caller's stream.
        # The caller keeps the host tensors unchanged until the copy has completed.
        with torch.cuda.stream(self.copy_stream):
            d = [t.to(self.device, non_blocking=True) for t in (pred_logits, pred_boxes, labels, tgt_boxes)]
            ready = torch.cuda.Event()
            ready.record(self.copy_stream)
        targets = PackedTargets(d[2], d[3], tuple(sizes))
        return PrefetchedBatch(d[0], d[1], targets, ready)

    def match(self, batch: PrefetchedBatch) -> MatchResult:
        """Match a prefetched batch on the current stream once its copy has landed."""
        stream = torch.cuda.current_stream(self.device)
        stream.wait_event(batch.ready)
        for t in (batch.logits, batch.boxes, batch.targets.labels, batch.targets.boxes):
            t.record_stream(stream)
        return match_packed(batch.logits, batch.boxes, batch.targets, self.group_detr, weights=self.weights)
