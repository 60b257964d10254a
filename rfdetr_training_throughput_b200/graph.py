"""The matcher step captured as a CUDA graph, for batches whose shape repeats.

``match_packed`` already runs on the device without a host synchronisation, but
every call still pays its host cost (plan lookup, three allocations, the FFI
call and its two kernel launches, ~30-50 us of Python and driver work).  On the production
step (5 layers x 8 images x 13 groups) that is as long as the GPU work itself.
``MatchGraph`` records the step once for a fixed shape (targets per image,
layers, queries, classes, group split, weights) and replays it with a single
host call.  Training loops whose per-image target counts repeat (fixed-size
crops, padded batches, a validation set) reuse one graph per distinct shape;
``MatchGraphCache`` keeps them.

The graph reads its inputs from its own device buffers (``logits``, ``boxes``,
``labels``, ``tgt_boxes``) and writes the pairs of every replay to the same
``pairs`` buffer (its own, or the ``out`` tensor given at construction): copy
new inputs in (``__call__`` does) and read or copy the result before the next
replay.  Stream capture covers the cost kernel (which also resets the
solver's counter) and the solver kernel, plus whatever the optional ``post``
hook enqueues after them (the pushed exchange's barrier kernel in
``sharded.ShardedMatcher``); plans and launch parameters are host-side values
fixed at capture time, which is exactly what a fixed shape pins.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Sequence

import torch

from .matcher import DEFAULT_WEIGHTS, MatchResult, PackedTargets, match_packed


class MatchGraph:
    """One matcher step of a fixed shape, captured as a CUDA graph on ``device``."""

    def __init__(self, sizes: Sequence[int], layers: int, queries: int, num_classes: int, group_detr: int, *,
                 weights: dict | None = None, device: torch.device | None = None, warmup: int = 2,
                 out: torch.Tensor | None = None, push=None, post=None):
        if not torch.cuda.is_available():
            raise RuntimeError("MatchGraph needs a CUDA device (there is no CPU path)")
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.sizes = tuple(int(s) for s in sizes)
        self.layers, self.queries, self.num_classes, self.group_detr = layers, queries, num_classes, group_detr
        self.weights = dict(DEFAULT_WEIGHTS if weights is None else weights)
        self.device = device
        images, total = len(self.sizes), sum(self.sizes)
        # static inputs, filled with valid values so the warm-up and capture runs are well defined
        self.logits = torch.zeros((layers, images, queries, num_classes), dtype=torch.float32, device=device)
        self.boxes = torch.full((layers, images, queries, 4), 0.5, dtype=torch.float32, device=device)
        self.labels = torch.zeros(total, dtype=torch.int64, device=device)
        self.tgt_boxes = torch.full((total, 4), 0.25, dtype=torch.float32, device=device)
        self._targets = PackedTargets.from_checked_sizes(self.labels, self.tgt_boxes, self.sizes, total)
        self._out = out  # optional caller buffer the pairs are written into (e.g. a collective's send buffer)
        self._push = push  # optional rfm_pair_push list the solver also writes every pair to
        self._post = post  # optional callable enqueued after the step (captured with it)

        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.device(device), torch.cuda.stream(side):
            for _ in range(max(1, warmup)):  # builds the plan and the launch caches outside the capture
                self._step()
        torch.cuda.current_stream(device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.device(device), torch.cuda.graph(self.graph):
            self.result = self._step()
        self.pairs = self.result.pairs

    def _step(self) -> MatchResult:
        res = match_packed(self.logits, self.boxes, self._targets, self.group_detr, weights=self.weights,
                           out=self._out, push=self._push)
        if self._post is not None:
            self._post()
        return res

    def replay(self) -> MatchResult:
        """Re-run the captured step on the current contents of the input buffers."""
        self.graph.replay()
        return self.result

    def __call__(self, pred_logits: torch.Tensor, pred_boxes: torch.Tensor, labels: torch.Tensor,
                 tgt_boxes: torch.Tensor) -> MatchResult:
        """Copy one batch (logits ``[L, B, Q, C]``, boxes ``[L, B, Q, 4]``, packed labels ``[S]`` and
        boxes ``[S, 4]``) into the graph's buffers and replay it."""
        for dst, src, name in ((self.logits, pred_logits, "pred_logits"), (self.boxes, pred_boxes, "pred_boxes"),
                               (self.labels, labels, "labels"), (self.tgt_boxes, tgt_boxes, "tgt_boxes")):
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError(f"{name} has shape {tuple(src.shape)}, the graph was captured for {tuple(dst.shape)}")
            dst.copy_(src, non_blocking=True)
        return self.replay()


class MatchGraphCache:
    """Graphs keyed by batch shape, least recently used dropped beyond ``capacity``."""

    def __init__(self, capacity: int = 8, weights: dict | None = None):
        self.capacity = capacity
        self.weights = dict(DEFAULT_WEIGHTS if weights is None else weights)
        self._graphs: OrderedDict[tuple, MatchGraph] = OrderedDict()

    def get(self, sizes: Sequence[int], layers: int, queries: int, num_classes: int, group_detr: int,
            device: torch.device) -> MatchGraph:
        key = (tuple(int(s) for s in sizes), layers, queries, num_classes, group_detr, str(device))
        g = self._graphs.get(key)
        if g is None:
            g = MatchGraph(key[0], layers, queries, num_classes, group_detr, weights=self.weights, device=device)
            self._graphs[key] = g
            if len(self._graphs) > self.capacity:
                self._graphs.popitem(last=False)
        else:
            self._graphs.move_to_end(key)
        return g

    def __call__(self, pred_logits: torch.Tensor, pred_boxes: torch.Tensor, targets: PackedTargets,
                 group_detr: int) -> MatchResult:
        layers, _, queries, num_classes = pred_logits.shape
        g = self.get(targets.sizes, layers, queries, num_classes, group_detr, pred_logits.device)
        return g(pred_logits, pred_boxes, targets.labels, targets.boxes)
