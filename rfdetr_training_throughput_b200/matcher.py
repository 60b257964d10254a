"""B200 drop-in for RF-DETR's Hungarian matching step.

``HungarianMatcher.forward(outputs, targets, group_detr)`` keeps rf-detr 1.10.1's
contract (its call sites are the patched methods at patches.py:123-149 and
patches.py:379-418): ``outputs["pred_logits"]`` ``[B, Q, C]`` and
``outputs["pred_boxes"]`` ``[B, Q, 4]`` (cxcywh), ``targets[b]["labels"]`` ``[T_b]``
and ``targets[b]["boxes"]`` ``[T_b, 4]``, ``group_detr`` query groups of
``Q // group_detr`` queries each.  It returns one ``(query_idx, target_idx)`` pair
of int64 device tensors per image, ``group_detr * min(Q // group_detr, T_b)``
pairs long: groups in order, and within a group the pairs SciPy's
``linear_sum_assignment`` returns for that group's ``[Q/G, T_b]`` block (ascending
query index), with the group offset ``g * Q/G`` added to the query index
(patches.py:398).

Two launches do the whole step on the device, with no host synchronisation:
``rfm_cost`` writes every layer's cost matrix (target-major: the transpose of the
compact ``[Q, sum T]`` matrix, so that both kernels move whole coalesced rows)
and ``rfm_lsap`` solves all ``layers x images x groups`` problems in place and
writes the index pairs at their final position.  ``match_packed`` is the
allocation-light core (packed targets in, one packed pair buffer out);
``match_layers`` and ``HungarianMatcher`` wrap it in rf-detr's list interface.

The sub-steps are exposed under the names of the functions the reference
patches: ``compute_compact_detection_cost_matrix`` (patches.py:123-149),
``assign_padded`` (patches.py:379-418) and ``batch_linear_assignment``
(kernels_lap.py:332-355 behind patches.py:314-317).

There is no CPU or Triton fallback: CPU tensors, segmentation outputs and
problems wider than ``MAX_COLS`` raise.
"""

from __future__ import annotations

import ctypes
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Sequence

import numpy as np
import torch

from . import _lib

DEFAULT_WEIGHTS = {"cost_class": 2.0, "cost_bbox": 5.0, "cost_giou": 2.0, "focal_alpha": 0.25}


def _stream_handle(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this matcher has no CPU path)")


def _aligned16(t: torch.Tensor) -> torch.Tensor:
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _round4(x: int) -> int:
    return (x + 3) // 4 * 4


# --------------------------------------------------------------------------- inputs / outputs


@dataclass
class PackedTargets:
    """All images' targets of a batch in two device tensors plus host-known sizes.

    ``labels`` ``[S]`` int64 and ``boxes`` ``[S, 4]`` float32 cxcywh hold image
    ``b``'s targets at rows ``offsets[b]:offsets[b+1]`` (``sizes`` is known on the
    host, as ``len(target["boxes"])`` is in rf-detr).
    """

    labels: torch.Tensor
    boxes: torch.Tensor
    sizes: tuple[int, ...]
    total: int = field(init=False, repr=False)

    def __post_init__(self) -> None:
        if type(self.sizes) is not tuple or not all(type(s) is int for s in self.sizes):
            self.sizes = tuple(int(s) for s in self.sizes)
        self.total = sum(self.sizes)

    @classmethod
    def from_checked_sizes(cls, labels: torch.Tensor, boxes: torch.Tensor, sizes: tuple[int, ...],
                           total: int) -> "PackedTargets":
        """Construct without re-validating ``sizes`` (a tuple of ints summing to ``total``), for
        callers that build the same split every step."""
        obj = cls.__new__(cls)
        obj.labels, obj.boxes, obj.sizes, obj.total = labels, boxes, sizes, total
        return obj

    @staticmethod
    def from_list(targets: Sequence[dict], device: torch.device | None = None) -> "PackedTargets":
        sizes = tuple(int(t["labels"].shape[0]) for t in targets)
        if any(int(t["boxes"].shape[0]) != s for t, s in zip(targets, sizes)):
            raise ValueError("targets[i]['labels'] and ['boxes'] disagree in length")
        if device is None:
            device = targets[0]["labels"].device if targets else torch.device("cuda")
        if not targets:
            return PackedTargets(torch.zeros(0, dtype=torch.int64, device=device),
                                 torch.zeros((0, 4), dtype=torch.float32, device=device), sizes)
        labels = torch.cat([t["labels"].reshape(-1) for t in targets]).to(device=device, dtype=torch.int64)
        boxes = torch.cat([t["boxes"].reshape(-1, 4) for t in targets]).to(device=device, dtype=torch.float32)
        return PackedTargets(labels.contiguous(), _aligned16(boxes.contiguous()), sizes)

    def checked(self) -> "PackedTargets":
        _require_cuda(self.labels, "labels")
        _require_cuda(self.boxes, "boxes")
        total = self.total
        if self.labels.shape != (total,) or self.boxes.shape != (total, 4):
            raise ValueError("packed targets do not match their sizes")
        labels = self.labels if self.labels.dtype == torch.int64 else self.labels.long()
        boxes = self.boxes if self.boxes.dtype == torch.float32 else self.boxes.float()
        labels = labels.contiguous()
        boxes = _aligned16(boxes.contiguous())
        if labels is self.labels and boxes is self.boxes:
            return self
        return PackedTargets(labels, boxes, self.sizes)


class MatchResult:
    """Packed result of one matcher step: ``pairs`` ``[2, total]`` int64 on the device.

    Layer ``l``, image ``b`` owns ``pairs[:, start:start+count]`` with the host-known
    ``count = group_detr * min(Q/G, T_b)``; ``layer(l)`` builds rf-detr's list of
    per-image ``(query_idx, target_idx)`` views (no copy).
    """

    def __init__(self, pairs: torch.Tensor, per_image: list[int], layers: int, images: int,
                 per_image_key: tuple[int, ...] | None = None):
        self.pairs = pairs
        self.per_image = per_image
        self.layers = layers
        self.images = images
        self._views = None
        self._key = per_image_key

    @property
    def per_image_key(self) -> tuple[int, ...]:
        """``per_image`` as a tuple (hashable; shared by every result of one step plan)."""
        if self._key is None:
            self._key = tuple(self.per_image)
        return self._key

    def _split(self):
        if self._views is None:
            self._views = (torch.split(self.pairs[0], self.per_image), torch.split(self.pairs[1], self.per_image))
        return self._views

    def layer(self, l: int) -> list[tuple[torch.Tensor, torch.Tensor]]:
        q, t = self._split()
        base = l * self.images
        return [(q[base + b], t[base + b]) for b in range(self.images)]

    def as_lists(self) -> list[list[tuple[torch.Tensor, torch.Tensor]]]:
        return [self.layer(l) for l in range(self.layers)]


# --------------------------------------------------------------------------- plans


@dataclass
class StepPlan:
    """Everything about one matcher step that depends only on host-known sizes."""

    sizes: tuple[int, ...]
    layers: int
    queries: int
    group_detr: int
    layout: int
    ld: int
    problems: np.ndarray  # PROBLEM_DTYPE, in launch order (largest tile first)
    order: np.ndarray  # launch index -> (layer, image, group) problem index
    plan: _lib.LsapPlan
    total_pairs: int
    per_image: list[int]  # pairs per (layer, image), layer-major
    device_blob: torch.Tensor  # problems, then the int32 CTA table, then int32 offsets [B+1]
    ctas_byte: int
    offsets_byte: int
    per_image_key: tuple = ()  # per_image as one shared tuple (a hashable cache key)

    @property
    def problems_ptr(self) -> int:
        return self.device_blob.data_ptr()

    @property
    def ctas_ptr(self) -> int:
        return self.device_blob.data_ptr() + self.ctas_byte

    @property
    def offsets_ptr(self) -> int:
        return self.device_blob.data_ptr() + self.offsets_byte


def strides(layout: int, ld: int) -> tuple[int, int]:
    """(stride_q, stride_t) of a cost layout with row stride ``ld``."""
    return (ld, 1) if layout == _lib.LAYOUT_QUERY_MAJOR else (1, ld)


def build_problems(sizes: Sequence[int], layers: int, queries: int, group_detr: int, ld: int,
                   layout: int = _lib.LAYOUT_QUERY_MAJOR):
    """Problem descriptors of a step, in (layer, image, group) order.

    Problem ``(l, b, g)`` is the ``[Q/G, T_b]`` block of layer ``l``'s compact
    matrix at rows ``g*Q/G ...`` and columns ``off[b] ...`` (or the same block of
    its target-major transpose); its pairs go to the ``(l, b)`` image chunk at
    ``g * min(Q/G, T_b)``.  The layer-image-group order and the group offset follow
    ``_stack_padded`` as patches.py:371,398 reads it.  Returns
    ``(problems, per_image_pairs, total_pairs, offsets)``; problems whose image has
    no target are dropped.
    """
    if group_detr < 1 or queries % group_detr:
        raise ValueError(f"num_queries {queries} is not a multiple of group_detr {group_detr}")
    sz = np.asarray(sizes, dtype=np.int64).reshape(-1)
    if (sz < 0).any():
        raise ValueError("negative target count")
    nimg = sz.shape[0]
    total_t = int(sz.sum())
    qg = queries // group_detr
    offsets = np.zeros(nimg + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(sz)
    pairs = np.minimum(sz, qg)
    per_image = np.tile(group_detr * pairs, layers)
    image_base = np.zeros(layers * nimg + 1, dtype=np.int64)
    image_base[1:] = np.cumsum(per_image)
    lay = np.repeat(np.arange(layers, dtype=np.int64), nimg * group_detr)
    img = np.tile(np.repeat(np.arange(nimg, dtype=np.int64), group_detr), layers)
    grp = np.tile(np.arange(group_detr, dtype=np.int64), layers * nimg)
    keep = sz[img] > 0
    lay, img, grp = lay[keep], img[keep], grp[keep]
    pr = np.zeros(lay.shape[0], dtype=_lib.PROBLEM_DTYPE)
    if layout == _lib.LAYOUT_QUERY_MAJOR:
        pr["cost_offset"] = lay * queries * ld + grp * qg * ld + offsets[img]
    else:
        pr["cost_offset"] = lay * total_t * ld + offsets[img] * ld + grp * qg
    pr["out_offset"] = image_base[lay * nimg + img] + grp * pairs[img]
    pr["num_queries"] = qg
    pr["num_targets"] = sz[img]
    pr["query_base"] = grp * qg
    return pr, [int(x) for x in per_image], int(image_base[-1]), offsets


class _PlanCache:
    """LRU of step plans keyed by sizes and shape; the last hit is also kept by the
    identity of its sizes tuple, so a training loop that reuses one sizes object
    skips hashing it."""

    def __init__(self, capacity: int = 64):
        self.capacity = capacity
        self._d: OrderedDict[tuple, StepPlan] = OrderedDict()
        self._last: tuple | None = None  # (sizes object, rest of the key, plan)

    def get(self, key: tuple, make) -> StepPlan:
        last = self._last
        if last is not None and last[0] is key[0] and last[1] == key[1:]:
            return last[2]
        hit = self._get(key, make)
        self._last = (key[0], key[1:], hit)
        return hit

    def _get(self, key: tuple, make) -> StepPlan:
        hit = self._d.get(key)
        if hit is not None:
            self._d.move_to_end(key)
            return hit
        value = make()
        self._d[key] = value
        if len(self._d) > self.capacity:
            self._d.popitem(last=False)
        return value

    def clear(self) -> None:
        self._d.clear()
        self._last = None


_PLANS = _PlanCache()


def plan_step(sizes: Sequence[int], layers: int, queries: int, group_detr: int, ld: int,
              device: torch.device, layout: int = _lib.LAYOUT_QUERY_MAJOR,
              tile_cap: int | None = None) -> StepPlan:
    """Cached host planning plus ONE non-blocking pinned upload of descriptors and offsets."""
    if type(sizes) is not tuple:
        sizes = tuple(int(s) for s in sizes)
    cap = _lib.default_tile_cap() if tile_cap is None else int(tile_cap)
    key = (sizes, layers, queries, group_detr, ld, layout, cap, str(device))

    def make() -> StepPlan:
        pr, per_image, total, offsets = build_problems(sizes, layers, queries, group_detr, ld, layout)
        need = pr["num_queries"].astype(np.int64) * pr["num_targets"].astype(np.int64)
        order = np.argsort(-need, kind="stable")
        pr = np.ascontiguousarray(pr[order])
        sq, st = strides(layout, ld)
        plan, ctas = _lib.make_plan(pr, sq, st, cap)
        pbytes = pr.view(np.uint8).reshape(-1)
        cbytes = ctas.view(np.uint8).reshape(-1)
        off32 = offsets.astype(np.int32)
        ctas_byte = (pbytes.shape[0] + 15) // 16 * 16
        offsets_byte = (ctas_byte + cbytes.shape[0] + 15) // 16 * 16
        blob = np.zeros(offsets_byte + off32.nbytes, dtype=np.uint8)
        blob[: pbytes.shape[0]] = pbytes
        blob[ctas_byte: ctas_byte + cbytes.shape[0]] = cbytes
        blob[offsets_byte:] = off32.view(np.uint8)
        host = torch.from_numpy(blob).pin_memory()
        dev = host.to(device, non_blocking=True)
        return StepPlan(sizes, layers, queries, group_detr, layout, ld, pr, order, plan, total, per_image, dev,
                        ctas_byte, offsets_byte, tuple(per_image))

    return _PLANS.get(key, make)


# --------------------------------------------------------------------------- kernels


def _stack_layer_outputs(outputs_list: Sequence[dict]) -> tuple[torch.Tensor, torch.Tensor]:
    logits = [o["pred_logits"] for o in outputs_list]
    boxes = [o["pred_boxes"] for o in outputs_list]
    for i, (lg, bx) in enumerate(zip(logits, boxes)):
        _require_cuda(lg, f"outputs[{i}]['pred_logits']")
        _require_cuda(bx, f"outputs[{i}]['pred_boxes']")
        if lg.dim() != 3 or bx.dim() != 3 or bx.shape[-1] != 4 or lg.shape[:2] != bx.shape[:2]:
            raise ValueError("expected pred_logits [B, Q, C] and pred_boxes [B, Q, 4]")
    if len(outputs_list) == 1:
        return logits[0].unsqueeze(0), boxes[0].unsqueeze(0)
    return torch.stack(logits), torch.stack(boxes)


def _prepare_predictions(logits: torch.Tensor, boxes: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _require_cuda(logits, "pred_logits")
    _require_cuda(boxes, "pred_boxes")
    if logits.dim() != 4 or boxes.dim() != 4 or boxes.shape[-1] != 4 or logits.shape[:3] != boxes.shape[:3]:
        raise ValueError("expected pred_logits [L, B, Q, C] and pred_boxes [L, B, Q, 4]")
    logits = logits.to(torch.float32).contiguous()
    boxes = _aligned16(boxes.to(torch.float32).contiguous())
    return logits, boxes


def launch_cost(logits: torch.Tensor, boxes: torch.Tensor, labels: torch.Tensor, tgt_boxes: torch.Tensor,
                offsets_ptr: int, sum_t: int, ld: int, layout: int, weights: dict, out: torch.Tensor,
                stream: ctypes.c_void_p | None = None) -> None:
    """Enqueue ``rfm_cost`` for logits [L,B,Q,C] / boxes [L,B,Q,4] into ``out``."""
    layers, nimg, queries, ncls = logits.shape
    lib = _lib.load()
    _lib.check("rfm_cost", lib.rfm_cost(
        _ptr(logits), _ptr(boxes), _ptr(labels), _ptr(tgt_boxes), ctypes.c_void_p(offsets_ptr),
        layers, nimg, queries, ncls, sum_t, ld, layout,
        float(weights["cost_class"]), float(weights["cost_bbox"]), float(weights["cost_giou"]),
        float(weights["focal_alpha"]), _ptr(out), _stream_handle(out.device) if stream is None else stream))


def launch_lsap(cost: torch.Tensor, plan: StepPlan, pairs: torch.Tensor, status: torch.Tensor | None,
                stream: ctypes.c_void_p | None = None, push: int | None = None) -> None:
    """Enqueue ``rfm_lsap`` over a planned step; ``pairs`` is int64 [2, total_pairs].  With ``push`` (the
    device address of a stored ``rfm_pair_push``; ``rfm_lsap_push``) every pair also goes to the push
    list's destinations."""
    lib = _lib.load()
    ws = None
    if plan.plan.workspace_bytes > 0:
        ws = torch.empty(int(plan.plan.workspace_bytes), dtype=torch.uint8, device=cost.device)
    args = (_ptr(cost), ctypes.c_void_p(plan.problems_ptr), ctypes.c_void_p(plan.ctas_ptr), ctypes.byref(plan.plan),
            _ptr(pairs[0]), _ptr(pairs[1]), _ptr(status), _ptr(ws))
    st = _stream_handle(cost.device) if stream is None else stream
    if push is None:
        _lib.check("rfm_lsap", lib.rfm_lsap(*args, st))
    else:
        _lib.check("rfm_lsap_push", lib.rfm_lsap_push(*args, ctypes.c_void_p(push), st))


def launch_match(logits: torch.Tensor, boxes: torch.Tensor, labels: torch.Tensor, tgt_boxes: torch.Tensor,
                 plan: StepPlan, sum_t: int, weights: dict, cost: torch.Tensor, pairs: torch.Tensor,
                 status: torch.Tensor | None, stream: ctypes.c_void_p | None = None,
                 push: int | None = None) -> None:
    """Enqueue ``rfm_match``: the cost kernel into the target-major ``cost`` [L, S, ld] and the solver over
    it, overlapped at their boundary (no memset between them, programmatic launch of the solver).  With
    ``push`` (the device address of a stored ``rfm_pair_push``; ``rfm_match_push``) every pair also goes
    to the push list's destinations."""
    layers, nimg, queries, ncls = logits.shape
    lib = _lib.load()
    ws = None
    if plan.plan.workspace_bytes > 0:
        ws = torch.empty(int(plan.plan.workspace_bytes), dtype=torch.uint8, device=cost.device)
    args = (_ptr(logits), _ptr(boxes), _ptr(labels), _ptr(tgt_boxes), ctypes.c_void_p(plan.offsets_ptr),
            layers, nimg, queries, ncls, sum_t, plan.ld,
            float(weights["cost_class"]), float(weights["cost_bbox"]), float(weights["cost_giou"]),
            float(weights["focal_alpha"]), _ptr(cost), ctypes.c_void_p(plan.problems_ptr),
            ctypes.c_void_p(plan.ctas_ptr), ctypes.byref(plan.plan), _ptr(pairs[0]), _ptr(pairs[1]), _ptr(status),
            _ptr(ws))
    st = _stream_handle(cost.device) if stream is None else stream
    if push is None:
        _lib.check("rfm_match", lib.rfm_match(*args, st))
    else:
        _lib.check("rfm_match_push", lib.rfm_match_push(*args, ctypes.c_void_p(push), st))


def raise_on_status(status: torch.Tensor) -> None:
    """Host check of per-problem solver status (synchronises; SciPy's error messages)."""
    st = status.cpu()
    if bool((st == _lib.STATUS_INVALID).any()):
        raise ValueError("matrix contains invalid numeric entries")
    if bool((st == _lib.STATUS_INFEASIBLE).any()):
        raise ValueError("cost matrix is infeasible")
    if bool((st != _lib.STATUS_OK).any()):
        raise RuntimeError("assignment solver reached its iteration bound")


# --------------------------------------------------------------------------- matcher


def _record(events: dict | None, name: str) -> None:
    if events is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events.setdefault(name, []).append(ev)


def match_packed(pred_logits: torch.Tensor, pred_boxes: torch.Tensor, targets: PackedTargets,
                 group_detr: int = 1, *, weights: dict | None = None, check_status: bool = False,
                 extras: dict | None = None, events: dict | None = None,
                 out: torch.Tensor | None = None, push: int | None = None) -> MatchResult:
    """One matcher step over logits ``[L, B, Q, C]`` and boxes ``[L, B, Q, 4]``, two launches.

    ``out``, when given, is an int64 ``[2, total_pairs]`` tensor (rows contiguous, e.g. a view
    into a collective's send buffer) the pairs are written into.  ``push``, when given, is the
    device address of a stored ``rfm_pair_push`` list of further destinations (other ranks'
    gathered buffers, see ``sharded.PeerExchange``) the solver writes every pair into as well.
    ``extras``, when given, receives the target-major cost buffer ``[L, S, ld]``
    (``"cost"``), its row stride and the step plan.  ``events``, when given,
    collects CUDA events recorded on the launching stream around each kernel
    (``"cost"`` and ``"lsap"``: start/end pairs); the step is then issued as two
    calls (``rfm_cost``, ``rfm_lsap``) instead of the one ``rfm_match``.
    """
    w = DEFAULT_WEIGHTS if weights is None else weights
    logits, boxes = _prepare_predictions(pred_logits, pred_boxes)
    tg = targets.checked()
    device = logits.device
    layers, nimg, queries, _ = logits.shape
    if len(tg.sizes) != nimg:
        raise ValueError(f"{len(tg.sizes)} targets for a batch of {nimg} images")
    sum_t = tg.total
    ld = _round4(queries)
    layout = _lib.LAYOUT_TARGET_MAJOR
    plan = plan_step(tg.sizes, layers, queries, group_detr, ld, device, layout)
    cost = torch.empty((layers, sum_t, ld), dtype=torch.float32, device=device)
    if out is None:
        pairs = torch.empty((2, plan.total_pairs), dtype=torch.int64, device=device)
    else:
        if (out.dtype != torch.int64 or out.device != device or tuple(out.shape) != (2, plan.total_pairs)
                or (plan.total_pairs and out.stride(1) != 1)):
            raise ValueError(f"out must be an int64 [2, {plan.total_pairs}] tensor with contiguous rows on {device}")
        pairs = out
    status = torch.empty(plan.problems.shape[0], dtype=torch.int32, device=device) if check_status else None
    stream = _stream_handle(device)
    if events is None and sum_t > 0 and plan.problems.shape[0] > 0:
        # one call: the cost kernel and the solver overlapped at their boundary
        launch_match(logits, boxes, tg.labels, tg.boxes, plan, sum_t, w, cost, pairs, status, stream, push)
    else:
        # two calls, so that events can be recorded around each kernel
        if sum_t > 0:
            _record(events, "cost")
            launch_cost(logits, boxes, tg.labels, tg.boxes, plan.offsets_ptr, sum_t, ld, layout, w, cost, stream)
            _record(events, "cost")
        if plan.problems.shape[0] > 0:
            _record(events, "lsap")
            launch_lsap(cost, plan, pairs, status, stream, push)
            _record(events, "lsap")
    if status is not None:
        raise_on_status(status)
    if extras is not None:
        extras.update(cost=cost, ld=ld, plan=plan, layout=layout)
    return MatchResult(pairs, plan.per_image, layers, nimg, plan.per_image_key)


def match_layers(outputs_list: Sequence[dict], targets: Sequence[dict] | PackedTargets, group_detr: int = 1, *,
                 weights: dict | None = None, check_status: bool = False, return_cost: bool = False,
                 extras: dict | None = None, events: dict | None = None) -> Any:
    """Match every decoder layer of one step against the same targets (the stacked
    single-pass path of patches.py:235-249), in two launches.

    Returns one list of per-image ``(query_idx, target_idx)`` tuples per layer; with
    ``return_cost`` also the compact ``[L, Q, sum T]`` cost matrix the solver used
    (a transposed view of the target-major buffer).
    """
    if not outputs_list:
        return []
    logits, boxes = _stack_layer_outputs(outputs_list)
    packed = targets if isinstance(targets, PackedTargets) else PackedTargets.from_list(targets, logits.device)
    ex = {} if (extras is None and return_cost) else extras
    res = match_packed(logits, boxes, packed, group_detr, weights=weights, check_status=check_status,
                       extras=ex, events=events)
    lists = res.as_lists()
    if return_cost:
        q = logits.shape[2]
        return lists, ex["cost"][:, :, :q].transpose(1, 2)
    return lists


def compute_compact_detection_cost_matrix(outputs: dict, targets: Sequence[dict] | PackedTargets, *,
                                          weights: dict | None = None) -> torch.Tensor:
    """Compact ``[Q, sum T]`` cost (``[L, Q, sum T]`` for 4-D logits), contiguous float32.

    Same result as the triton_matcher patch's method (patches.py:123-149) without the
    padded intermediate.  Labels are always clamped into ``[0, C-1]``
    (kernels_matcher.py:133-134).
    """
    w = DEFAULT_WEIGHTS if weights is None else weights
    lg, bx = outputs["pred_logits"], outputs["pred_boxes"]
    _require_cuda(lg, "pred_logits")
    squeeze = lg.dim() == 3
    if squeeze:
        lg, bx = lg.unsqueeze(0), bx.unsqueeze(0)
    lg, bx = _prepare_predictions(lg, bx)
    layers, nimg, queries, _ = lg.shape
    packed = targets if isinstance(targets, PackedTargets) else PackedTargets.from_list(targets, lg.device)
    tg = packed.checked()
    sum_t = sum(tg.sizes)
    out = torch.empty((layers, queries, sum_t), dtype=torch.float32, device=lg.device)
    if sum_t > 0:
        offs = torch.from_numpy(np.concatenate([[0], np.cumsum(tg.sizes)]).astype(np.int32)).pin_memory()
        offs = offs.to(lg.device, non_blocking=True)
        launch_cost(lg, bx, tg.labels, tg.boxes, offs.data_ptr(), sum_t, sum_t, _lib.LAYOUT_QUERY_MAJOR, w, out)
    return out[0] if squeeze else out


def assign_padded(cost_matrices: Sequence[torch.Tensor], sizes: Sequence[int], group_width: int,
                  group_detr: int, *, check_status: bool = False) -> list[list[tuple[torch.Tensor, torch.Tensor]]]:
    """``_assignment._assign_padded`` contract (patches.py:379-418), solved in place.

    ``cost_matrices`` holds one compact ``[group_width * group_detr, sum T]``
    matrix per layer.  No padding, stacking or sorting pass: the solver reads each
    ``[group_width, T_b]`` block where it lies and writes the pairs at their final
    position.  Returns, per layer, per image, ``(query_idx, target_idx)``.
    """
    results = []
    for layer, cost in enumerate(cost_matrices):
        _require_cuda(cost, f"cost_matrices[{layer}]")
        if cost.dtype != torch.float32:
            cost = cost.float()
        if cost.dim() != 2 or cost.stride(1) != 1:
            cost = cost.contiguous()
        queries = group_width * group_detr
        if cost.shape[0] != queries or cost.shape[1] != sum(sizes):
            raise ValueError(f"cost matrix {tuple(cost.shape)} does not match {queries} queries x {sum(sizes)} targets")
        ld = int(cost.stride(0))
        plan = plan_step(sizes, 1, queries, group_detr, ld, cost.device, _lib.LAYOUT_QUERY_MAJOR)
        pairs = torch.empty((2, plan.total_pairs), dtype=torch.int64, device=cost.device)
        status = torch.empty(plan.problems.shape[0], dtype=torch.int32, device=cost.device) if check_status else None
        if plan.problems.shape[0] > 0:
            launch_lsap(cost, plan, pairs, status)
        if status is not None:
            raise_on_status(status)
        results.append(MatchResult(pairs, plan.per_image, 1, len(sizes)).layer(0))
    return results


def batch_linear_assignment(cost: torch.Tensor, *, check_status: bool = False) -> torch.Tensor:
    """``torch_linear_assignment.batch_linear_assignment`` contract (kernels_lap.py:336-341).

    ``cost`` ``[P, W, T]`` float32 CUDA -> ``[P, W]`` int64 task of each worker, -1
    when unassigned, each problem solved as ``scipy.optimize.linear_sum_assignment``
    solves it.
    """
    _require_cuda(cost, "cost")
    if cost.dim() != 3:
        raise ValueError("cost must be [problems, workers, tasks]")
    cost = cost.to(torch.float32).contiguous()
    nprob, workers, tasks = cost.shape
    if max(workers, tasks) > _lib.MAX_COLS:
        raise ValueError(f"problems wider than {_lib.MAX_COLS} columns are outside the supported envelope")
    lib = _lib.load()
    matching = torch.empty((nprob, workers), dtype=torch.int64, device=cost.device)
    if nprob == 0 or workers == 0:
        return matching
    ws_bytes = int(lib.rfm_lsap_dense_workspace_bytes(nprob, workers, tasks))
    if ws_bytes < 0:
        raise _lib.RfmError("rfm_lsap_dense_workspace_bytes", -ws_bytes)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cost.device) if ws_bytes else None
    status = torch.empty(nprob, dtype=torch.int32, device=cost.device) if check_status else None
    _lib.check("rfm_lsap_dense", lib.rfm_lsap_dense(
        _ptr(cost), nprob, workers, tasks, _ptr(matching), _ptr(status), _ptr(ws), _stream_handle(cost.device)))
    if status is not None:
        raise_on_status(status)
    return matching


class HungarianMatcher(torch.nn.Module):
    """Drop-in for ``rfdetr.models.matcher.HungarianMatcher`` (detection path).

    Constructor arguments mirror rf-detr's (``cost_class``, ``cost_bbox``,
    ``cost_giou``, ``focal_alpha``; focal gamma is fixed at 2,
    kernels_matcher.py:49-50).
    """

    def __init__(self, cost_class: float = 1.0, cost_bbox: float = 1.0, cost_giou: float = 1.0,
                 focal_alpha: float = 0.25, **unused: Any):
        super().__init__()
        self.cost_class = float(cost_class)
        self.cost_bbox = float(cost_bbox)
        self.cost_giou = float(cost_giou)
        self.focal_alpha = float(focal_alpha)
        if self.cost_class == 0 and self.cost_bbox == 0 and self.cost_giou == 0:
            raise ValueError("all costs can't be 0")

    @property
    def weights(self) -> dict:
        return {"cost_class": self.cost_class, "cost_bbox": self.cost_bbox, "cost_giou": self.cost_giou,
                "focal_alpha": self.focal_alpha}

    @torch.no_grad()
    def forward(self, outputs: dict, targets: Sequence[dict], group_detr: int = 1):
        if "pred_masks" in outputs:
            raise NotImplementedError("segmentation matching is outside this matcher (detection path only)")
        return match_layers([outputs], targets, group_detr, weights=self.weights)[0]

    @torch.no_grad()
    def forward_layers(self, outputs_list: Sequence[dict], targets: Sequence[dict], group_detr: int = 1):
        """All decoder layers of a step at once (the stacked_costs path, patches.py:235-249)."""
        return match_layers(outputs_list, targets, group_detr, weights=self.weights)

    @torch.no_grad()
    def _compute_compact_detection_cost_matrix(self, outputs: dict, targets: Sequence[dict], *,
                                               clamp_target_labels: bool = False) -> torch.Tensor:
        return compute_compact_detection_cost_matrix(outputs, targets, weights=self.weights)
