"""Install the B200 matcher into an importable rf-detr, by the reference's patch names.

Mirrors the reference's plugin interface for this path (patches.py:704-735): a
``PATCHES`` registry of named, opt-in monkeypatches and ``apply_patches("a,b")``,
which applies them in order, returns one description per patch and raises
``KeyError`` on an unknown name.  The hot-path names keep their meaning:

``triton_matcher``  ``HungarianMatcher._compute_compact_detection_cost_matrix``
                    -> ``rfm_cost`` (patches.py:100-152)
``cuda_lap``        ``torch_linear_assignment.batch_linear_assignment``
                    -> ``rfm_lsap_dense`` (patches.py:291-327)
``device_indices``  ``rfdetr.models._assignment._assign_padded``
                    -> ``rfm_lsap`` on the compact matrices in place (patches.py:330-421)
``stacked_costs``   raise rf-detr's stacked-cost budget so all layers share one pass
                    (patches.py:235-249)
``matcher``         ``HungarianMatcher.forward`` -> the two-launch device step (new: the
                    whole matcher in one call, detection outputs only)
``box_loss``        ``SetCriterion.loss_boxes`` -> ``rfm_box_loss_forward/backward`` on the
                    matcher's index pairs (new: the criterion consumer of the indices,
                    DETR's loss_boxes contract)
``fused_msda``      rf-detr's deformable-attention core ``ms_deform_attn_core_pytorch`` ->
                    ``rfm_msda_forward/backward`` (patches.py:566-614); export-layout calls
                    (rank-5 sampling locations) keep the original core
``fused_msda_native`` ``MSDeformAttn.forward`` with the value kept in the kernel's layout, no
                    copy (patches.py:617-635); export mode keeps the original forward
``label_loss``      ``SetCriterion.loss_labels`` -> ``rfm_label_loss_forward/backward`` on the
                    index pairs (new: the criterion's classification loss, the IoU-aware
                    BCE when the criterion has ``ia_bce_loss`` set, else the sigmoid focal
                    loss; the varifocal and position-supervised variants raise)

Unlike the reference there is no fallback to the original implementation for
CPU tensors or out-of-envelope inputs: the patched functions raise instead.
"""

from __future__ import annotations

import importlib
from typing import Callable

from . import matcher as _m


def _module(name: str):
    try:
        return importlib.import_module(name)
    except ImportError as e:  # pragma: no cover - exercised with a stub in tests
        raise ImportError(f"{name} is not importable; install rf-detr to patch it") from e


def _apply_triton_matcher() -> str:
    cls = _module("rfdetr.models.matcher").HungarianMatcher

    def compute_compact_detection_cost_matrix(self, outputs, targets, *, clamp_target_labels=False):
        if "pred_masks" in outputs:
            raise NotImplementedError("segmentation costs are outside this matcher")
        weights = {"cost_class": self.cost_class, "cost_bbox": self.cost_bbox, "cost_giou": self.cost_giou,
                   "focal_alpha": self.focal_alpha}
        return _m.compute_compact_detection_cost_matrix(outputs, targets, weights=weights)

    cls._compute_compact_detection_cost_matrix = compute_compact_detection_cost_matrix
    return "triton_matcher: compact cost matrix built by the sm_100a rfm_cost kernel"


def _apply_cuda_lap() -> str:
    module = _module("torch_linear_assignment.assignment")
    module.batch_linear_assignment = _m.batch_linear_assignment
    package = _module("torch_linear_assignment")
    package.batch_linear_assignment = _m.batch_linear_assignment
    return "cuda_lap: batch_linear_assignment solved by the SciPy-exact sm_100a solver"


def _apply_device_indices() -> str:
    module = _module("rfdetr.models._assignment")

    def assign_padded(cost_matrices, sizes, group_width, group_detr):
        return _m.assign_padded(cost_matrices, sizes, group_width, group_detr)

    module._assign_padded = assign_padded
    return "device_indices: assignment solved in place and unpacked on the device"


def _apply_stacked_costs() -> str:
    module = _module("rfdetr.models.matcher")
    module._STACKED_COST_ELEMENT_LIMIT = 1 << 40
    return "stacked_costs: matcher folds all layers into one cost-construction pass"


def _apply_matcher() -> str:
    cls = _module("rfdetr.models.matcher").HungarianMatcher
    cls.forward = _m.HungarianMatcher.forward
    cls.forward_layers = _m.HungarianMatcher.forward_layers
    if not hasattr(cls, "weights"):
        cls.weights = _m.HungarianMatcher.weights
    return "matcher: HungarianMatcher.forward runs the two-launch device step"


def _apply_box_loss() -> str:
    cls = _module("rfdetr.models.criterion").SetCriterion
    from .loss import criterion_loss_boxes

    def loss_boxes(self, outputs, targets, indices, num_boxes):
        return criterion_loss_boxes(outputs, targets, indices, num_boxes)

    cls.loss_boxes = loss_boxes
    return "box_loss: SetCriterion.loss_boxes computed from the index pairs by the sm_100a loss kernels"


def _apply_label_loss() -> str:
    cls = _module("rfdetr.models.criterion").SetCriterion
    from .loss import criterion_loss_labels

    def loss_labels(self, outputs, targets, indices, num_boxes, log=True):
        if getattr(self, "use_varifocal_loss", False) or getattr(self, "use_position_supervised_loss", False):
            raise NotImplementedError("only the IoU-aware BCE and the sigmoid focal classification losses run here")
        mode = "ia_bce" if getattr(self, "ia_bce_loss", False) else "focal"
        return criterion_loss_labels(outputs, targets, indices, num_boxes, log, mode=mode,
                                     focal_alpha=getattr(self, "focal_alpha", 0.25))

    cls.loss_labels = loss_labels
    return "label_loss: SetCriterion.loss_labels computed from the index pairs by the sm_100a loss kernels"


def _apply_fused_msda() -> str:
    module = _module("rfdetr.models.ops.modules.ms_deform_attn")
    from .msda import deformable_attention

    original = module.ms_deform_attn_core_pytorch

    def core(value, value_spatial_shapes, sampling_locations, attention_weights, value_spatial_shapes_hw=None):
        if sampling_locations.dim() != 6:  # the export layout: not a training call
            return original(value, value_spatial_shapes, sampling_locations, attention_weights,
                            value_spatial_shapes_hw=value_spatial_shapes_hw)
        return deformable_attention(value, value_spatial_shapes, sampling_locations, attention_weights)

    module.ms_deform_attn_core_pytorch = core
    return "fused_msda: deformable attention core on the sm_100a rfm_msda kernels"


def _apply_fused_msda_native() -> str:
    cls = _module("rfdetr.models.ops.modules.ms_deform_attn").MSDeformAttn
    from .msda import module_forward

    original = cls.forward

    def forward(self, *args, **kwargs):
        if getattr(self, "_export", False):
            return original(self, *args, **kwargs)
        return module_forward(self, *args, **kwargs)

    cls.forward = forward
    return "fused_msda_native: MSDeformAttn.forward reaches the rfm_msda kernels without a layout copy"


PATCHES: dict[str, Callable[[], str]] = {
    "triton_matcher": _apply_triton_matcher,
    "cuda_lap": _apply_cuda_lap,
    "device_indices": _apply_device_indices,
    "stacked_costs": _apply_stacked_costs,
    "matcher": _apply_matcher,
    "box_loss": _apply_box_loss,
    "label_loss": _apply_label_loss,
    "fused_msda": _apply_fused_msda,
    "fused_msda_native": _apply_fused_msda_native,
}


def apply_patches(names: str) -> list[str]:
    """Apply a comma-separated patch list; returns one description per patch."""
    applied: list[str] = []
    for name in [item.strip() for item in names.split(",") if item.strip()]:
        if name not in PATCHES:
            raise KeyError(f"unknown patch {name!r}; available: {sorted(PATCHES)}")
        applied.append(PATCHES[name]())
    return applied
