"""rfm_cost on the GPU against the numpy oracle and the torch-operator golden fixtures."""

import numpy as np
import pytest
import torch

from conftest import COST_RTOL
from golden_io import matcher_case, names, to_targets
from oracle import cost as ocost
from rfdetr_training_throughput_b200 import matcher, workloads

pytestmark = pytest.mark.gpu


def _gpu_cost(logits, boxes, labels, tboxes, weights):
    dev = torch.device("cuda")
    outputs = {"pred_logits": torch.as_tensor(logits, device=dev), "pred_boxes": torch.as_tensor(boxes, device=dev)}
    out = matcher.compute_compact_detection_cost_matrix(outputs, to_targets(labels, tboxes, dev), weights=weights)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _assert_close(gpu, ref):
    """The cost contract: |gpu - ref| <= 1e-5 * max(|ref|, 1).  That is plain relative error for
    entries of magnitude >= 1 (checked separately below) and an absolute 1e-5 below it, where a
    cost is the small difference of larger terms (5 L1 + 2 focal - 2 GIoU) and its rounding error
    scales with those terms rather than with the difference."""
    assert gpu.shape == ref.shape
    assert np.isfinite(gpu).all()
    bound = COST_RTOL * np.maximum(np.abs(ref), 1.0)
    worst = float((np.abs(gpu - ref) / bound).max(initial=0.0))
    assert worst <= 1.0, f"cost differs by {worst:.3f}x the tolerance"
    big = np.abs(ref) >= 1.0
    if big.any():
        assert float((np.abs(gpu - ref)[big] / np.abs(ref)[big]).max()) <= COST_RTOL


@pytest.mark.parametrize("name", names("matcher"))
def test_cost_golden(name):
    logits, boxes, labels, tboxes, _g, w, golden, _p = matcher_case(name)
    gpu = _gpu_cost(logits, boxes, labels, tboxes, w)
    _assert_close(gpu, ocost.compact_cost(logits, boxes, labels, tboxes, **w))
    _assert_close(gpu, golden)


@pytest.mark.parametrize("name", ["cpu1", "step", "crowd", "ties"])
def test_cost_workloads(name):
    wl = workloads.make(name, images=4) if name in ("crowd", "ties") else workloads.make(name)
    labels = [t["labels"].numpy() for t in wl.targets]
    tboxes = [t["boxes"].numpy() for t in wl.targets]
    gpu = _gpu_cost(wl.pred_logits.numpy(), wl.pred_boxes.numpy(), labels, tboxes, wl.weights)
    _assert_close(gpu, ocost.compact_cost(wl.pred_logits.numpy(), wl.pred_boxes.numpy(), labels, tboxes, **wl.weights))


def test_box_terms_are_tight():
    """With cost_class = 0 only L1 and GIoU remain: every add and multiply follows the reference
    chain's float32 order exactly, so the two fast quotients are the only difference (~1 ulp)."""
    wl = workloads.make("step", layers=2)
    w = dict(wl.weights, cost_class=0.0)
    labels = [t["labels"].numpy() for t in wl.targets]
    tboxes = [t["boxes"].numpy() for t in wl.targets]
    gpu = _gpu_cost(wl.pred_logits.numpy(), wl.pred_boxes.numpy(), labels, tboxes, w)
    ref = ocost.compact_cost(wl.pred_logits.numpy(), wl.pred_boxes.numpy(), labels, tboxes, **w)
    assert float((np.abs(gpu - ref) / np.maximum(np.abs(ref), 1.0)).max()) <= 1e-6
    assert float((gpu == ref).mean()) > 0.5


def test_labels_are_clamped_and_degenerate_boxes_finite():
    wl = workloads.make("cpu1")
    labels = [np.array([-3, 0, 1, 7, 1, 0, 2, 5, -1, 0, 1, 1], dtype=np.int64)]
    tboxes = [wl.targets[0]["boxes"].numpy().copy()]
    tboxes[0][:, 2:] = 0.0
    boxes = wl.pred_boxes.numpy().copy()
    boxes[..., 2:] = 0.0
    gpu = _gpu_cost(wl.pred_logits.numpy(), boxes, labels, tboxes, wl.weights)
    _assert_close(gpu, ocost.compact_cost(wl.pred_logits.numpy(), boxes, labels, tboxes, **wl.weights))


def test_both_layouts_are_bit_identical():
    """The fused step's target-major matrix is the transpose of the drop-in compact matrix, bit for bit."""
    for name, kw in (("step", {"layers": 2, "images": 3}), ("crowd", {"images": 2})):
        wl = workloads.make(name, **kw)
        dev = torch.device("cuda")
        _, tmajor = matcher.match_layers(wl.outputs_list(dev), wl.targets_on(dev), wl.group_detr,
                                         weights=wl.weights, return_cost=True)
        outs = {"pred_logits": wl.pred_logits.to(dev), "pred_boxes": wl.pred_boxes.to(dev)}
        qmajor = matcher.compute_compact_detection_cost_matrix(outs, wl.targets_on(dev), weights=wl.weights)
        s = sum(wl.sizes)
        assert qmajor.shape == (wl.layers, wl.queries, s) and qmajor.is_contiguous()
        assert torch.equal(tmajor, qmajor)


def test_target_major_padding_is_zero():
    wl = workloads.make("step", layers=1, images=3)
    dev = torch.device("cuda")
    logits = torch.zeros((1, 2, 6, 2), device=dev)
    boxes = torch.full((1, 2, 6, 4), 0.5, device=dev)
    packed = matcher.PackedTargets(torch.zeros(3, dtype=torch.int64, device=dev),
                                   torch.full((3, 4), 0.25, device=dev), (1, 2))
    ex = {}
    matcher.match_packed(logits, boxes, packed, 1, weights=wl.weights, extras=ex)
    cost = ex["cost"]
    assert cost.shape == (1, 3, 8)
    assert bool((cost[..., 6:] == 0).all()) and bool((cost[..., :6] != 0).all())


def test_empty_targets():
    wl = workloads.make("step", layers=1, images=2)
    dev = torch.device("cuda")
    targets = [{"labels": torch.zeros(0, dtype=torch.int64, device=dev),
                "boxes": torch.zeros(0, 4, device=dev)} for _ in range(2)]
    out = matcher.compute_compact_detection_cost_matrix(wl.outputs_list(dev)[0], targets, weights=wl.weights)
    assert out.shape == (wl.queries, 0)


def test_image_lookup_across_many_empty_images():
    """Targets of one CTA spread over hundreds of images, most of them empty: the
    shared window of image offsets and its global-memory fallback both give each
    target its own image's predictions (both layouts, against the oracle)."""
    rng = np.random.default_rng(7)
    nimg, queries = 700, 8
    sizes = np.zeros(nimg, dtype=np.int64)
    sizes[[0, 1, 130, 131, 300, 450, 451, 699]] = [2, 1, 3, 1, 2, 1, 4, 2]
    logits = rng.normal(0.0, 1.5, (1, nimg, queries, 2)).astype(np.float32)
    boxes = (1.0 / (1.0 + np.exp(-rng.normal(0.0, 1.0, (1, nimg, queries, 4))))).astype(np.float32)
    labels = [rng.integers(0, 2, int(t)).astype(np.int64) for t in sizes]
    tboxes = [np.concatenate([rng.uniform(0.1, 0.9, (int(t), 2)), rng.uniform(0.02, 0.5, (int(t), 2))],
                             axis=1).astype(np.float32) for t in sizes]
    w = dict(cost_class=2.0, cost_bbox=5.0, cost_giou=2.0, focal_alpha=0.25)
    ref = ocost.compact_cost(logits, boxes, labels, tboxes, **w)
    gpu = _gpu_cost(logits, boxes, labels, tboxes, w)
    _assert_close(gpu, ref)
    dev = torch.device("cuda")
    outputs = [{"pred_logits": torch.as_tensor(logits[0], device=dev),
                "pred_boxes": torch.as_tensor(boxes[0], device=dev)}]
    _, tmajor = matcher.match_layers(outputs, to_targets(labels, tboxes, dev), 1, weights=w, return_cost=True)
    assert torch.equal(tmajor.cpu(), torch.as_tensor(gpu).reshape(tmajor.shape))


@pytest.mark.parametrize("queries", [5, 7, 9])
def test_odd_query_counts_both_layouts_and_zero_padding(queries):
    """Q not a multiple of the per-thread query pair: the last pair is half padding (q >= Q) or
    all padding (ld - Q >= 2); pads are written as 0 and the real columns match the query-major
    matrix bit for bit."""
    rng = np.random.default_rng(queries)
    sizes = [3, 1, 4]
    logits = torch.as_tensor(rng.normal(0, 1.5, (1, 3, queries, 2)).astype(np.float32), device="cuda")
    boxes = torch.as_tensor((1 / (1 + np.exp(-rng.normal(0, 1, (1, 3, queries, 4))))).astype(np.float32),
                            device="cuda")
    labels = torch.as_tensor(rng.integers(0, 2, sum(sizes)), device="cuda")
    tboxes = torch.as_tensor(np.concatenate([rng.uniform(0.1, 0.9, (sum(sizes), 2)),
                                             rng.uniform(0.02, 0.5, (sum(sizes), 2))], 1).astype(np.float32),
                             device="cuda")
    packed = matcher.PackedTargets(labels, tboxes, tuple(sizes))
    w = dict(cost_class=2.0, cost_bbox=5.0, cost_giou=2.0, focal_alpha=0.25)
    ex = {}
    matcher.match_packed(logits, boxes, packed, 1, weights=w, extras=ex)
    offs = np.concatenate([[0], np.cumsum(sizes)])
    targets = [{"labels": labels[offs[b]:offs[b + 1]], "boxes": tboxes[offs[b]:offs[b + 1]]} for b in range(3)]
    qmajor = matcher.compute_compact_detection_cost_matrix({"pred_logits": logits, "pred_boxes": boxes}, targets,
                                                           weights=w)
    torch.cuda.synchronize()
    tm = ex["cost"]
    assert tm.shape[-1] == (queries + 3) // 4 * 4
    assert bool((tm[..., queries:] == 0).all())
    assert torch.equal(tm[..., :queries].transpose(1, 2), qmajor)
