"""MatchGraph: the captured step must return exactly what match_packed returns (index pairs:
exact equality) for every batch of its shape, including the wide solver layout, and must
refuse batches of another shape.  The replayed pairs of the production step are also checked
directly against SciPy on the device-computed cost matrix."""

import numpy as np
import pytest
import torch
from scipy.optimize import linear_sum_assignment

from oracle.matcher import solve_blocks

from rfdetr_training_throughput_b200 import MatchGraph, MatchGraphCache, matcher, workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _inputs(wl):
    packed = matcher.PackedTargets.from_list(wl.targets_on(DEV), DEV)
    return wl.pred_logits.to(DEV), wl.pred_boxes.to(DEV), packed


def _eager(wl):
    logits, boxes, packed = _inputs(wl)
    return matcher.match_packed(logits, boxes, packed, wl.group_detr, weights=wl.weights).pairs.clone()


@pytest.mark.parametrize("name,kw", [("step", {}), ("sweep", {"images": 1024})])
def test_graph_replays_match_eager_steps(name, kw):
    wl = workloads.make(name, **kw)
    g = MatchGraph(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, weights=wl.weights)
    logits, boxes, packed = _inputs(wl)
    res = g(logits, boxes, packed.labels, packed.boxes)
    torch.cuda.synchronize()
    assert torch.equal(res.pairs, _eager(wl))
    # a second batch of the same shape: new predictions, new target boxes and labels
    gen = torch.Generator().manual_seed(5)
    logits2 = (wl.pred_logits + torch.randn(wl.pred_logits.shape, generator=gen)).to(DEV)
    boxes2 = torch.sigmoid(torch.randn(wl.pred_boxes.shape, generator=gen)).to(DEV)
    labels2 = torch.randint(0, wl.classes, packed.labels.shape, generator=gen).to(DEV)
    tboxes2 = (packed.boxes.cpu() * 0.5 + 0.25).to(DEV)
    res2 = g(logits2, boxes2, labels2, tboxes2)
    torch.cuda.synchronize()
    expect = matcher.match_packed(logits2, boxes2, matcher.PackedTargets(labels2, tboxes2, tuple(wl.sizes)),
                                  wl.group_detr, weights=wl.weights)
    torch.cuda.synchronize()
    assert torch.equal(res2.pairs, expect.pairs)
    assert res2.per_image == expect.per_image


def scipy_pairs(wl, logits, boxes, packed) -> np.ndarray:
    """SciPy's pairs for every (layer, image, group) block of the device-computed cost, in the packed
    order of a MatchResult (layer-major, images in order, groups in order)."""
    ex = {}
    matcher.match_packed(logits, boxes, packed, wl.group_detr, weights=wl.weights, extras=ex)
    cost = ex["cost"][:, :, : wl.queries].transpose(1, 2).cpu().numpy()  # compact [L, Q, S]
    cols = []
    for l in range(wl.layers):
        for q, t in solve_blocks(cost[l], wl.sizes, wl.group_detr, solver=linear_sum_assignment):
            cols.append(np.stack([q, t]))
    return np.concatenate(cols, axis=1)


def test_graph_replay_equals_scipy_on_the_device_cost():
    wl = workloads.make("step")
    g = MatchGraph(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, weights=wl.weights)
    logits, boxes, packed = _inputs(wl)
    res = g(logits, boxes, packed.labels, packed.boxes)
    torch.cuda.synchronize()
    assert np.array_equal(res.pairs.cpu().numpy(), scipy_pairs(wl, logits, boxes, packed))


def test_graph_refuses_other_shapes_and_cache_keys_by_shape():
    wl = workloads.make("step", layers=2, images=3)
    logits, boxes, packed = _inputs(wl)
    cache = MatchGraphCache(weights=wl.weights)
    first = cache(logits, boxes, packed, wl.group_detr)
    torch.cuda.synchronize()
    assert torch.equal(first.pairs, _eager(wl))
    g = cache.get(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, DEV)
    with pytest.raises(ValueError):
        g(logits[:, :2], boxes[:, :2], packed.labels, packed.boxes)
    wl2 = workloads.make("step", layers=2, images=4)
    logits2, boxes2, packed2 = _inputs(wl2)
    second = cache(logits2, boxes2, packed2, wl2.group_detr)
    torch.cuda.synchronize()
    assert torch.equal(second.pairs, _eager(wl2))
    assert cache.get(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, DEV) is g


def test_graph_replay_does_not_synchronise():
    wl = workloads.make("step")
    g = MatchGraph(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, weights=wl.weights)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        for _ in range(3):
            g.replay()
    finally:
        torch.cuda.set_sync_debug_mode(0)
    torch.cuda.synchronize()
