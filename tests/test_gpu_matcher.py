"""The whole matcher step on the GPU: HungarianMatcher.forward / forward_layers against the oracle."""

import numpy as np
import pytest
import torch
from scipy.optimize import linear_sum_assignment as scipy_lsa

from conftest import COST_RTOL
from oracle import cost as ocost
from oracle.lsap import linear_sum_assignment as oracle_lsa
from oracle.matcher import solve_blocks
from rfdetr_training_throughput_b200 import matcher, workloads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def _run(wl):
    res, cost = matcher.match_layers(wl.outputs_list(DEV), wl.targets_on(DEV), wl.group_detr,
                                     weights=wl.weights, return_cost=True)
    torch.cuda.synchronize()
    s = sum(wl.sizes)
    return res, cost[:, :, :s].cpu().numpy()


def _check_same_matrix(wl, res, cost, solver):
    """Indices identical to the reference solver run on the device-computed matrix."""
    for layer in range(wl.layers):
        expect = solve_blocks(cost[layer], wl.sizes, wl.group_detr, solver=solver)
        for b, (q, t) in enumerate(res[layer]):
            assert q.dtype == torch.int64 and t.dtype == torch.int64 and q.is_cuda
            assert np.array_equal(q.cpu().numpy(), expect[b][0]), (layer, b)
            assert np.array_equal(t.cpu().numpy(), expect[b][1]), (layer, b)


def _objective(cost_layer, sizes, pairs):
    total, col = 0.0, 0
    offs = np.concatenate([[0], np.cumsum(sizes)])
    for b, (q, t) in enumerate(pairs):
        q = np.asarray(q)
        t = np.asarray(t)
        total += float(cost_layer[q, offs[b] + t].astype(np.float64).sum()) if len(q) else 0.0
    return total


@pytest.mark.parametrize("name,kw", [("cpu1", {}), ("step", {}), ("ties", {}), ("crowd", {}),
                                     ("sweep", {"images": 128})])
def test_forward_matches_scipy_on_device_cost(name, kw):
    """Every persistent solver layout: one problem per CTA (cpu1, step: small batches), the early-load
    warps (ties, crowd: 64+ rows) and register warps pulling from the counter (sweep at 128 images:
    1,664 problems, more than fit at once one per CTA); the full sweep's wide layout is tested below."""
    wl = workloads.make(name, **kw)
    res, cost = _run(wl)
    _check_same_matrix(wl, res, cost, scipy_lsa)


@pytest.mark.parametrize("name", ["step", "ties", "crowd"])
def test_forward_against_full_oracle(name):
    """Cost within tolerance of the numpy oracle; the oracle's own assignment has the same objective."""
    wl = workloads.make(name)
    res, cost = _run(wl)
    labels = [t["labels"].numpy() for t in wl.targets]
    tboxes = [t["boxes"].numpy() for t in wl.targets]
    ref = ocost.compact_cost(wl.pred_logits.numpy(), wl.pred_boxes.numpy(), labels, tboxes, **wl.weights)
    assert (np.abs(cost - ref) <= COST_RTOL * np.maximum(np.abs(ref), 1.0)).all()
    for layer in range(wl.layers):
        oracle_pairs = solve_blocks(ref[layer], wl.sizes, wl.group_detr)
        mine = [(q.cpu().numpy(), t.cpu().numpy()) for q, t in res[layer]]
        a = _objective(ref[layer], wl.sizes, mine)
        b = _objective(ref[layer], wl.sizes, oracle_pairs)
        assert abs(a - b) <= 1e-4 * max(1.0, abs(b))


def test_full_sweep_against_oracle_on_device_cost():
    wl = workloads.make("sweep")
    res, cost = _run(wl)
    _check_same_matrix(wl, res, cost, oracle_lsa)


def test_result_structure_and_validity():
    wl = workloads.make("ties")
    res, _ = _run(wl)
    qg = wl.queries // wl.group_detr
    assert len(res) == wl.layers and len(res[0]) == wl.images
    for b, (q, t) in enumerate(res[0]):
        n = min(qg, wl.sizes[b])
        assert q.shape == (wl.group_detr * n,) and t.shape == q.shape
        if n == 0:
            continue
        q = q.cpu().numpy().reshape(wl.group_detr, n)
        t = t.cpu().numpy().reshape(wl.group_detr, n)
        for g in range(wl.group_detr):
            assert (q[g] >= g * qg).all() and (q[g] < (g + 1) * qg).all()
            assert len(np.unique(q[g])) == n
            assert len(np.unique(t[g])) == n and (t[g] >= 0).all() and (t[g] < wl.sizes[b]).all()
            assert (np.diff(q[g]) > 0).all()


def test_matcher_module_interface():
    wl = workloads.make("step", layers=1)
    m = matcher.HungarianMatcher(**wl.weights)
    out = m(wl.outputs_list(DEV)[0], wl.targets_on(DEV), group_detr=wl.group_detr)
    layers = m.forward_layers(wl.outputs_list(DEV), wl.targets_on(DEV), group_detr=wl.group_detr)
    assert len(out) == wl.images
    for (q1, t1), (q2, t2) in zip(out, layers[0]):
        assert torch.equal(q1, q2) and torch.equal(t1, t2)
    c = m._compute_compact_detection_cost_matrix(wl.outputs_list(DEV)[0], wl.targets_on(DEV))
    assert c.shape == (wl.queries, sum(wl.sizes))


def test_bf16_logits_are_accepted():
    wl = workloads.make("step", layers=1, images=2)
    outs = wl.outputs_list(DEV)
    outs[0]["pred_logits"] = outs[0]["pred_logits"].to(torch.bfloat16)
    res = matcher.match_layers(outs, wl.targets_on(DEV), wl.group_detr, weights=wl.weights)
    assert len(res[0]) == 2


def test_no_host_synchronisation():
    wl = workloads.make("step")
    outs, tgts = wl.outputs_list(DEV), wl.targets_on(DEV)
    matcher.match_layers(outs, tgts, wl.group_detr, weights=wl.weights)  # warm the plan cache
    wl2 = workloads.make("step", shard=3)  # new sizes: planning and upload happen inside the check
    outs2, tgts2 = wl2.outputs_list(DEV), wl2.targets_on(DEV)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        for _ in range(2):
            matcher.match_layers(outs, tgts, wl.group_detr, weights=wl.weights)
        matcher.match_layers(outs2, tgts2, wl2.group_detr, weights=wl2.weights)
    finally:
        torch.cuda.set_sync_debug_mode(0)
    torch.cuda.synchronize()


def test_status_reports_invalid_costs():
    wl = workloads.make("step", layers=1, images=2)
    outs = wl.outputs_list(DEV)
    outs[0]["pred_logits"] = outs[0]["pred_logits"].clone()
    outs[0]["pred_logits"][0, 5, :] = float("nan")
    with pytest.raises(ValueError, match="invalid"):
        matcher.match_layers(outs, wl.targets_on(DEV), wl.group_detr, weights=wl.weights, check_status=True)


def _narrow_batch(seed=21, images=800, group_detr=13, qg=64):
    rng = np.random.default_rng(seed)
    queries = group_detr * qg
    sizes = np.clip(rng.poisson(8, images), 1, 60)
    logits = rng.normal(-2.0, 1.5, (1, images, queries, 2)).astype(np.float32)
    boxes = (1.0 / (1.0 + np.exp(-rng.normal(0.0, 1.0, (1, images, queries, 4))))).astype(np.float32)
    labels = torch.as_tensor(np.concatenate([rng.integers(0, 2, t) for t in sizes]), device=DEV)
    tboxes = torch.as_tensor(np.concatenate([np.concatenate([rng.uniform(0.1, 0.9, (t, 2)), rng.uniform(0.02, 0.5, (t, 2))],
                                                            axis=1) for t in sizes]).astype(np.float32), device=DEV)
    return (torch.as_tensor(logits, device=DEV), torch.as_tensor(boxes, device=DEV),
            matcher.PackedTargets(labels, tboxes, tuple(int(t) for t in sizes)), group_detr)


def test_large_batch_reports_invalid_problem_only():
    """A NaN box in a 10,400-problem batch (the wide solver layout): exactly that (image, group)
    problem reports invalid entries, writes -1 pairs, and every other pair is unchanged."""
    logits, boxes, targets, group_detr = _narrow_batch()
    clean = matcher.match_packed(logits, boxes, targets, group_detr)
    bad_boxes = boxes.clone()
    bad_boxes[0, 5, 70, 2] = float("nan")  # image 5, query 70 -> group 1
    with pytest.raises(ValueError, match="invalid"):
        matcher.match_packed(logits, bad_boxes, targets, group_detr, check_status=True)
    res = matcher.match_packed(logits, bad_boxes, targets, group_detr)
    torch.cuda.synchronize()
    off = np.concatenate([[0], np.cumsum(res.per_image)])
    t5 = targets.sizes[5]
    lo = int(off[5]) + 1 * t5  # group 1 of image 5: pairs after group 0's t5 pairs
    diff = (res.pairs != clean.pairs).any(dim=0).nonzero().flatten().cpu().numpy()
    assert diff.min() >= lo and diff.max() < lo + t5
    assert bool((res.pairs[:, lo:lo + t5] == -1).all())


def test_large_batch_of_narrow_groups_against_oracle():
    """10,400 problems of 64 queries: a batch large enough for the solver's wide layout (duals and
    tie keys in shared memory) with the 128-column instantiation; indices identical to the C oracle
    on the device-computed matrix."""
    rng = np.random.default_rng(21)
    images, group_detr, qg = 800, 13, 64
    queries = group_detr * qg
    sizes = np.clip(rng.poisson(8, images), 1, 60)
    logits = rng.normal(-2.0, 1.5, (1, images, queries, 2)).astype(np.float32)
    boxes = (1.0 / (1.0 + np.exp(-rng.normal(0.0, 1.0, (1, images, queries, 4))))).astype(np.float32)
    targets = [{"labels": torch.as_tensor(rng.integers(0, 2, t), device=DEV),
                "boxes": torch.as_tensor(np.concatenate([rng.uniform(0.1, 0.9, (t, 2)), rng.uniform(0.02, 0.5, (t, 2))],
                                                        axis=1).astype(np.float32), device=DEV)} for t in sizes]
    outputs = [{"pred_logits": torch.as_tensor(logits[0], device=DEV), "pred_boxes": torch.as_tensor(boxes[0], device=DEV)}]
    res, cost = matcher.match_layers(outputs, targets, group_detr, return_cost=True)
    torch.cuda.synchronize()
    cost = cost[0, :, : int(sizes.sum())].cpu().numpy()
    expect = solve_blocks(cost, [int(t) for t in sizes], group_detr, solver=oracle_lsa)
    for b, (q, t) in enumerate(res[0]):
        assert np.array_equal(q.cpu().numpy(), expect[b][0]), b
        assert np.array_equal(t.cpu().numpy(), expect[b][1]), b
