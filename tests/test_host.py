"""Host-side planning and interface behaviour of the matcher (no GPU)."""

import numpy as np
import pytest
import torch

from rfdetr_training_throughput_b200 import matcher, workloads


def test_build_problems_layout_brute_force():
    sizes = [3, 0, 5, 1]
    layers, queries, g, ld = 2, 12, 3, 12
    pr, per_image, total, offsets = matcher.build_problems(sizes, layers, queries, g, ld)
    qg = queries // g
    expect = []
    cursor = 0
    for l in range(layers):
        for b, t in enumerate(sizes):
            n = min(qg, t)
            for gi in range(g):
                if t:
                    expect.append((l * queries * ld + gi * qg * ld + offsets[b], cursor + gi * n, qg, t, gi * qg))
            cursor += g * n
    got = [(int(p["cost_offset"]), int(p["out_offset"]), int(p["num_queries"]), int(p["num_targets"]),
            int(p["query_base"])) for p in pr]
    assert got == expect
    assert total == cursor == sum(per_image)
    assert per_image == [g * min(qg, t) for _ in range(layers) for t in sizes]


def test_build_problems_target_major_offsets():
    sizes = [3, 0, 5]
    layers, queries, g, ld = 2, 12, 3, 12
    pr, _, _, offsets = matcher.build_problems(sizes, layers, queries, g, ld, layout=1)
    qg = queries // g
    s = sum(sizes)
    expect = [l * s * ld + offsets[b] * ld + gi * qg for l in range(layers) for b, t in enumerate(sizes)
              for gi in range(g) if t]
    assert [int(x) for x in pr["cost_offset"]] == expect
    assert matcher.strides(0, 7) == (7, 1) and matcher.strides(1, 7) == (1, 7)


def test_build_problems_rejects_bad_groups():
    with pytest.raises(ValueError):
        matcher.build_problems([3], 1, 10, 3, 4)


def test_wide_problem_pairs_capped_by_group_width():
    pr, per_image, total, _ = matcher.build_problems([7], 1, 10, 2, 8)
    assert per_image == [2 * 5] and total == 10


def test_cpu_tensors_are_rejected_no_fallback():
    wl = workloads.make("cpu1")
    m = matcher.HungarianMatcher(**wl.weights)
    with pytest.raises(ValueError, match="CUDA"):
        m(wl.outputs_list()[0], wl.targets)
    with pytest.raises(ValueError, match="CUDA"):
        matcher.batch_linear_assignment(torch.zeros(2, 3, 3))


def test_segmentation_outputs_are_out_of_scope():
    m = matcher.HungarianMatcher()
    with pytest.raises(NotImplementedError):
        m({"pred_logits": None, "pred_boxes": None, "pred_masks": None}, [])


def test_workloads_match_their_descriptions():
    step = workloads.make("step")
    assert (step.layers, step.images, step.group_detr, step.queries, step.classes) == (5, 8, 13, 3900, 2)
    assert step.num_problems == 520
    assert all(1 <= s <= 60 for s in step.sizes)
    ties = workloads.make("ties")
    assert ties.sizes[:3] == [0, 1, 300]
    assert set(np.unique(ties.pred_logits.numpy()).tolist()) <= {-2.0, 0.0, 2.0}
    assert torch.equal(torch.round(ties.pred_boxes * 16) / 16, ties.pred_boxes)
    crowd = workloads.make("crowd")
    assert all(100 <= s <= 300 for s in crowd.sizes) and crowd.classes == 91
    sweep = workloads.make("sweep", images=64)
    assert sweep.num_problems == 64 * 13
    # reseeding per shard gives different data of the same shape
    a, b = workloads.make("sweep", images=4, shard=0), workloads.make("sweep", images=4, shard=1)
    assert a.pred_logits.shape == b.pred_logits.shape and not torch.equal(a.pred_logits, b.pred_logits)
