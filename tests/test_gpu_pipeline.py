"""PrefetchingMatcher: batches uploaded on a copy stream while the previous batch is matched give
exactly the pairs match_packed gives for each batch (index pairs: exact equality), and the first
batch's pairs are checked directly against SciPy on the device-computed cost matrix."""

import numpy as np
import pytest
import torch
from test_gpu_graph import scipy_pairs

from rfdetr_training_throughput_b200 import matcher, workloads
from rfdetr_training_throughput_b200.pipeline import PrefetchingMatcher

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def test_prefetched_batches_match_like_match_packed():
    batches = []
    for seed_images in (64, 64, 64):
        wl = workloads.make("sweep", images=seed_images, shard=len(batches))  # three different batches
        batches.append((wl.pred_logits.pin_memory(), wl.pred_boxes.pin_memory(),
                        torch.cat([t["labels"] for t in wl.targets]).pin_memory(),
                        torch.cat([t["boxes"] for t in wl.targets]).pin_memory(), tuple(wl.sizes)))
    group_detr, weights = wl.group_detr, wl.weights
    expect = []
    for lg, bx, lb, tb, sz in batches:
        r = matcher.match_packed(lg.to(DEV), bx.to(DEV), matcher.PackedTargets(lb.to(DEV), tb.to(DEV), sz),
                                 group_detr, weights=weights)
        expect.append(r.pairs.clone())
    torch.cuda.synchronize()
    pm = PrefetchingMatcher(group_detr, weights=weights, device=DEV)
    outs = []
    order = [0, 1, 2, 1, 0, 2, 2]
    nxt = pm.prefetch(*batches[order[0]])
    for k, b in enumerate(order):
        cur = nxt
        if k + 1 < len(order):
            nxt = pm.prefetch(*batches[order[k + 1]])
        outs.append(pm.match(cur).pairs.clone())
    torch.cuda.synchronize()
    for b, got in zip(order, outs):
        assert torch.equal(got, expect[b])
    wl0 = workloads.make("sweep", images=64, shard=0)
    lg, bx, lb, tb, sz = batches[0]
    packed = matcher.PackedTargets(lb.to(DEV), tb.to(DEV), sz)
    assert np.array_equal(outs[0].cpu().numpy(), scipy_pairs(wl0, lg.to(DEV), bx.to(DEV), packed))
