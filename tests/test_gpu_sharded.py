"""sharded_match on one GPU through a one-rank NCCL group: the device path writes its pairs into
the all-gather's send buffer and must return exactly match_packed's pairs (integers: exact
equality), on the same step twice so the reused buffers are exercised."""

import os
import socket

import pytest
import torch
import torch.distributed as dist

from rfdetr_training_throughput_b200 import matcher, sharded, workloads

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture
def one_rank_group():
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        yield
    finally:
        dist.destroy_process_group()


def test_sharded_match_equals_match_packed_on_one_rank(one_rank_group):
    dev = torch.device("cuda", 0)
    wl = workloads.make("sweep", images=40)
    logits, boxes = wl.pred_logits.to(dev), wl.pred_boxes.to(dev)
    packed = matcher.PackedTargets.from_list(wl.targets_on(dev), dev)
    expect = matcher.match_packed(logits, boxes, packed, wl.group_detr, weights=wl.weights)
    for _ in range(2):
        pairs, per = sharded.sharded_match(logits, boxes, packed.labels, packed.boxes, wl.sizes, wl.group_detr,
                                           weights=wl.weights)
        torch.cuda.synchronize()
        assert torch.equal(pairs, expect.pairs)
        assert per == expect.per_image


def test_match_packed_out_argument_is_checked():
    dev = torch.device("cuda", 0)
    wl = workloads.make("step", layers=1, images=2)
    packed = matcher.PackedTargets.from_list(wl.targets_on(dev), dev)
    res = matcher.match_packed(wl.pred_logits.to(dev), wl.pred_boxes.to(dev), packed, wl.group_detr,
                               weights=wl.weights)
    buf = torch.full((3, 2, res.pairs.shape[1] + 5), -9, dtype=torch.int64, device=dev)
    view = buf[1, :, 2:2 + res.pairs.shape[1]]  # rows contiguous, row stride larger than the row
    matcher.match_packed(wl.pred_logits.to(dev), wl.pred_boxes.to(dev), packed, wl.group_detr,
                         weights=wl.weights, out=view)
    torch.cuda.synchronize()
    assert torch.equal(view, res.pairs)
    assert bool((buf[0] == -9).all()) and bool((buf[2] == -9).all()) and bool((buf[1, :, :2] == -9).all())
    with pytest.raises(ValueError):
        matcher.match_packed(wl.pred_logits.to(dev), wl.pred_boxes.to(dev), packed, wl.group_detr,
                             weights=wl.weights, out=torch.empty((2, 3), dtype=torch.int64, device=dev))


def test_sharded_matcher_graph_equals_match_packed(one_rank_group):
    dev = torch.device("cuda", 0)
    wl = workloads.make("sweep", images=40)
    logits, boxes = wl.pred_logits.to(dev), wl.pred_boxes.to(dev)
    packed = matcher.PackedTargets.from_list(wl.targets_on(dev), dev)
    expect = matcher.match_packed(logits, boxes, packed, wl.group_detr, weights=wl.weights)
    sm = sharded.ShardedMatcher(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, weights=wl.weights,
                                device=dev)
    for _ in range(2):
        pairs = sm(logits, boxes, packed.labels, packed.boxes)
        torch.cuda.synchronize()
        assert torch.equal(pairs, expect.pairs)
    assert sm.per_image == expect.per_image


def _perturbed(wl, dev):
    """The workload's predictions with the queries of every image rotated by 7: same shapes and
    targets, other pairs."""
    return wl.pred_logits.roll(7, dims=2).to(dev), wl.pred_boxes.roll(7, dims=2).to(dev)


def test_pushed_exchange_equals_match_packed_on_one_rank(one_rank_group):
    """ShardedMatcher(exchange="push") on one rank: the solver's pushes and the barrier kernel, the
    two parity buffers alternating, each result still intact after the next step."""
    dev = torch.device("cuda", 0)
    wl = workloads.make("sweep", images=40)
    packed = matcher.PackedTargets.from_list(wl.targets_on(dev), dev)
    inputs = [(wl.pred_logits.to(dev), wl.pred_boxes.to(dev)), _perturbed(wl, dev)]
    expect = [matcher.match_packed(lg, bx, packed, wl.group_detr, weights=wl.weights).pairs for lg, bx in inputs]
    assert not torch.equal(expect[0], expect[1])
    sm = sharded.ShardedMatcher(wl.sizes, wl.layers, wl.queries, wl.classes, wl.group_detr, weights=wl.weights,
                                device=dev, exchange="push")
    try:
        prev = None
        for step in range(4):
            lg, bx = inputs[step % 2]
            got = sm(lg, bx, packed.labels, packed.boxes, padded=True)
            torch.cuda.synchronize()
            assert torch.equal(got.flat(), expect[step % 2])
            if prev is not None:  # the previous step's buffer is not touched by this one
                assert torch.equal(prev.flat(), expect[(step - 1) % 2])
            prev = got
        sm.check()
        assert sm.exchange.error() == 0
    finally:
        sm.close()


def test_peer_barrier_gives_up_and_reports():
    """A barrier whose other rank never arrives (a flag nothing sets) returns after its poll limit
    with the error word set; the step counter still advances and the context stays usable."""
    from rfdetr_training_throughput_b200 import _lib
    import ctypes

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    words = torch.zeros(64, dtype=torch.int32, device=dev)  # flags 0..7, counter 8, error 9
    base = words.data_ptr()
    args = _lib.PeerSyncArgs(world=2, rank=0, spin_limit=2000, flags=base, epoch=base + 32, error=base + 36)
    args.arrive[0] = base           # this rank's own flag
    args.arrive[1] = base + 4 * 40  # "rank 1's" copy of it: a word no one reads
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.check("rfm_peer_sync", lib.rfm_peer_sync(ctypes.byref(args), stream))
    torch.cuda.synchronize()
    w = words.cpu().tolist()
    assert w[0] == 1 and w[1] == 0 and w[8] == 1 and w[9] == 1 and w[40] == 1
    assert float(torch.ones(4, device=dev).sum()) == 4.0
