"""Image-sharded matcher sweep over several GPUs with an all-gather of the index pairs.

A large batch of images is split into contiguous, balanced image ranges, one per
rank (each image's ``layers x groups`` problems are independent, so there is no
exchange during matching).  Every rank matches its range with ``match_packed`` and
the packed int64 pairs of all ranks are then gathered with one
``all_gather_into_tensor`` (NCCL over NVLink on GPUs, gloo in the CPU tests), so
every rank ends with the whole batch's per-image ``(query_idx, target_idx)``.
Sizes are known on every host, so the gather needs no count exchange: each
rank's chunk is padded to the largest rank's pair count.  With ``padded=True``
the result is the gathered buffer itself (``GatheredPairs``: per-image views at
host-known offsets, no copy); otherwise the padding is squeezed out with one
concatenation into a flat ``[2, total]`` tensor.

``ShardedMatcher(exchange="push")`` replaces the all-gather on GPUs: the solver
itself stores every pair into every rank's gathered buffer (``PeerExchange``:
CUDA IPC mappings of the other ranks' buffers, plain stores over NVLink), and a
one-warp barrier kernel ends the step, so the exchange overlaps the solve and
the whole step is one graph replay.
"""

from __future__ import annotations

import ctypes
from functools import lru_cache
from typing import Callable, Sequence

import numpy as np
import torch
import torch.distributed as dist


def shard_bounds(num_images: int, world: int) -> list[tuple[int, int]]:
    """Contiguous image ranges ``[start, end)`` per rank; sizes differ by at most one."""
    if world < 1:
        raise ValueError("world size must be >= 1")
    base, extra = divmod(num_images, world)
    bounds, start = [], 0
    for r in range(world):
        end = start + base + (1 if r < extra else 0)
        bounds.append((start, end))
        start = end
    return bounds


def pairs_per_image(sizes: Sequence[int], layers: int, queries: int, group_detr: int) -> np.ndarray:
    """Host-known pair count of every (layer, image): ``group_detr * min(Q/G, T_b)``."""
    qg = queries // group_detr
    per = group_detr * np.minimum(np.asarray(sizes, dtype=np.int64), qg)
    return np.tile(per, layers)


class _Shard:
    """Host-only split of a batch for one rank: image bounds, pair counts per rank and per
    (layer, image), this rank's sizes tuple (one object, so the matcher's plan cache hits by
    identity) and its slice of the packed targets."""

    def __init__(self, sizes: tuple[int, ...], layers: int, queries: int, group_detr: int, world: int, rank: int):
        self.bounds = shard_bounds(len(sizes), world)
        offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        self.counts, self.per, self.per_rank = [], [], []
        for a, b in self.bounds:
            pi = pairs_per_image(sizes[a:b], layers, queries, group_detr)
            self.counts.append(int(pi.sum()))
            self.per_rank.append(tuple(int(x) for x in pi))
            self.per.extend(self.per_rank[-1])
        self.layers = layers
        self.lo, self.hi = self.bounds[rank]
        self.t_lo, self.t_hi = int(offsets[self.lo]), int(offsets[self.hi])
        self.local_sizes = tuple(sizes[self.lo:self.hi])
        self.width = max(self.counts) if self.counts else 0
        self.buffers: dict = {}

    def gather_buffers(self, device, world: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Send ``[1, 2, width]`` and receive ``[world, 2, width]`` int64 buffers, reused across steps."""
        key = (str(device), world)
        if key not in self.buffers:
            self.buffers[key] = (torch.empty((1, 2, self.width), dtype=torch.int64, device=device),
                                 torch.empty((world, 2, self.width), dtype=torch.int64, device=device))
        return self.buffers[key]


@lru_cache(maxsize=64)
def _shard_cached(sizes: tuple[int, ...], layers: int, queries: int, group_detr: int, world: int,
                  rank: int) -> _Shard:
    return _Shard(sizes, layers, queries, group_detr, world, rank)


_LAST_SHARD: list = [None]  # (sizes object, rest of the key, shard) of the last call


def _shard(sizes: tuple[int, ...], layers: int, queries: int, group_detr: int, world: int, rank: int) -> _Shard:
    """The cached split; a loop that passes the same sizes object every step skips hashing it."""
    rest = (layers, queries, group_detr, world, rank)
    last = _LAST_SHARD[0]
    if last is not None and last[0] is sizes and last[1] == rest:
        return last[2]
    sh = _shard_cached(sizes, *rest)
    _LAST_SHARD[0] = (sizes, rest, sh)
    return sh


def _unpad(recv: torch.Tensor, counts: Sequence[int]) -> torch.Tensor:
    return torch.cat([recv[r, :, : int(counts[r])] for r in range(recv.shape[0])], dim=1)


class GatheredPairs:
    """Every rank's pairs as the all-gather left them, with no copy.

    ``recv`` is ``[world, 2, width]`` int64: rank ``r``'s pairs are ``recv[r, :, :counts[r]]``, in
    its (layer, image) order (layer-major, images in order), the rest of the row is padding that
    is never read.  All offsets are host-known, so views need no synchronisation: ``layer(l)``
    gives rf-detr's per-image ``(query_idx, target_idx)`` list for the whole batch, ``rank_pairs(r)``
    one rank's ``[2, counts[r]]`` block, and ``flat()`` the ``[2, total]`` concatenation (one copy).
    The buffer is reused by the next gather of the same matcher.
    """

    def __init__(self, recv: torch.Tensor, counts: Sequence[int], per_rank: Sequence[tuple[int, ...]], layers: int):
        self.recv = recv
        self.counts = list(counts)
        self.per_rank = list(per_rank)
        self.layers = layers
        self._views: list | None = None

    def rank_pairs(self, r: int) -> torch.Tensor:
        return self.recv[r, :, : self.counts[r]]

    def flat(self) -> torch.Tensor:
        return _unpad(self.recv, self.counts)

    def _split(self):
        if self._views is None:
            self._views = [(torch.split(self.recv[r, 0, : self.counts[r]], self.per_rank[r]),
                            torch.split(self.recv[r, 1, : self.counts[r]], self.per_rank[r]))
                           for r in range(len(self.counts))]
        return self._views

    def layer(self, l: int) -> list[tuple[torch.Tensor, torch.Tensor]]:
        out = []
        for r, (qs, ts) in enumerate(self._split()):
            n = len(self.per_rank[r]) // self.layers  # images of rank r
            out.extend(zip(qs[l * n:(l + 1) * n], ts[l * n:(l + 1) * n]))
        return out


def exchange_layout(world: int, width: int) -> dict[str, int]:
    """Byte layout of one rank's ``PeerExchange`` buffer: two ``[world, 2, width]`` int64 gathered
    buffers (step parity 0 and 1; rank ``r``'s pairs in row ``r``), then a 256-byte block of
    ``MAX_PUSH`` uint32 flags (flag ``j`` raised by rank ``j``), the step counter, the error word
    and (at +64) this rank's ``rfm_pair_push`` list."""
    from . import _lib

    if not 1 <= world <= _lib.MAX_PUSH:
        raise ValueError(f"a pushed exchange takes 1..{_lib.MAX_PUSH} ranks, not {world}")
    if width < 0:
        raise ValueError("width must be >= 0")
    parity_elems = world * 2 * width
    flags = (2 * parity_elems * 8 + 255) // 256 * 256
    return {"parity_elems": parity_elems, "flags": flags, "epoch": flags + 4 * _lib.MAX_PUSH,
            "error": flags + 4 * _lib.MAX_PUSH + 4, "push": flags + 64, "bytes": flags + 256}


class _DeviceWords:
    """``__cuda_array_interface__`` of ``n`` words at a raw device address, for ``torch.as_tensor``."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 2,
                                         "strides": None}


class PeerExchange:
    """The gathered buffers of a pushed exchange, mapped on every rank of ``group``.

    Each rank allocates one buffer (``exchange_layout``) with ``rfm_peer_alloc``, the ranks swap
    the 64-byte IPC handles with ``all_gather_object``, and each rank maps the others' buffers
    (``rfm_peer_open``).  ``push`` is the ``rfm_pair_push`` list that sends this rank's pairs into
    row ``rank`` of every rank's buffer (itself included); ``sync`` enqueues the step's barrier
    (``rfm_peer_sync``), which also advances the step counter that picks the buffer parity.  The
    result of the last step stays readable until the step after the next one.  Waits are bounded
    (``spin_limit`` polls, about a second by default); ``check`` reports a wait that gave up.
    Call ``close`` on every rank (collectively) before the process group goes.
    """

    DEFAULT_SPIN_LIMIT = 1 << 22  # polls of at most 256 ns each: about a second

    def __init__(self, width: int, group=None, device: torch.device | None = None,
                 spin_limit: int = DEFAULT_SPIN_LIMIT):
        from . import _lib

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.width = int(width)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        lay = exchange_layout(self.world, self.width)
        self.layout = lay
        self.recv, self._control, self._opened, self.base, self._closed = [], None, [], 0, False
        lib = _lib.load()
        ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        with torch.cuda.device(self.device):
            rc = lib.rfm_peer_alloc(lay["bytes"], ctypes.byref(ptr), handle)
        self.base = int(ptr.value) if rc == _lib.RFM_OK else 0
        handles: list = [None] * self.world
        with torch.cuda.device(self.device):  # NCCL's object gather stages on the current device
            dist.all_gather_object(handles, handle.raw if self.base else None, group=group)
        peers = []
        failure = None if self.base else f"rfm_peer_alloc: {_lib.error_string(rc)}"
        with torch.cuda.device(self.device):
            for j, h in enumerate(handles):
                if failure is not None:
                    break
                if h is None:
                    failure = f"rank {j} has no buffer"
                elif j == self.rank:
                    peers.append(self.base)
                else:
                    p = ctypes.c_void_p()
                    rc = lib.rfm_peer_open(h, ctypes.byref(p))
                    if rc != _lib.RFM_OK:
                        failure = f"rfm_peer_open of rank {j}: {_lib.error_string(rc)}"
                        break
                    self._opened.append(int(p.value))
                    peers.append(int(p.value))
        # every rank learns whether every rank mapped every buffer, so all of them go on or none does
        ok = torch.tensor([0 if failure else 1], dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if not bool(ok.item()):
            self._release(lib)
            raise RuntimeError(f"pushed exchange unavailable on rank {self.rank}: {failure or 'a peer failed'}")
        self.peers = peers
        words = torch.as_tensor(_DeviceWords(self.base, 2 * lay["parity_elems"], "<i8"), device=self.device)
        self.recv = [words[k * lay["parity_elems"]:(k + 1) * lay["parity_elems"]].view(self.world, 2, self.width)
                     for k in (0, 1)]
        self._control = torch.as_tensor(_DeviceWords(self.base + lay["flags"], 64, "<i4"), device=self.device)
        row = self.rank * 2 * self.width * 8
        plist = _lib.PairPush(count=self.world, reserved=0, parity_stride=lay["parity_elems"],
                              epoch=self.base + lay["epoch"])
        self.sync_args = _lib.PeerSyncArgs(world=self.world, rank=self.rank, spin_limit=int(spin_limit),
                                           flags=self.base + lay["flags"], epoch=self.base + lay["epoch"],
                                           error=self.base + lay["error"])
        for j, p in enumerate(peers):
            plist.query_out[j] = p + row
            plist.target_out[j] = p + row + self.width * 8
            self.sync_args.arrive[j] = p + lay["flags"] + 4 * self.rank
        with torch.cuda.device(self.device):
            _lib.check("rfm_pair_push_store", lib.rfm_pair_push_store(ctypes.byref(plist),
                                                                      ctypes.c_void_p(self.base + lay["push"])))
        self.push_list = plist
        self.push = self.base + lay["push"]  # device address of the stored list, for the solver
        self.steps = 0  # barriers executed (not counting captured ones)
        with torch.cuda.device(self.device):
            dist.barrier(group=group)  # every buffer mapped before any rank pushes

    def sync(self) -> None:
        """Enqueue the step's barrier on the current stream (captured into a graph when capturing)."""
        from . import _lib
        from .matcher import _stream_handle

        _lib.check("rfm_peer_sync", _lib.load().rfm_peer_sync(ctypes.byref(self.sync_args),
                                                              _stream_handle(self.device)))
        if not torch.cuda.is_current_stream_capturing():
            self.steps += 1

    def parity(self) -> int:
        """Buffer parity of the last step run (its barrier counted in ``steps``)."""
        if self.steps == 0:
            raise RuntimeError("no step has run on this exchange")
        return (self.steps - 1) & 1

    def result(self, counts: Sequence[int], per_rank: Sequence[tuple[int, ...]], layers: int) -> "GatheredPairs":
        return GatheredPairs(self.recv[self.parity()], counts, per_rank, layers)

    def error(self) -> int:
        """The error word (synchronises): 1 when a barrier wait gave up."""
        return int(self._control[(self.layout["error"] - self.layout["flags"]) // 4].item())

    def check(self) -> None:
        if self.error():
            raise RuntimeError("pushed exchange: a rank did not reach the barrier in time")

    def _release(self, lib) -> None:
        """Collective teardown: every rank unmaps, then (nobody mapping them any more) frees."""
        from . import _lib

        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            dist.barrier(group=self.group)
            for p in self._opened:
                _lib.check("rfm_peer_close", lib.rfm_peer_close(ctypes.c_void_p(p)))
            self._opened = []
            dist.barrier(group=self.group)
        self.recv, self._control = [], None
        if self.base:
            with torch.cuda.device(self.device):
                _lib.check("rfm_peer_free", lib.rfm_peer_free(ctypes.c_void_p(self.base)))
            self.base = 0

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's, after every rank is done with them."""
        from . import _lib

        if self._closed:
            return
        self._closed = True
        self._release(_lib.load())


def gather_pairs(local_pairs: torch.Tensor, counts: Sequence[int], group=None) -> torch.Tensor:
    """All-gather ``[2, counts[rank]]`` int64 chunks; returns ``[2, sum(counts)]`` in rank order.
    Chunks are padded to the largest count; the padding is never read."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    width = max(int(c) for c in counts) if counts else 0
    send = torch.empty((1, 2, width), dtype=local_pairs.dtype, device=local_pairs.device)
    n = int(counts[rank])
    if n:
        send[0, :, :n] = local_pairs[:, :n]
    recv = torch.empty((world, 2, width), dtype=local_pairs.dtype, device=local_pairs.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    return _unpad(recv, counts)


def sharded_match(pred_logits: torch.Tensor, pred_boxes: torch.Tensor, labels: torch.Tensor,
                  boxes: torch.Tensor, sizes: Sequence[int], group_detr: int, *,
                  weights: dict | None = None, group=None, padded: bool = False,
                  local_solver: Callable | None = None) -> tuple[torch.Tensor | GatheredPairs, list[int]]:
    """Match a batch split by image across the ranks of ``group``.

    ``pred_logits`` ``[L, B, Q, C]`` / ``pred_boxes`` ``[L, B, Q, 4]`` and the packed
    ``labels``/``boxes`` may hold the whole batch or only this rank's image range
    (detected from the leading image dimension).  Returns the gathered ``[2, total]``
    pairs (per rank, layer-major, images in order; with ``padded`` the
    ``GatheredPairs`` buffer itself) and the per-(layer, image) pair counts in the
    same order.  ``local_solver(logits, boxes, labels, boxes, sizes,
    group_detr) -> [2, n]`` replaces the device step (used by CPU tests).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if type(sizes) is not tuple:
        sizes = tuple(int(s) for s in sizes)
    layers, nimg_in, queries, _ = pred_logits.shape
    sh = _shard(sizes, layers, queries, group_detr, world, rank)
    if nimg_in == len(sizes):  # whole batch given: slice this rank's images and targets
        pred_logits = pred_logits[:, sh.lo:sh.hi]
        pred_boxes = pred_boxes[:, sh.lo:sh.hi]
        labels = labels[sh.t_lo:sh.t_hi]
        boxes = boxes[sh.t_lo:sh.t_hi]
    elif nimg_in != sh.hi - sh.lo:
        raise ValueError(f"rank {rank} holds {nimg_in} images, its shard has {sh.hi - sh.lo}")
    n = sh.counts[rank]
    if local_solver is None:
        from .matcher import PackedTargets, match_packed

        # the local pairs land directly in the collective's send buffer
        send, recv = sh.gather_buffers(pred_logits.device, world)
        targets = PackedTargets.from_checked_sizes(labels, boxes, sh.local_sizes, sh.t_hi - sh.t_lo)
        match_packed(pred_logits, pred_boxes, targets, group_detr, weights=weights, out=send[0, :, :n])
        dist.all_gather_into_tensor(recv, send, group=group)
        if padded:
            return GatheredPairs(recv, sh.counts, sh.per_rank, layers), sh.per
        return _unpad(recv, sh.counts), sh.per
    local = local_solver(pred_logits, pred_boxes, labels, boxes, list(sh.local_sizes), group_detr)
    flat = gather_pairs(local, sh.counts, group)
    if padded:
        width = max(sh.counts) if sh.counts else 0
        recv = flat.new_zeros((world, 2, width))
        start = 0
        for r, c in enumerate(sh.counts):
            recv[r, :, :c] = flat[:, start:start + c]
            start += c
        return GatheredPairs(recv, sh.counts, sh.per_rank, layers), sh.per
    return flat, sh.per


class ShardedMatcher:
    """``sharded_match`` for a batch shape that repeats.  Inputs are this rank's image range
    (``pred_logits`` ``[L, hi - lo, Q, C]`` etc.); construct it on every rank of ``group`` with the
    same arguments.

    ``exchange="nccl"``: this rank's step is a captured ``MatchGraph`` writing straight into the
    all-gather's send buffer, so a call is one graph replay and one ``all_gather_into_tensor``
    (plus one concatenation unless the caller takes the padded ``GatheredPairs``).

    ``exchange="push"`` (CUDA devices, up to 8 ranks): the captured step's solver stores every
    pair into every rank's gathered buffer itself and the step ends with ``PeerExchange``'s
    barrier kernel, so a call is one graph replay and no collective.  Results alternate between
    two buffers; the one a call returns stays valid until the call after the next.  Run steps through
    ``__call__`` or ``replay`` (not ``graph.replay``), which keep count of the buffer parity.  Call
    ``close`` on every rank when done."""

    def __init__(self, sizes: Sequence[int], layers: int, queries: int, num_classes: int, group_detr: int, *,
                 weights: dict | None = None, group=None, device: torch.device | None = None,
                 exchange: str = "nccl", spin_limit: int = PeerExchange.DEFAULT_SPIN_LIMIT):
        from .graph import MatchGraph

        if exchange not in ("nccl", "push"):
            raise ValueError(f"exchange must be 'nccl' or 'push', not {exchange!r}")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.mode = exchange
        sizes = tuple(int(s) for s in sizes)
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.shard = _shard(sizes, layers, queries, group_detr, self.world, self.rank)
        n = self.shard.counts[self.rank]
        self.exchange = None
        if exchange == "push":
            self.exchange = PeerExchange(self.shard.width, group=group, device=device, spin_limit=spin_limit)
            self.local = torch.empty((2, n), dtype=torch.int64, device=device)  # the solver's own copy
            self.graph = MatchGraph(self.shard.local_sizes, layers, queries, num_classes, group_detr,
                                    weights=weights, device=device, out=self.local, push=self.exchange.push,
                                    post=self.exchange.sync)
        else:
            self.send, self.recv = self.shard.gather_buffers(device, self.world)
            self.graph = MatchGraph(self.shard.local_sizes, layers, queries, num_classes, group_detr,
                                    weights=weights, device=device, out=self.send[0, :, :n])
        self.bounds = (self.shard.lo, self.shard.hi)
        self.per_image = self.shard.per

    def replay(self) -> None:
        """Run the captured step on the graph's input buffers (push: the exchange included)."""
        self.graph.replay()
        if self.exchange is not None:
            self.exchange.steps += 1

    def gather(self, padded: bool = False) -> torch.Tensor | GatheredPairs:
        """The whole batch's pairs of the last replay: ``[2, total]`` in rank order, or with
        ``padded`` the gathered buffer itself (no concatenation).  ``nccl`` runs the all-gather
        here; ``push`` has exchanged them already."""
        if self.exchange is not None:
            res = self.exchange.result(self.shard.counts, self.shard.per_rank, self.shard.layers)
            return res if padded else res.flat()
        dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        if padded:
            return GatheredPairs(self.recv, self.shard.counts, self.shard.per_rank, self.shard.layers)
        return _unpad(self.recv, self.shard.counts)

    def __call__(self, pred_logits: torch.Tensor, pred_boxes: torch.Tensor, labels: torch.Tensor,
                 tgt_boxes: torch.Tensor, padded: bool = False) -> torch.Tensor | GatheredPairs:
        self.graph(pred_logits, pred_boxes, labels, tgt_boxes)
        if self.exchange is not None:
            self.exchange.steps += 1
        return self.gather(padded)

    def check(self) -> None:
        """Raise if a pushed exchange's barrier gave up waiting (synchronises)."""
        if self.exchange is not None:
            self.exchange.check()

    def close(self) -> None:
        """Release the pushed exchange's mappings (collective over ``group``); the graph goes too."""
        self.graph = None
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None
