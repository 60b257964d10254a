"""The C ABI library loads on a host without a GPU and exports what include/rfm.h declares."""

import ctypes
import os
import re

import numpy as np
import pytest

from rfdetr_training_throughput_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions() -> set[str]:
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(rfm_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = header_functions()
    assert declared, "no declarations found"
    assert declared == set(_lib.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name


def test_version_and_error_strings():
    assert "sm_100a" in _lib.version()
    assert _lib.error_string(0) == "ok"
    assert _lib.error_string(1) == "invalid argument"
    assert _lib.error_string(2) == "outside the supported envelope"
    assert _lib.error_string(99) == "unknown error"


def test_problem_struct_layout_matches_header():
    text = open(os.path.join(ROOT, "include", "rfm.h")).read()
    body = re.search(r"typedef struct rfm_problem \{(.*?)\} rfm_problem;", text, re.S).group(1)
    fields = re.findall(r"(int\d+_t)\s+(\w+);", body)
    assert [f[1] for f in fields] == list(_lib.PROBLEM_DTYPE.names)
    sizes = {"int64_t": 8, "int32_t": 4}
    assert [sizes[f[0]] for f in fields] == [_lib.PROBLEM_DTYPE[n].itemsize for n in _lib.PROBLEM_DTYPE.names]
    assert ctypes.sizeof(_lib.LsapPlan) == 56


def test_invalid_arguments_are_rejected_before_any_cuda_call():
    lib = _lib.load()
    # negative sizes, ld < sum_targets
    qm, tm = _lib.LAYOUT_QUERY_MAJOR, _lib.LAYOUT_TARGET_MAJOR
    assert lib.rfm_cost(None, None, None, None, None, 0, 1, 1, 1, 0, 0, qm, 1.0, 1.0, 1.0, 0.25, None, None) == 1
    assert lib.rfm_cost(None, None, None, None, None, 1, 1, 1, 1, 8, 4, qm, 1.0, 1.0, 1.0, 0.25, None, None) == 1
    # target-major rows must hold every query and keep 16-byte alignment
    assert lib.rfm_cost(None, None, None, None, None, 1, 1, 8, 1, 3, 6, tm, 1.0, 1.0, 1.0, 0.25, None, None) == 1
    assert lib.rfm_cost(None, None, None, None, None, 1, 1, 8, 1, 3, 10, tm, 1.0, 1.0, 1.0, 0.25, None, None) == 1
    assert lib.rfm_cost(None, None, None, None, None, 1, 1, 8, 1, 3, 8, 7, 1.0, 1.0, 1.0, 0.25, None, None) == 1
    # zero-sized output: nothing to do
    assert lib.rfm_cost(None, None, None, None, None, 1, 1, 1, 1, 0, 0, qm, 1.0, 1.0, 1.0, 0.25, None, None) == 0
    plan = _lib.LsapPlan(cols_per_lane=10, max_rows=1, num_problems=3, num_ctas=1, cta_smem_bytes=4096,
                         tile_cap_floats=0, flags=0, reserved=0, stride_q=1, stride_t=8, workspace_bytes=0)
    assert lib.rfm_lsap(None, None, None, ctypes.byref(plan), None, None, None, None, None) == 1
    assert lib.rfm_lsap(None, None, None, None, None, None, None, None, None) == 1
    plan.cols_per_lane = 7
    assert lib.rfm_lsap(None, None, None, ctypes.byref(plan), None, None, None, None, None) == 1
    # rfm_match: the plan must address the target-major matrix the call writes (stride_q 1,
    # stride_t ld), and a plan with problems needs targets
    match_args = lambda p, ld, s: (None, None, None, None, None, 1, 1, 8, 1, s, ld, 1.0, 1.0, 1.0, 0.25, None,
                                   None, None, p, None, None, None, None, None)
    assert lib.rfm_match(*match_args(None, 8, 3)) == 1
    assert lib.rfm_match(*match_args(ctypes.byref(plan), 12, 3)) == 1  # plan made for ld 8
    assert lib.rfm_match(*match_args(ctypes.byref(plan), 8, 0)) == 1   # problems but no targets
    persistent = _lib.LsapPlan(cols_per_lane=10, max_rows=1, num_problems=3, num_ctas=0, cta_smem_bytes=4096,
                               tile_cap_floats=0, flags=1, reserved=0, stride_q=1, stride_t=8, workspace_bytes=256)
    assert lib.rfm_match(*match_args(ctypes.byref(persistent), 8, 3)) == 1  # persistent plan, no workspace
    assert lib.rfm_lsap_dense(None, -1, 3, 3, None, None, None, None) == 1
    assert lib.rfm_lsap_dense(None, 4, 2000, 3, None, None, None, None) == 2
    assert lib.rfm_lsap_dense_workspace_bytes(-1, 3, 3) < 0


def test_push_structs_match_header(tmp_path):
    """ctypes mirrors of rfm_pair_push / rfm_peer_sync_args against the header, compiled with gcc."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("no gcc")
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "rfm.h"\nint main(void) {\n'
                   '  printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(rfm_pair_push), offsetof(rfm_pair_push, epoch),\n'
                   '         offsetof(rfm_pair_push, target_out), sizeof(rfm_peer_sync_args),\n'
                   '         offsetof(rfm_peer_sync_args, flags), offsetof(rfm_peer_sync_args, error));\n'
                   '  return 0;\n}\n')
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert got == [ctypes.sizeof(_lib.PairPush), _lib.PairPush.epoch.offset, _lib.PairPush.target_out.offset,
                   ctypes.sizeof(_lib.PeerSyncArgs), _lib.PeerSyncArgs.flags.offset, _lib.PeerSyncArgs.error.offset]


def test_push_and_peer_arguments_are_rejected_before_any_cuda_call():
    lib = _lib.load()
    fake = 1 << 40  # never dereferenced: every call below fails its checks first
    for bad in (dict(count=9), dict(count=-1), dict(count=1, reserved=1), dict(count=1, epoch=None),
                dict(count=2, epoch=fake, parity_stride=-1)):
        push = _lib.PairPush(**{"count": 1, "epoch": fake, **bad})
        for d in range(_lib.MAX_PUSH):
            push.query_out[d] = fake
            push.target_out[d] = fake
        assert lib.rfm_pair_push_store(ctypes.byref(push), fake) == 1, bad
    push = _lib.PairPush(count=2, epoch=fake)
    push.query_out[0] = push.target_out[0] = push.query_out[1] = fake  # target_out[1] missing
    assert lib.rfm_pair_push_store(ctypes.byref(push), fake) == 1
    push.target_out[1] = fake
    assert lib.rfm_pair_push_store(ctypes.byref(push), fake + 8) == 1  # destination not 16-byte aligned
    assert lib.rfm_pair_push_store(None, fake) == 1 and lib.rfm_pair_push_store(ctypes.byref(push), None) == 1
    plan = _lib.LsapPlan(cols_per_lane=10, max_rows=1, num_problems=3, num_ctas=1, cta_smem_bytes=4096,
                         tile_cap_floats=0, flags=0, reserved=0, stride_q=1, stride_t=8, workspace_bytes=0)
    assert lib.rfm_lsap_push(fake, fake, fake, ctypes.byref(plan), fake, fake, None, None, fake + 4, None) == 1
    assert lib.rfm_peer_sync(None, None) == 1
    for bad in (dict(world=0), dict(world=9), dict(rank=2), dict(rank=-1), dict(spin_limit=0), dict(flags=None),
                dict(error=None), dict(epoch=None)):
        args = _lib.PeerSyncArgs(**{"world": 2, "rank": 0, "spin_limit": 10, "flags": fake, "epoch": fake,
                                    "error": fake, **bad})
        args.arrive[0] = args.arrive[1] = fake
        assert lib.rfm_peer_sync(ctypes.byref(args), None) == 1, bad
    args = _lib.PeerSyncArgs(world=2, rank=0, spin_limit=10, flags=fake, epoch=fake, error=fake)
    args.arrive[0] = fake  # arrive[1] missing
    assert lib.rfm_peer_sync(ctypes.byref(args), None) == 1
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    assert lib.rfm_peer_alloc(0, ctypes.byref(ptr), handle) == 1
    assert lib.rfm_peer_alloc(256, None, handle) == 1
    assert lib.rfm_peer_open(None, ctypes.byref(ptr)) == 1
    assert lib.rfm_peer_close(None) == 1 and lib.rfm_peer_free(None) == 1


def _cta_cover(ctas, n):
    """The CTA table covers problems 0..n-1 once, in order, with 1-4 warps each."""
    nxt = 0
    for first, count, slot, zero in ctas.tolist():
        assert first == nxt and 1 <= count <= 4 and slot % 16 == 0 and zero == 0
        nxt += count
    assert nxt == n


def test_planner_modes_and_workspace():
    sizes = [250, 300, 60, 8, 0]
    pr = np.zeros(len(sizes), dtype=_lib.PROBLEM_DTYPE)
    pr["num_queries"] = 300
    pr["num_targets"] = sizes
    # query-major source (strides q: 1000, t: 1): tall tiles above the on-chip cap (64 KB) are
    # transposed into scratch, the square one is read in place, the small one is staged
    plan, ctas = _lib.make_plan(pr, 1000, 1)
    assert plan.cols_per_lane == 10 and plan.max_rows == 300 and plan.num_problems == 5
    assert pr["scratch_offset"].tolist() == [0, -1, 300 * 250, -1, -1]
    assert plan.workspace_bytes == (300 * 250 + 300 * 60) * 4
    assert plan.stride_q == 1000 and plan.stride_t == 1 and plan.tile_cap_floats == 16384
    _cta_cover(ctas, 5)
    assert plan.cta_smem_bytes == max(c * s for _, c, s, _ in ctas.tolist())
    assert plan.flags == 0
    # target-major source (q: 1, t: 4000): tall problems' solver rows are contiguous and are read
    # in place; only the square one (solver rows = queries, strided here) needs scratch
    pr2 = pr.copy()
    plan2, _ = _lib.make_plan(pr2, 1, 4000)
    assert pr2["scratch_offset"].tolist() == [-1, 0, -1, -1, -1] and plan2.workspace_bytes == 300 * 300 * 4
    # a zero cap stages nothing; rows are then read straight from L2/HBM, four warps per CTA
    pr3 = pr.copy()
    plan3, ctas3 = _lib.make_plan(pr3, 1, 4000, tile_cap=0)
    assert plan3.workspace_bytes == 300 * 300 * 4 and ctas3.tolist()[0][1] == 4
    # small staged tiles share CTAs (query-major source)
    small = np.zeros(9, dtype=_lib.PROBLEM_DTYPE)
    small["num_queries"] = 300
    small["num_targets"] = [12, 12, 10, 9, 8, 8, 8, 8, 3]
    plan4, ctas4 = _lib.make_plan(small, 1000, 1)
    _cta_cover(ctas4, 9)
    assert plan4.workspace_bytes == 0 and plan4.num_ctas < 9
    # every problem row-contiguous: persistent warps, a queue word in the workspace, no CTA table
    plan5, ctas5 = _lib.make_plan(small.copy(), 1, 4000)
    assert plan5.flags == _lib.PLAN_PERSISTENT and plan5.num_ctas == 0 and len(ctas5) == 0
    assert plan5.workspace_bytes == 256 and plan5.cta_smem_bytes % 4 == 0
    wide = np.zeros(1, dtype=_lib.PROBLEM_DTYPE)
    wide["num_queries"] = 64
    wide["num_targets"] = 1025
    with pytest.raises(_lib.RfmError):
        _lib.make_plan(wide, 1025, 1)
    bad = np.zeros(1, dtype=_lib.PROBLEM_DTYPE)
    bad["num_queries"] = -1
    with pytest.raises(_lib.RfmError):
        _lib.make_plan(bad, 1, 1)


def test_dense_workspace_bytes():
    lib = _lib.load()
    assert lib.rfm_lsap_dense_workspace_bytes(520, 300, 12) == 256  # the claim counter of batches of 512+
    assert lib.rfm_lsap_dense_workspace_bytes(511, 300, 12) == 0
    assert lib.rfm_lsap_dense_workspace_bytes(40, 300, 250) == 40 * 300 * 250 * 4
    assert lib.rfm_lsap_dense_workspace_bytes(40, 300, 300) == 0
