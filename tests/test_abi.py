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
    assert ctypes.sizeof(_lib.LsapPlan) == 24


def test_invalid_arguments_are_rejected_before_any_cuda_call():
    lib = _lib.load()
    # negative sizes, ld < sum_targets
    assert lib.rfm_cost(None, None, None, None, None, 0, 1, 1, 1, 0, 0, 1.0, 1.0, 1.0, 0.25, None, None) == 1
    assert lib.rfm_cost(None, None, None, None, None, 1, 1, 1, 1, 8, 4, 1.0, 1.0, 1.0, 0.25, None, None) == 1
    # zero-sized output: nothing to do
    assert lib.rfm_cost(None, None, None, None, None, 1, 1, 1, 1, 0, 0, 1.0, 1.0, 1.0, 0.25, None, None) == 0
    plan = _lib.LsapPlan(cols_per_lane=10, tile_floats=0, max_rows=1, num_problems=3, workspace_bytes=0)
    assert lib.rfm_lsap(None, 8, None, ctypes.byref(plan), None, None, None, None, None) == 1
    assert lib.rfm_lsap(None, 8, None, None, None, None, None, None, None) == 1
    assert lib.rfm_lsap_dense(None, -1, 3, 3, None, None, None, None) == 1
    assert lib.rfm_lsap_dense(None, 4, 2000, 3, None, None, None, None) == 2
    assert lib.rfm_lsap_dense_workspace_bytes(-1, 3, 3) < 0


def test_planner_modes_and_workspace():
    pr = np.zeros(5, dtype=_lib.PROBLEM_DTYPE)
    pr["num_queries"] = 300
    pr["num_targets"] = [8, 250, 300, 0, 60]
    plan = _lib.make_plan(pr)
    assert plan.cols_per_lane == 10
    assert plan.max_rows == 300
    assert plan.num_problems == 5
    # tall tiles above the on-chip budget (64 KB) are staged in scratch; square/wide ones are
    # read in place; 300 x (60|1) floats = 73 KB is above the budget as well
    assert pr["scratch_offset"].tolist() == [-1, 0, -1, -1, 300 * 250]
    assert plan.workspace_bytes == (300 * 250 + 300 * 60) * 4
    assert plan.tile_floats == 16384
    pr2 = np.zeros(2, dtype=_lib.PROBLEM_DTYPE)
    pr2["num_queries"] = 300
    pr2["num_targets"] = [8, 12]
    plan2 = _lib.make_plan(pr2)
    assert plan2.workspace_bytes == 0 and plan2.tile_floats == 300 * 13
    wide = np.zeros(1, dtype=_lib.PROBLEM_DTYPE)
    wide["num_queries"] = 64
    wide["num_targets"] = 1025
    with pytest.raises(_lib.RfmError):
        _lib.make_plan(wide)
    bad = np.zeros(1, dtype=_lib.PROBLEM_DTYPE)
    bad["num_queries"] = -1
    with pytest.raises(_lib.RfmError):
        _lib.make_plan(bad)


def test_dense_workspace_bytes():
    lib = _lib.load()
    assert lib.rfm_lsap_dense_workspace_bytes(520, 300, 12) == 0
    assert lib.rfm_lsap_dense_workspace_bytes(40, 300, 250) == 40 * 300 * 250 * 4
    assert lib.rfm_lsap_dense_workspace_bytes(40, 300, 300) == 0
