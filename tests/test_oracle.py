"""The CPU oracle pinned against the reference's own operators and SciPy (no GPU)."""

import numpy as np
import pytest
import torch
from scipy.optimize import linear_sum_assignment as scipy_lsa

from golden_io import lsap_case, matcher_case, names
from oracle import cost as ocost
from oracle import cpu_path
from oracle.lsap import linear_sum_assignment as oracle_lsa
from oracle.matcher import solve_blocks


def _same(a, b):
    return np.array_equal(np.asarray(a[0]), np.asarray(b[0])) and np.array_equal(np.asarray(a[1]), np.asarray(b[1]))


@pytest.mark.parametrize("seed", range(4))
def test_oracle_lsap_matches_scipy_random_and_tied(seed):
    rng = np.random.default_rng(seed)
    for trial in range(400):
        nr, nc = int(rng.integers(1, 45)), int(rng.integers(1, 45))
        kind = trial % 5
        if kind == 0:
            m = rng.standard_normal((nr, nc))
        elif kind == 1:
            m = rng.integers(0, 4, (nr, nc)) / 4
        elif kind == 2:
            m = np.full((nr, nc), 2.5)
        elif kind == 3:
            m = rng.integers(-3, 4, (nr, nc)).astype(np.float64)
        else:
            m = np.round(rng.standard_normal((nr, nc)) * 8) / 8
        m = m.astype(np.float32)
        assert _same(oracle_lsa(m), scipy_lsa(m)), (seed, trial, m.shape)


def test_oracle_lsap_matcher_shapes():
    rng = np.random.default_rng(11)
    for nt in (1, 2, 12, 37, 60, 150, 299, 300):
        m = rng.standard_normal((300, nt)).astype(np.float32)
        assert _same(oracle_lsa(m), scipy_lsa(m))
    for nt in (301, 400):  # wide: one target per query, untransposed
        m = rng.standard_normal((300, nt)).astype(np.float32)
        assert _same(oracle_lsa(m), scipy_lsa(m))


@pytest.mark.parametrize("name", names("lsap"))
def test_oracle_lsap_golden(name):
    for m, res, r, c in lsap_case(name):
        if res == "ok":
            assert _same(oracle_lsa(m), (r, c))
        else:
            with pytest.raises(ValueError, match="infeasible" if res == "infeasible" else "invalid"):
                oracle_lsa(m)


@pytest.mark.parametrize("name", names("matcher"))
def test_oracle_cost_golden(name):
    logits, boxes, labels, tboxes, _g, w, cost, _pairs = matcher_case(name)
    mine = ocost.compact_cost(logits, boxes, labels, tboxes, **w)
    assert mine.shape == cost.shape
    np.testing.assert_allclose(mine, cost, rtol=0, atol=2e-6 * max(1.0, float(np.abs(cost).max(initial=1.0))))
    assert np.isfinite(mine).all()


@pytest.mark.parametrize("name", names("matcher"))
def test_oracle_pairs_golden(name):
    _l, _b, labels, _t, group_detr, _w, cost, pairs = matcher_case(name)
    sizes = [len(x) for x in labels]
    for layer, (q, t) in enumerate(pairs):
        got = solve_blocks(cost[layer], sizes, group_detr)
        assert np.array_equal(np.concatenate([g[0] for g in got]), q)
        assert np.array_equal(np.concatenate([g[1] for g in got]), t)


def test_scipy_order_is_query_ascending():
    """The output-order convention: pairs come back sorted by query within a group."""
    _l, _b, labels, _t, group_detr, _w, cost, _p = matcher_case("step_small")
    sizes = [len(x) for x in labels]
    for q, _t in solve_blocks(cost[0], sizes, group_detr):
        per_group = q.reshape(group_detr, -1)
        assert (np.diff(per_group, axis=1) > 0).all()


def test_cpu_path_agrees_with_numpy_oracle():
    logits, boxes, labels, tboxes, group_detr, w, cost, pairs = matcher_case("step_small")
    targets = [{"labels": torch.from_numpy(l), "boxes": torch.from_numpy(b)} for l, b in zip(labels, tboxes)]
    torch_cost = cpu_path.compact_cost(torch.from_numpy(logits), torch.from_numpy(boxes), targets, w).numpy()
    np.testing.assert_array_equal(torch_cost, cost)
    m = cpu_path.CpuMatcher(threads=4)
    try:
        got = m.match(torch.from_numpy(logits), torch.from_numpy(boxes), targets, group_detr, w)
    finally:
        m.close()
    for layer, (q, t) in enumerate(pairs):
        assert np.array_equal(np.concatenate([g[0] for g in got[layer]]), q)
        assert np.array_equal(np.concatenate([g[1] for g in got[layer]]), t)


def test_oracle_batch_descriptors():
    from oracle.lsap import solve_batch

    rng = np.random.default_rng(3)
    m = rng.standard_normal((40, 17)).astype(np.float32)
    desc = np.array([[0, 0, 20, 5, 100], [5, 5, 20, 12, 0], [20 * 17 + 3, 17, 20, 14, 7]], dtype=np.int64)
    q, t, st = solve_batch(m, 17, desc, 17 + 14)
    assert (st == 0).all()
    r, c = scipy_lsa(m[:20, :5])
    assert np.array_equal(q[:5], r + 100) and np.array_equal(t[:5], c)
    r, c = scipy_lsa(m[20:, 3:17])
    assert np.array_equal(q[17:31], r + 7) and np.array_equal(t[17:31], c)
