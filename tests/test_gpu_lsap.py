"""The device solver against SciPy itself and the C oracle: identical indices, ties included."""

import numpy as np
import pytest
import torch
from scipy.optimize import linear_sum_assignment as scipy_lsa

from golden_io import lsap_case, names
from oracle.lsap import linear_sum_assignment as oracle_lsa
from rfdetr_training_throughput_b200 import _lib, matcher

pytestmark = pytest.mark.gpu


def _dense_expected(cost: np.ndarray) -> np.ndarray:
    """[P, W, T] -> [P, W] matching as torch_linear_assignment builds it from SciPy (patches.py:216-228)."""
    out = np.full(cost.shape[:2], -1, dtype=np.int64)
    for p in range(cost.shape[0]):
        if cost.shape[2] == 0:
            continue
        r, c = scipy_lsa(cost[p])
        out[p, r] = c
    return out


def _solve_dense(cost: np.ndarray, **kw) -> np.ndarray:
    got = matcher.batch_linear_assignment(torch.as_tensor(cost, device="cuda"), **kw)
    return got.cpu().numpy()


@pytest.mark.parametrize("shape", [(520, 300, 1), (520, 300, 12), (520, 300, 37), (104, 300, 60),
                                   (8, 300, 300), (1, 16, 16), (3, 64, 0), (6, 300, 333), (4, 64, 16),
                                   (3, 600, 40), (5, 40, 1000),
                                   # long problems: one four-warp CTA each at 1, 5 and 3 per SM (the
                                   # last square, rows read in place), then too many for one wave
                                   (140, 300, 90), (700, 300, 70), (300, 200, 200), (1300, 300, 66),
                                   (700, 100, 64),
                                   # more than one wave: two-warp CTAs claiming problems from the counter
                                   (2000, 300, 60), (1600, 300, 12)])
def test_dense_random(shape):
    rng = np.random.default_rng(sum(shape))
    cost = (rng.random(shape, dtype=np.float32) * 10 - 5).astype(np.float32)
    assert np.array_equal(_solve_dense(cost), _dense_expected(cost))


@pytest.mark.parametrize("q", [4, 16])
@pytest.mark.parametrize("shape", [(64, 300, 8), (32, 300, 40), (16, 300, 150), (8, 300, 260), (8, 300, 300),
                                   (6, 40, 40), (6, 120, 200)])
def test_dense_quantised_ties(shape, q):
    rng = np.random.default_rng(shape[2] * q)
    cost = (rng.integers(0, q, shape) / q).astype(np.float32)
    assert np.array_equal(_solve_dense(cost), _dense_expected(cost))


def test_dense_constant_matrix():
    cost = np.full((4, 300, 8), 1.5, dtype=np.float32)
    assert np.array_equal(_solve_dense(cost), _dense_expected(cost))


@pytest.mark.parametrize("name", names("lsap"))
def test_golden_lsap(name):
    for m, res, r, c in lsap_case(name):
        batch = m[None]
        if res == "ok":
            got = _solve_dense(batch)[0]
            expect = np.full(m.shape[0], -1, dtype=np.int64)
            expect[r] = c
            assert np.array_equal(got, expect)
        else:
            msg = "infeasible" if res == "infeasible" else "invalid"
            with pytest.raises(ValueError, match=msg):
                _solve_dense(batch, check_status=True)
            assert (_solve_dense(batch) == -1).all()


def test_near_ties_need_float64():
    """Costs 1e-6 apart only resolve as SciPy does with float64 path costs."""
    rng = np.random.default_rng(5)
    base = rng.integers(0, 4, (64, 300, 10)).astype(np.float32)
    bump = rng.random(base.shape) < 0.05
    base[bump] += np.float32(2.0 ** -20)
    assert np.array_equal(_solve_dense(base), _dense_expected(base))


def test_assign_padded_on_compact_matrix():
    """The _assign_padded contract on a compact [G*300, sum T] matrix, against the C oracle."""
    rng = np.random.default_rng(9)
    sizes = [5, 0, 17, 1, 300, 9]
    g = 3
    cost = rng.integers(0, 8, (g * 300, sum(sizes))).astype(np.float32) / 8
    res = matcher.assign_padded([torch.as_tensor(cost, device="cuda")], sizes, 300, g)[0]
    col = 0
    for b, t in enumerate(sizes):
        q_exp, t_exp = [], []
        for gi in range(g if t else 0):
            r, c = oracle_lsa(cost[gi * 300:(gi + 1) * 300, col:col + t])
            q_exp.append(r + gi * 300)
            t_exp.append(c)
        col += t
        qs, ts = res[b]
        assert np.array_equal(qs.cpu().numpy(), np.concatenate(q_exp) if q_exp else np.zeros(0))
        assert np.array_equal(ts.cpu().numpy(), np.concatenate(t_exp) if t_exp else np.zeros(0))


def test_repeat_calls_are_deterministic():
    rng = np.random.default_rng(2)
    cost = torch.as_tensor((rng.integers(0, 3, (200, 300, 24)) / 3).astype(np.float32), device="cuda")
    a = matcher.batch_linear_assignment(cost)
    b = matcher.batch_linear_assignment(cost)
    assert torch.equal(a, b)


def _target_major_matrix(sizes, width, groups, kind, rng):
    """A target-major compact matrix [sum T, groups * width] of the given value kind."""
    shape = (sum(sizes), groups * width)
    if kind == "uniform":
        m = rng.random(shape, dtype=np.float32) * 10 - 5
    elif kind.startswith("ties"):
        q = int(kind[4:])
        m = (rng.integers(0, q, shape) / q).astype(np.float32)
    else:  # "inf": a third of the entries +inf, and one target of image 1 unmatchable in group 0
        m = rng.random(shape, dtype=np.float32)
        m[rng.random(shape) < 0.3] = np.inf
        m[sizes[0], :width] = np.inf
    return np.ascontiguousarray(m.astype(np.float32))


@pytest.mark.parametrize("sizes,width,groups,kind", [
    ((297, 250, 180, 120, 64), 300, 2, "uniform"),  # 297 x 300 floats exceed an SM's shared memory
    ((260, 200, 100, 70), 300, 3, "ties4"),
    ((99, 80, 64, 70), 100, 4, "ties2"),  # at most 128 columns
    ((220, 150, 90), 300, 2, "inf"),
    (tuple(range(64, 124, 3)), 300, 13, "ties8"),  # 260 problems: two per SM
    (tuple(range(64, 114)), 300, 13, "uniform"),  # 650 problems: five per SM, two warps each
    (tuple(range(64, 100)), 100, 20, "ties4"),  # 720 problems of at most 128 columns, two warps each
    # more problems than fit one wave: two-warp CTAs claiming problems from a counter (row-contiguous)
    (tuple(64 + i % 40 for i in range(120)), 300, 13, "ties4"),  # 1,560 long problems
    (tuple(8 + i % 30 for i in range(150)), 300, 13, "uniform"),  # 1,950 short problems
    ((300, 180, 90), 300, 2, "ties4"),  # square problems: solver rows run across the target-major rows
])
@pytest.mark.parametrize("layout", ["target_major", "query_major"])
def test_long_problems_one_cta_each(sizes, width, groups, kind, layout):
    """Small batches of long problems (64+ solver rows): the launch that gives every problem a CTA,
    stages its rows in shared memory (row-contiguous blocks directly, the others as a transposed copy,
    partly in scratch when it does not fit) and runs its searches on all four warps.  Indices and
    statuses are compared with SciPy problem by problem."""
    rng = np.random.default_rng(sum(sizes) + width + groups)
    m = _target_major_matrix(sizes, width, groups, kind, rng)
    dev = torch.device("cuda")
    if layout == "target_major":
        cost = torch.as_tensor(m, device=dev)
        code = _lib.LAYOUT_TARGET_MAJOR
    else:
        cost = torch.as_tensor(np.ascontiguousarray(m.T), device=dev)
        code = _lib.LAYOUT_QUERY_MAJOR
    plan = matcher.plan_step(sizes, 1, groups * width, groups, cost.shape[1], dev, code)
    pairs = torch.empty((2, plan.total_pairs), dtype=torch.int64, device=dev)
    status = torch.empty(plan.problems.shape[0], dtype=torch.int32, device=dev)
    matcher.launch_lsap(cost, plan, pairs, status)
    per_image = matcher.MatchResult(pairs, plan.per_image, 1, len(sizes)).layer(0)
    status_of = {int(plan.order[i]): int(s) for i, s in enumerate(status.cpu().numpy())}
    off = np.concatenate([[0], np.cumsum(sizes)])
    for b, t in enumerate(sizes):
        qs, ts = (x.cpu().numpy() for x in per_image[b])
        n = min(width, t)
        for g in range(groups):
            block = m[off[b]:off[b + 1], g * width:(g + 1) * width].T  # [queries, targets]
            chunk = slice(g * n, (g + 1) * n)
            try:
                r, c = scipy_lsa(block)
            except ValueError:
                assert status_of[b * groups + g] == _lib.STATUS_INFEASIBLE
                assert (qs[chunk] == -1).all() and (ts[chunk] == -1).all()
                continue
            assert status_of[b * groups + g] == _lib.STATUS_OK
            assert np.array_equal(qs[chunk], r + g * width)
            assert np.array_equal(ts[chunk], c)
