"""The reference's own GPU solver (lsap_kernel / batch_lap_cuda, kernels_lap.py:69-305, built from its
source by oracle/build_ref.py into oracle/_ref) against this library's solver on the batches the
benchmark times them on: both must assign every task and reach the same total cost (the reference
solves in float32 with fast math and does not reproduce SciPy's tie-breaking, so indices may differ;
the objective agrees within 1e-4 relative, its own verify bound at kernels_lap.py:422-431).  Skipped
when no build of the reference solver is present."""

import pytest
import torch

from oracle import build_ref
from rfdetr_training_throughput_b200 import matcher

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    mod = build_ref.load()
    if mod is None:
        pytest.skip("no build of the reference solver in oracle/_ref")
    return mod


@pytest.mark.parametrize("tasks", [12, 60, 219])
def test_reference_solver_reaches_the_same_objective(ref, tasks):
    g = torch.Generator().manual_seed(5000 + tasks)
    cost = torch.rand((64, 300, tasks), generator=g).cuda()
    ours = matcher.batch_linear_assignment(cost)
    theirs = ref.batch_lap_cuda(cost)
    torch.cuda.synchronize()
    for m in (ours, theirs):
        assigned = m >= 0
        assert bool((assigned.sum(dim=1) == tasks).all())
        for p in range(cost.shape[0]):
            assert torch.equal(torch.sort(m[p][assigned[p]]).values, torch.arange(tasks, device=m.device))
    obj = lambda m: torch.where(m >= 0, cost.gather(2, m.clamp(min=0).unsqueeze(-1)).squeeze(-1), 0).sum(1)  # noqa: E731
    a, b = obj(ours).double(), obj(theirs).double()
    assert bool(((a - b).abs() <= 1e-4 * a.abs().clamp(min=1)).all())
