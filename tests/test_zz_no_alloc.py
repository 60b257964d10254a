"""rfm_lsap_dense_noalloc: the solver for callers that cannot allocate device memory.

Such callers (an FFI host without a device allocator, or a training step that must
not add a cudaMalloc/cudaFree beside the framework's caching allocator) call this
entry point instead of rfm_lsap_dense; it uses a scratch array built into the
library.  The test calls both entry points through the C ABI on batches that need
scratch, twice in a row with different data, and requires identical matchings
(index outputs: the tolerance is exact equality, as for every solver test); the
no-allocation results are also checked against SciPy itself, problem by problem.
"""

import ctypes

import numpy as np
import pytest
import torch
from scipy.optimize import linear_sum_assignment

from rfdetr_training_throughput_b200 import _lib

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_workspace(lib, cost):
    p, w, t = cost.shape
    ws_bytes = int(lib.rfm_lsap_dense_workspace_bytes(p, w, t))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda") if ws_bytes else None
    out = torch.empty((p, w), dtype=torch.int64, device="cuda")
    assert lib.rfm_lsap_dense(_ptr(cost), p, w, t, _ptr(out), None, _ptr(ws), _stream()) == 0
    return out, ws_bytes


def _without_workspace(lib, cost):
    p, w, t = cost.shape
    out = torch.full((p, w), -7, dtype=torch.int64, device="cuda")
    status = torch.full((p,), -1, dtype=torch.int32, device="cuda")
    assert lib.rfm_lsap_dense_noalloc(_ptr(cost), p, w, t, _ptr(out), _ptr(status), _stream()) == 0
    return out, status


def test_noalloc_matches_the_workspace_entry_point_on_two_calls():
    lib = _lib.load()
    # tall tiles above the on-chip budget: both entry points stage them in scratch
    shapes = [(12, 300, 200), (9, 300, 150)]
    for call, shape in enumerate(shapes):
        rng = np.random.default_rng(100 + call)
        cost = torch.as_tensor((rng.integers(0, 6, shape) / 6).astype(np.float32), device="cuda")
        ref, ws_bytes = _with_workspace(lib, cost)
        assert 0 < ws_bytes <= _lib.NOALLOC_SCRATCH_BYTES
        got, status = _without_workspace(lib, cost)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {call}"
        assert bool((status == 0).all())
        host = cost.cpu().numpy()
        for p in range(shape[0]):
            rows, cols = linear_sum_assignment(host[p])
            expect = np.full(shape[1], -1, dtype=np.int64)
            expect[rows] = cols
            assert np.array_equal(got[p].cpu().numpy(), expect), f"call {call}, problem {p}"


def test_noalloc_rejects_batches_beyond_its_scratch():
    lib = _lib.load()
    p, w, t = 64, 1000, 900  # needs 64 * 1000 * 900 * 4 bytes of scratch, far above the built-in array
    assert lib.rfm_lsap_dense_workspace_bytes(p, w, t) > _lib.NOALLOC_SCRATCH_BYTES
    dummy = torch.zeros(4, dtype=torch.float32, device="cuda")
    out = torch.zeros(4, dtype=torch.int64, device="cuda")
    assert lib.rfm_lsap_dense_noalloc(_ptr(dummy), p, w, t, _ptr(out), None, _stream()) == _lib.RFM_ERR_UNSUPPORTED
    assert lib.rfm_lsap_dense_noalloc(_ptr(dummy), -1, w, t, _ptr(out), None, _stream()) == _lib.RFM_ERR_INVALID_ARGUMENT
