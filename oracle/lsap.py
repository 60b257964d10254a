"""TEST INFRASTRUCTURE ONLY: ctypes binding of the C restatement of SciPy's
``rectangular_lsap`` (``oracle/lsap.c``).  See that file for the semantics."""

from __future__ import annotations

import ctypes

import numpy as np

from oracle.build import build

_lib = None

OK, INFEASIBLE, INVALID = 0, 1, 2


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(build())
        lib.oracle_lsap.restype = ctypes.c_int
        lib.oracle_lsap.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                    ctypes.c_void_p, ctypes.c_void_p]
        lib.oracle_lsap_batch.restype = None
        lib.oracle_lsap_batch.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib = lib
    return _lib


def linear_sum_assignment(cost: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Same contract as ``scipy.optimize.linear_sum_assignment`` for a 2-D float32 matrix."""
    c = np.ascontiguousarray(cost, dtype=np.float32)
    if c.ndim != 2:
        raise ValueError("expected a matrix")
    nr, nc = c.shape
    n = min(nr, nc)
    rows = np.zeros(n, dtype=np.int64)
    cols = np.zeros(n, dtype=np.int64)
    rc = _load().oracle_lsap(nr, nc, c.ctypes.data, nc, rows.ctypes.data, cols.ctypes.data)
    if rc == INVALID:
        raise ValueError("matrix contains invalid numeric entries")
    if rc == INFEASIBLE:
        raise ValueError("cost matrix is infeasible")
    return rows, cols


def solve_batch(cost: np.ndarray, ld: int, desc: np.ndarray, total_pairs: int):
    """Batched solve over problem descriptors ``desc[p] = (cost_offset, out_offset, nq, nt, query_base)``.

    ``cost`` is the flat float32 matrix the offsets address.  Returns
    ``(query_out, target_out, status)``.
    """
    c = np.ascontiguousarray(cost.reshape(-1), dtype=np.float32)
    d = np.ascontiguousarray(desc, dtype=np.int64).reshape(-1, 5)
    q = np.full(total_pairs, -1, dtype=np.int64)
    t = np.full(total_pairs, -1, dtype=np.int64)
    st = np.zeros(d.shape[0], dtype=np.int32)
    _load().oracle_lsap_batch(c.ctypes.data, ld, d.ctypes.data, d.shape[0], q.ctypes.data, t.ctypes.data,
                              st.ctypes.data)
    return q, t, st
