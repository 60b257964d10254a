"""ctypes binding of ``librfm.so``, the sm_100a C ABI declared in ``include/rfm.h``.

There is no CPU fallback: if the library is missing or fails to load, every
entry point raises.  The library is built in-tree by
``python -m rfdetr_training_throughput_b200.build``.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librfm.so")

RFM_OK = 0
RFM_ERR_INVALID_ARGUMENT = 1
RFM_ERR_UNSUPPORTED = 2
RFM_ERR_LAUNCH = 3
RFM_ERR_NO_DEVICE = 4

STATUS_OK = 0
STATUS_INFEASIBLE = 1
STATUS_INVALID = 2
STATUS_NO_SINK = 3

MAX_COLS = 1024

#: Every symbol include/rfm.h declares.
EXPORTS = (
    "rfm_version",
    "rfm_error_string",
    "rfm_cost",
    "rfm_lsap_make_plan",
    "rfm_lsap",
    "rfm_match",
    "rfm_lsap_dense_workspace_bytes",
    "rfm_lsap_dense",
    "rfm_lsap_dense_noalloc",
    "rfm_box_loss_forward",
    "rfm_box_loss_backward",
    "rfm_label_loss_parts",
    "rfm_label_loss_forward",
    "rfm_label_loss_backward",
    "rfm_msda_forward",
    "rfm_msda_backward",
    "rfm_pair_push_store",
    "rfm_lsap_push",
    "rfm_match_push",
    "rfm_peer_alloc",
    "rfm_peer_open",
    "rfm_peer_close",
    "rfm_peer_free",
    "rfm_peer_sync",
)

#: RFM_MAX_PUSH: destinations of one pushed solve, ranks of one pushed exchange.
MAX_PUSH = 8
#: Bytes of a CUDA IPC handle (rfm_peer_alloc / rfm_peer_open).
IPC_HANDLE_BYTES = 64

#: Size of the built-in scratch of rfm_lsap_dense_noalloc (RFM_NOALLOC_SCRATCH_BYTES).
NOALLOC_SCRATCH_BYTES = 16 << 20

#: numpy mirror of ``struct rfm_problem`` (40 bytes).
PROBLEM_DTYPE = np.dtype(
    [
        ("cost_offset", "<i8"),
        ("out_offset", "<i8"),
        ("scratch_offset", "<i8"),
        ("num_queries", "<i4"),
        ("num_targets", "<i4"),
        ("query_base", "<i4"),
        ("reserved", "<i4"),
    ]
)
assert PROBLEM_DTYPE.itemsize == 40


PLAN_PERSISTENT = 1

LABEL_LOSS_FOCAL = 0
LABEL_LOSS_IA_BCE = 1
LABEL_LOSS_PART_ELEMS = 8192

LAYOUT_QUERY_MAJOR = 0
LAYOUT_TARGET_MAJOR = 1


class LsapPlan(ctypes.Structure):
    """Mirror of ``struct rfm_lsap_plan``."""

    _fields_ = [
        ("cols_per_lane", ctypes.c_int32),
        ("max_rows", ctypes.c_int32),
        ("num_problems", ctypes.c_int32),
        ("num_ctas", ctypes.c_int32),
        ("cta_smem_bytes", ctypes.c_int32),
        ("tile_cap_floats", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("stride_q", ctypes.c_int64),
        ("stride_t", ctypes.c_int64),
        ("workspace_bytes", ctypes.c_int64),
    ]


class PairPush(ctypes.Structure):
    """Mirror of ``struct rfm_pair_push``."""

    _fields_ = [
        ("count", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("parity_stride", ctypes.c_int64),
        ("epoch", ctypes.c_void_p),
        ("query_out", ctypes.c_void_p * MAX_PUSH),
        ("target_out", ctypes.c_void_p * MAX_PUSH),
    ]


class PeerSyncArgs(ctypes.Structure):
    """Mirror of ``struct rfm_peer_sync_args``."""

    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("spin_limit", ctypes.c_int64),
        ("arrive", ctypes.c_void_p * MAX_PUSH),
        ("flags", ctypes.c_void_p),
        ("epoch", ctypes.c_void_p),
        ("error", ctypes.c_void_p),
    ]


assert ctypes.sizeof(PairPush) == 152 and ctypes.sizeof(PeerSyncArgs) == 104


class RfmError(RuntimeError):
    """A non-zero return code from the C ABI."""

    def __init__(self, func: str, code: int):
        self.code = code
        super().__init__(f"{func} failed: {error_string(code)} (code {code})")


_lib: ctypes.CDLL | None = None

_p = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


def load() -> ctypes.CDLL:
    """Load ``librfm.so`` once; raise if it is missing or incomplete."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is not built; run `python -m rfdetr_training_throughput_b200.build` "
            "(there is no CPU fallback)"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name in EXPORTS:
        if not hasattr(lib, name):
            raise RuntimeError(f"{LIB_PATH} does not export {name}")
    lib.rfm_version.restype = ctypes.c_char_p
    lib.rfm_version.argtypes = []
    lib.rfm_error_string.restype = ctypes.c_char_p
    lib.rfm_error_string.argtypes = [_i32]
    lib.rfm_cost.restype = _i32
    lib.rfm_cost.argtypes = [_p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i64, _i32,
                             _f32, _f32, _f32, _f32, _p, _p]
    lib.rfm_lsap_make_plan.restype = _i32
    lib.rfm_lsap_make_plan.argtypes = [_p, _i32, _i64, _i64, _i64, _p, ctypes.POINTER(LsapPlan)]
    lib.rfm_lsap.restype = _i32
    lib.rfm_lsap.argtypes = [_p, _p, _p, ctypes.POINTER(LsapPlan), _p, _p, _p, _p, _p]
    lib.rfm_match.restype = _i32
    lib.rfm_match.argtypes = [_p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _f32, _f32, _f32, _p,
                              _p, _p, ctypes.POINTER(LsapPlan), _p, _p, _p, _p, _p]
    lib.rfm_lsap_dense_workspace_bytes.restype = _i64
    lib.rfm_lsap_dense_workspace_bytes.argtypes = [_i32, _i32, _i32]
    lib.rfm_lsap_dense.restype = _i32
    lib.rfm_lsap_dense.argtypes = [_p, _i32, _i32, _i32, _p, _p, _p, _p]
    lib.rfm_box_loss_forward.restype = _i32
    lib.rfm_box_loss_forward.argtypes = [_p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _p, _p, _p]
    lib.rfm_box_loss_backward.restype = _i32
    lib.rfm_box_loss_backward.argtypes = [_p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _p, _p, _p, _p]
    lib.rfm_label_loss_parts.restype = _i64
    lib.rfm_label_loss_parts.argtypes = [_i32, _i32, _i32, _i32]
    lib.rfm_label_loss_forward.restype = _i32
    lib.rfm_label_loss_forward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _f32,
                                           _p, _p, _p]
    lib.rfm_label_loss_backward.restype = _i32
    lib.rfm_label_loss_backward.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _f32,
                                            _p, _p, _p]
    lib.rfm_msda_forward.restype = _i32
    lib.rfm_msda_forward.argtypes = [_p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p, _p]
    lib.rfm_msda_backward.restype = _i32
    lib.rfm_msda_backward.argtypes = [_p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _p, _p, _p,
                                      _p]
    lib.rfm_lsap_dense_noalloc.restype = _i32
    lib.rfm_lsap_dense_noalloc.argtypes = [_p, _i32, _i32, _i32, _p, _p, _p]
    lib.rfm_pair_push_store.restype = _i32
    lib.rfm_pair_push_store.argtypes = [ctypes.POINTER(PairPush), _p]
    lib.rfm_lsap_push.restype = _i32
    lib.rfm_lsap_push.argtypes = [_p, _p, _p, ctypes.POINTER(LsapPlan), _p, _p, _p, _p, _p, _p]
    lib.rfm_match_push.restype = _i32
    lib.rfm_match_push.argtypes = [_p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _f32, _f32, _f32,
                                   _p, _p, _p, ctypes.POINTER(LsapPlan), _p, _p, _p, _p, _p, _p]
    lib.rfm_peer_alloc.restype = _i32
    lib.rfm_peer_alloc.argtypes = [_i64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
    lib.rfm_peer_open.restype = _i32
    lib.rfm_peer_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
    lib.rfm_peer_close.restype = _i32
    lib.rfm_peer_close.argtypes = [_p]
    lib.rfm_peer_free.restype = _i32
    lib.rfm_peer_free.argtypes = [_p]
    lib.rfm_peer_sync.restype = _i32
    lib.rfm_peer_sync.argtypes = [ctypes.POINTER(PeerSyncArgs), _p]
    _lib = lib
    return lib


def error_string(code: int) -> str:
    return load().rfm_error_string(code).decode()


def version() -> str:
    return load().rfm_version().decode()


def check(func: str, code: int) -> None:
    if code != RFM_OK:
        raise RfmError(func, code)


def default_tile_cap() -> int:
    """On-chip tile cap for the solver (floats); ``RFM_LSAP_TILE_CAP`` overrides the library default."""
    return int(os.environ.get("RFM_LSAP_TILE_CAP", "-1"))


def make_plan(problems: np.ndarray, stride_q: int, stride_t: int,
              tile_cap: int | None = None) -> tuple[LsapPlan, np.ndarray]:
    """Run the host-side planner over a ``PROBLEM_DTYPE`` array.

    Fills the problems' scratch offsets in place; returns the plan and the CTA
    table (int32 ``[num_ctas, 4]``) to upload next to the problems.
    """
    if problems.dtype != PROBLEM_DTYPE or not problems.flags.c_contiguous:
        raise ValueError("problems must be a contiguous PROBLEM_DTYPE array")
    plan = LsapPlan()
    ctas = np.zeros((max(problems.shape[0], 1), 4), dtype=np.int32)
    cap = default_tile_cap() if tile_cap is None else int(tile_cap)
    check("rfm_lsap_make_plan",
          load().rfm_lsap_make_plan(problems.ctypes.data if problems.size else None, problems.shape[0],
                                    int(stride_q), int(stride_t), cap, ctas.ctypes.data, ctypes.byref(plan)))
    return plan, np.ascontiguousarray(ctas[: plan.num_ctas])
