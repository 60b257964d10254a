"""B200 (sm_100a) Hungarian matching for RF-DETR: fused cost kernel + exact batched LSAP.

Public API: ``HungarianMatcher`` (drop-in for rf-detr's), ``match_layers``,
``match_packed``, ``compute_compact_detection_cost_matrix``, ``assign_padded``,
``batch_linear_assignment``, ``MatchGraph`` / ``MatchGraphCache`` (the step as a
CUDA graph for repeated shapes) and ``patches.apply_patches`` (monkeypatches an
importable rf-detr).
"""

from .matcher import (  # noqa: F401
    HungarianMatcher,
    assign_padded,
    batch_linear_assignment,
    compute_compact_detection_cost_matrix,
    match_layers,
    match_packed,
)
from .graph import MatchGraph, MatchGraphCache  # noqa: F401
