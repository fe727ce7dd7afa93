"""Topology maintenance of Block-ELL weights, on the device holding them.

Same names and argument meaning as the reference's ``looped_blockell/opt``
(``compaction.compact_single_layer``, ``column_reorder.*``).  These are index
operations over [R, K] arrays and gathers of whole tiles, done with tensor
operations on the weights' own device; the dense -> Block-ELL conversion that
precedes them has its own kernels (``kernels.convert``).
"""

from .compaction import compact_single_layer  # noqa: F401
from .column_reorder import (apply_permutation_to_block_ell, compute_column_importance,  # noqa: F401
                             compute_k_active_macros, compute_permutation, full_reorder_step,
                             reorder_swiglu_dff)
