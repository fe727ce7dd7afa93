"""Block-ELL kernels for B200 (sm_100a), called through the C ABI of
libbell_b200.so.  The reference's ``looped_blockell/kernels/__init__.py`` is an
empty placeholder; this package fills it with the fused SwiGLU forward, the
single Block-ELL projection, the ternary path and the loop ops, and registers
the reference's native op names under ``torch.ops.titan`` (see ``torch_ops``).
"""

from .ops import (TILE_IN_OUT, TILE_OUT_IN, block_ell_linear, block_ell_swiglu_fwd,  # noqa: F401
                  block_ell_swiglu_fwd_with_intermediate, plan_bytes, read_status, rmsnorm)
from .loop import (diagonal_injection, looped_ffn, persistent_mlp_step, pin_weights_l2,  # noqa: F401
                   unpin_weights_l2)

# reference name for the fused op (csrc/block_ell/block_ell_ops.cpp:51)
swiglu_fwd = block_ell_swiglu_fwd
