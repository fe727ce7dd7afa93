"""Block-ELL kernels for B200 (sm_100a), called through the C ABI of
libbell_b200.so.  The reference's ``looped_blockell/kernels/__init__.py`` is an
empty placeholder; this package fills it with the fused SwiGLU forward, the
single Block-ELL projection, the SwiGLU backward (``backward``), the ternary
path, the loop ops and host-buffer (pipelined) entry points, and registers the reference's native op names under
``torch.ops.titan`` on import (``torch_ops``; skipped when those names are
already defined in the process).
"""

from .ops import (TILE_IN_OUT, TILE_OUT_IN, block_ell_linear, block_ell_swiglu_fwd,  # noqa: F401
                  block_ell_swiglu_fwd_with_intermediate, plan_bytes, read_status, rmsnorm)
from .loop import (diagonal_injection, inject_rmsnorm, looped_ffn, persistent_mlp_step,  # noqa: F401
                   pin_weights_l2, unpin_weights_l2)
from .backward import (block_ell_sddmm, block_ell_swiglu, block_ell_swiglu_bwd, down_silu_bwd,  # noqa: F401
                       silu_mul_bwd, transpose_ell, transposed_topology)
from .convert import dense_to_block_ell  # noqa: F401
from .stream import block_ell_swiglu_fwd_host, looped_ffn_host, pipeline_tokens  # noqa: F401
from . import torch_ops as _torch_ops

_torch_ops.register()

# reference name for the fused op (csrc/block_ell/block_ell_ops.cpp:51)
swiglu_fwd = block_ell_swiglu_fwd
swiglu_bwd = block_ell_swiglu_bwd
