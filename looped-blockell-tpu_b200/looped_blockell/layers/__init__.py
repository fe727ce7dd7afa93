"""Drop-in Python op surface of looped_blockell.layers (Block-ELL format,
BlockELLLinear, MLPBlock, RMSNorm)."""

from .block_ell import (BlockELLConfig, BlockELLTensor, block_ell_matmul, block_ell_to_dense,  # noqa: F401
                        create_block_ell_from_dense, create_random_topology)
from .mlp import BlockELLLinear, MLPBlock  # noqa: F401
from .norms import RMSNorm  # noqa: F401
