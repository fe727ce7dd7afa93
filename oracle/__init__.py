"""CPU oracle for the Block-ELL SwiGLU hot path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference algorithm of
bigwolfeman/looped-blockell-tpu for the Block-ELL SwiGLU forward path
and its backward.
It exists so the CUDA path can be checked against it.  Only the test suite,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it, and only as a checker or as the timed CPU
baseline.  The product package (``looped_blockell``) never imports it and has
no CPU fallback.

Pinning: ``tests/golden/make_golden.py`` imports the reference's own runnable
PyTorch/NumPy code (``interop/pt_model.py`` MLPBlock and RMSNorm,
``interop/convert_checkpoint.py`` _block_ell_to_dense, ``bonsai-test/bitlinear.py``
quantizers) and commits its outputs as fixtures under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this oracle against them.
"""

from .bell_oracle import *  # noqa: F401,F403
