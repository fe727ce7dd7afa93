"""looped_blockell (B200): the Block-ELL SwiGLU path of looped-blockell-tpu,
rebuilt for sm_100a.  ``layers`` keeps the reference's Python op surface;
``kernels`` holds the CUDA-backed ops."""

__version__ = "0.1.0"
