"""Build the C-ABI extension libbell_b200.so for sm_100a.

    python looped-blockell-tpu_b200/csrc/setup.py [-v] [-f]

Compiles every kernel source with nvcc (-gencode arch=compute_100a,code=sm_100a)
and links the shared library next to the Python package
(looped_blockell/libbell_b200.so), so it ships with the source tree.
"""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from build_lib import build  # noqa: E402

if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
