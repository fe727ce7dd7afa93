"""Build libbell_b200.so (the C-ABI extension) for sm_100a with nvcc.

The library is written in-tree next to the Python package
(``looped_blockell/libbell_b200.so``) so it travels with the source tree.
Objects are cached under ``csrc/_build/`` and rebuilt when a source or header
is newer.  Used by ``csrc/setup.py`` and by ``__graft_entry__.build()``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

CSRC = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(CSRC)
REPO = os.path.dirname(PKG_ROOT)
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(CSRC, "_build")
LIB = os.path.join(PKG_ROOT, "looped_blockell", "libbell_b200.so")

SOURCES = ["bell_common.cu", "bell_bf16.cu", "bell_bf16_t.cu", "bell_f32.cu", "bell_ternary.cu", "bell_loop.cu", "bell_loop_kernel.cu", "bell_noalloc.cu", "bell_bwd.cu", "bell_convert.cu", "bell_small.cu", "bell_exchange.cu", "bell_f32x.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills", "-I" + INCLUDE, "-I" + CSRC]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    out = [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return out


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False, extra_flags=None) -> str:
    """Compile every source for sm_100a and link the shared library; returns its path."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    hdrs = _headers()
    extra = list(extra_flags or [])
    srcs = [s for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]
    objs = []

    def compile_one(src):
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        path = os.path.join(CSRC, src)
        if force or _stale(obj, [path] + hdrs):
            cmd = [nvcc, *ARCH, *FLAGS, *extra, "-c", path, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
            if verbose and (r.stdout or r.stderr):
                print(r.stdout, r.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(compile_one, srcs))

    if force or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "shared", "-o", LIB, *objs,
               "-Xlinker", "-rpath,/usr/local/cuda/lib64"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
