"""catseye_b200 — catseye's matrix-multiply hot path (sgemm + LLM matmul) on B200.

The product is libcatsgpu.so (catseye_b200/csrc, C ABI in include/catsgpu.h);
this package is its Python host mirror.  There is no CPU fallback.
"""
import os
import subprocess

from . import _lib  # noqa: F401
from ._lib import CatsGpuError, LIB_PATH  # noqa: F401

HERE = os.path.dirname(os.path.abspath(__file__))


def build(verbose=False):
    """Compile libcatsgpu.so for sm_100a (nvcc cross-compiles without a GPU)."""
    out = None if verbose else subprocess.DEVNULL
    subprocess.check_call(["make", "-j8", "-C", os.path.join(HERE, "csrc")], stdout=out)
    return LIB_PATH
