"""libcatsgpu.so loads and exports every function include/catsgpu.h declares.
CPU only: nothing here launches a kernel."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "catsgpu.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cats_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from catseye_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        import catseye_b200
        catseye_b200.build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("cats_gpu_matmul_q4_0_q8", "cats_gpu_matmul_f32", "cats_gpu_quantize_q8", "cats_sgemm",
                 "cats_gemm_rnn", "cats_gemm_rnt", "cats_gemm_rtn", "cats_gpu_llama2_transformer"):
        assert must in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_the_header():
    from catseye_b200._lib import SIGNATURES
    assert set(declared_functions()) <= set(SIGNATURES)


def test_no_gpu_means_clean_error(lib):
    """Without a device the library reports an error instead of crashing."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    lib.cats_gpu_init.restype = ctypes.c_int
    assert lib.cats_gpu_init(0) != 0
