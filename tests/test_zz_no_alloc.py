"""cats_sgemm_dev_noalloc: the device sgemm for callers that cannot allocate
device memory (their device memory belongs to another allocator, or they must
not meet cudaMalloc's implicit synchronisation).  Its split-K workspace is a
fixed array compiled into the library, so it allocates nothing.

Checked through the C ABI against cats_sgemm_dev on the same inputs, for two
calls in a row that both use the shared workspace, at the 1e-5 normwise bar
of the other sgemm tests; and a problem whose workspace would not fit is
refused before any launch.  This file runs last (its name sorts last) and
also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(scope="module")
def lib():
    from catseye_b200 import _lib
    return _lib.load()


def _call(fn, ta, tb, m, n, k, a, lda, b, ldb, beta, c, ldc):
    return fn(ta.encode(), tb.encode(), m, n, k, 1.0, C.c_void_p(a.data_ptr()), lda, C.c_void_p(b.data_ptr()), ldb,
              beta, C.c_void_p(c.data_ptr()), ldc, None)


def _rel(a, b):
    return float((a - b).norm() / b.norm())


def test_noalloc_matches_sgemm_dev_twice(lib):
    import torch
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(11)
    # skinny shapes, so the plan splits K through the workspace
    for (ta, tb, m, n, k) in (("N", "N", 64, 1024, 4096), ("T", "N", 96, 512, 3000)):
        a = torch.rand((k, m) if ta == "T" else (m, k), device="cuda", generator=g) * 2 - 1
        b = torch.rand((n, k) if tb == "T" else (k, n), device="cuda", generator=g) * 2 - 1
        lda, ldb = a.shape[1], b.shape[1]
        c0 = torch.rand((m, n), device="cuda", generator=g)
        want = c0.clone()
        assert _call(lib.cats_sgemm_dev, ta, tb, m, n, k, a, lda, b, ldb, 1.0, want, n) == 0
        for _ in range(2):   # two calls in a row over the same shared workspace
            got = c0.clone()
            assert _call(lib.cats_sgemm_dev_noalloc, ta, tb, m, n, k, a, lda, b, ldb, 1.0, got, n) == 0
            torch.cuda.synchronize()
            assert _rel(got, want) < TOL
        # a different problem in between must not see the previous call's partial sums
        a2 = torch.rand_like(a) * 2 - 1
        want2 = torch.zeros((m, n), device="cuda")
        got2 = torch.full((m, n), float("nan"), device="cuda")
        assert _call(lib.cats_sgemm_dev, ta, tb, m, n, k, a2, lda, b, ldb, 0.0, want2, n) == 0
        assert _call(lib.cats_sgemm_dev_noalloc, ta, tb, m, n, k, a2, lda, b, ldb, 0.0, got2, n) == 0
        torch.cuda.synchronize()
        assert _rel(got2, want2) < TOL


def test_noalloc_refuses_a_workspace_it_cannot_hold(lib):
    import torch
    m, n, k = 64, 8192, 8192   # 64 tiles -> 5 K-splits of 64x8192 partials = 2.6 M floats > 2 M
    a = torch.zeros((m, k), device="cuda")
    b = torch.zeros((k, n), device="cuda")
    c = torch.zeros((m, n), device="cuda")
    assert _call(lib.cats_sgemm_dev_noalloc, "N", "N", m, n, k, a, k, b, n, 0.0, c, n) == 2   # CATS_ERR_ARG
    lib.cats_gpu_clear_error()
