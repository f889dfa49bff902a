"""cats_sgemm_dev_noalloc: the device sgemm for callers that cannot allocate
device memory (their device memory belongs to another allocator, or they must
not meet cudaMalloc's implicit synchronisation).  Its split-K workspace is a
fixed array compiled into the library, so it allocates nothing.

Checked through the C ABI against cats_sgemm_dev on the same inputs, for two
calls in a row that both use the shared workspace, at the 1e-5 normwise bar
of the other sgemm tests, and once against the CPU oracle; a skinny product
whose natural K split would overflow the array runs with fewer splits; and,
where a second GPU is visible, a tensor-core-sized call on device 1 after
device 0.  This file runs last (its name sorts last) and also passes alone in
a fresh process."""
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


def test_noalloc_matches_the_oracle(lib):
    import torch
    from oracle.cpu import Oracle
    torch.cuda.set_device(0)
    rng = np.random.default_rng(12)
    m, n, k = 64, 768, 2048   # split K through the array
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    want = Oracle().sgemm("N", "N", m, n, k, 1.0, a.reshape(-1), b.reshape(-1), 1.0, c.reshape(-1))
    ga, gb, gc = (torch.from_numpy(v).cuda() for v in (a, b, c))
    assert _call(lib.cats_sgemm_dev_noalloc, "N", "N", m, n, k, ga, k, gb, n, 1.0, gc, n) == 0
    torch.cuda.synchronize()
    got = gc.cpu().numpy().reshape(-1)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < TOL
    assert lib.cats_gpu_device_error() == 0


def test_noalloc_fits_the_split_to_the_array(lib):
    import torch
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(13)
    # 64 tiles would take 5 K splits of 64x8192 partials (2.6 M floats) > the
    # 2 M-float array: the plan takes 4 instead and the product still runs
    m, n, k = 64, 8192, 8192
    a = torch.rand((m, k), device="cuda", generator=g) * 2 - 1
    b = torch.rand((k, n), device="cuda", generator=g) * 2 - 1
    want = torch.zeros((m, n), device="cuda")
    got = torch.full((m, n), float("nan"), device="cuda")
    assert _call(lib.cats_sgemm_dev, "N", "N", m, n, k, a, k, b, n, 0.0, want, n) == 0
    assert _call(lib.cats_sgemm_dev_noalloc, "N", "N", m, n, k, a, k, b, n, 0.0, got, n) == 0
    torch.cuda.synchronize()
    assert _rel(got, want) < TOL


def test_noalloc_on_a_second_device(lib):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU visible")
    g = torch.Generator(device="cpu").manual_seed(14)
    m, n, k = 512, 512, 1024   # a tensor-core-sized product (raised shared-memory limit per device)
    a = torch.rand((m, k), generator=g) * 2 - 1
    b = torch.rand((k, n), generator=g) * 2 - 1
    outs = []
    for dev in (0, 1):
        torch.cuda.set_device(dev)
        da, db = a.cuda(dev), b.cuda(dev)
        c = torch.zeros((m, n), device=f"cuda:{dev}")
        assert _call(lib.cats_sgemm_dev_noalloc, "N", "N", m, n, k, da, k, db, n, 0.0, c, n) == 0
        torch.cuda.synchronize(dev)
        outs.append(c.cpu())
    torch.cuda.set_device(0)
    want = (a.double() @ b.double()).float()
    for o in outs:
        assert float((o - want).norm() / want.norm()) < TOL
