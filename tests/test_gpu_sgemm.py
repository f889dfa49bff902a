"""CUDA sgemm (NN / NT / TN as catseye.h calls them) against the oracle and
the golden fixtures; normwise relative error <= 1e-5."""
import os

import numpy as np
import pytest

from models import rel

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(scope="module")
def mm(gpu):
    from catseye_b200 import matmul
    return matmul


def test_sgemm_golden(mm):
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "cnn.npz"))
    for k in g.files:
        if not k.endswith("_C") or k.startswith(("conv", "lin", "im2col")):
            continue
        base, b = k[:-2].rsplit("_b", 1)
        M, N, K = (int(v) for v in base.split("_")[1:])
        c = g[base + "_C0"].copy()
        mm.sgemm(base[0], base[1], M, N, K, 1.0, g[base + "_A"], g[base + "_B"], float(b), c)
        assert rel(c, g[k]) < TOL, k


SHAPES = [(1, 1, 1), (7, 5, 3), (33, 17, 45), (64, 64, 64), (128, 128, 128), (129, 131, 257), (256, 256, 256),
          (1000, 3, 7), (3, 1000, 7), (64, 1024, 27), (64, 1024, 576), (128, 256, 1152), (128, 10, 256),
          (64, 4096, 4096), (512, 512, 512)]


@pytest.mark.parametrize("ta,tb", [("N", "N"), ("N", "T"), ("T", "N"), ("T", "T")])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_sgemm_shapes(mm, orc, ta, tb, M, N, K):
    rng = np.random.default_rng(M * 10007 + N * 101 + K)
    A = rng.uniform(-1, 1, M * K).astype(np.float32)
    B = rng.uniform(-1, 1, K * N).astype(np.float32)
    C0 = rng.uniform(-1, 1, M * N).astype(np.float32)
    for alpha, beta in ((1.0, 0.0), (1.0, 1.0), (0.5, 0.25)):
        c = C0.copy()
        mm.sgemm(ta, tb, M, N, K, alpha, A, B, beta, c)
        assert rel(c, orc.sgemm(ta, tb, M, N, K, alpha, A, B, beta, C0)) < TOL, (alpha, beta)


def test_beta_zero_ignores_nan_in_c(mm, orc):
    rng = np.random.default_rng(4)
    A = rng.uniform(-1, 1, 40 * 30).astype(np.float32)
    B = rng.uniform(-1, 1, 30 * 20).astype(np.float32)
    c = np.full(40 * 20, np.nan, np.float32)
    mm.sgemm("N", "N", 40, 20, 30, 1.0, A, B, 0.0, c)
    assert rel(c, orc.sgemm("N", "N", 40, 20, 30, 1.0, A, B, 0.0, np.zeros(800, np.float32))) < TOL


def test_sgemm_dev_leading_dimensions(mm, orc):
    import torch
    rng = np.random.default_rng(8)
    M, N, K = 70, 90, 110
    A = torch.from_numpy(rng.uniform(-1, 1, (M, K + 6)).astype(np.float32)).cuda()
    B = torch.from_numpy(rng.uniform(-1, 1, (K, N + 2)).astype(np.float32)).cuda()
    C = torch.zeros(M, N + 10, device="cuda")
    mm.sgemm_dev("N", "N", M, N, K, 1.0, A, K + 6, B, N + 2, 0.0, C, N + 10)
    torch.cuda.synchronize()
    want = orc.sgemm("N", "N", M, N, K, 1.0, A[:, :K].cpu().numpy(), B[:, :N].cpu().numpy(), 0.0,
                     np.zeros(M * N, np.float32))
    assert rel(C[:, :N].cpu().numpy().reshape(-1), want) < TOL
    assert float(C[:, N:].abs().max()) == 0.0


def test_gemm_forms_drop_in(gpu, orc):
    """cats_gemm_rnn/rnt/rtn have catseye.h's gemm_* signatures."""
    import ctypes as C
    rng = np.random.default_rng(6)
    M, N, K = 31, 29, 37
    A = rng.uniform(-1, 1, M * K).astype(np.float32)
    B = rng.uniform(-1, 1, K * N).astype(np.float32)
    for name, ta, tb in (("cats_gemm_rnn", "N", "N"), ("cats_gemm_rnt", "N", "T"), ("cats_gemm_rtn", "T", "N")):
        c = np.zeros(M * N, np.float32)
        getattr(gpu, name)(M, N, K, 1.0, C.c_void_p(A.ctypes.data), C.c_void_p(B.ctypes.data), 0.0,
                           C.c_void_p(c.ctypes.data))
        assert rel(c, orc.sgemm(ta, tb, M, N, K, 1.0, A, B, 0.0, np.zeros(M * N, np.float32))) < TOL
