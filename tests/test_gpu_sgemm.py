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


# Shapes the tensor-core (3xTF32) kernel takes: M*N*K >= 2^24 with the
# contiguous extents a multiple of 4.  Ragged edges in every dimension, K
# tails shorter than one 32-deep slice, K splits (few output tiles, long K),
# a single output row block, a long-K product whose error budget is the
# tightest, and 160 output tiles on 148 SMs (the 12 past the last full wave
# run as 3 K pieces each, summed afterwards).
TC_SHAPES = [(300, 260, 1000), (196, 4100, 36), (4, 4096, 1024), (1024, 1024, 8192), (132, 516, 2052),
             (128, 128, 4096), (2048, 64, 1536), (2500, 2020, 2000)]


@pytest.mark.parametrize("ta,tb", [("N", "N"), ("N", "T"), ("T", "N"), ("T", "T")])
@pytest.mark.parametrize("M,N,K", TC_SHAPES)
def test_sgemm_tensor_core_shapes(mm, orc, ta, tb, M, N, K):
    rng = np.random.default_rng(M * 7919 + N * 31 + K)
    A = rng.uniform(-1, 1, M * K).astype(np.float32)
    B = rng.uniform(-1, 1, K * N).astype(np.float32)
    C0 = rng.uniform(-1, 1, M * N).astype(np.float32)
    for alpha, beta in ((1.0, 0.0), (0.5, 0.25)):
        c = C0.copy()
        mm.sgemm(ta, tb, M, N, K, alpha, A, B, beta, c)
        assert np.isfinite(c).all()
        assert rel(c, orc.sgemm(ta, tb, M, N, K, alpha, A, B, beta, C0)) < TOL, (alpha, beta)


def test_sgemm_tensor_core_wide_range(mm):
    """3xTF32 keeps fp32 accuracy where plain TF32 (10-bit mantissa) would not:
    operands spread over 2^-20..2^20, checked element-wise in float64."""
    rng = np.random.default_rng(12)
    M, N, K = 256, 384, 512
    A = (rng.uniform(-1, 1, M * K) * 2.0 ** rng.integers(-20, 20, M * K)).astype(np.float32)
    B = (rng.uniform(-1, 1, K * N) * 2.0 ** rng.integers(-20, 20, K * N)).astype(np.float32)
    c = np.zeros(M * N, np.float32)
    mm.sgemm("N", "N", M, N, K, 1.0, A, B, 0.0, c)
    want = A.reshape(M, K).astype(np.float64) @ B.reshape(K, N).astype(np.float64)
    mag = np.abs(A.reshape(M, K)).astype(np.float64) @ np.abs(B.reshape(K, N)).astype(np.float64)
    # |error| against the sum of |a||b|: each 3xTF32 product is within
    # 3 * 2^-22 of a*b and fp32 accumulation adds ~sqrt(K) * 2^-24, while one
    # tf32 rounding (2^-11) of the dominant terms would show as ~2^-12
    assert float(np.max(np.abs(c.reshape(M, N) - want) / mag)) < 2.0 ** -16


def test_beta_zero_ignores_nan_in_c(mm, orc):
    rng = np.random.default_rng(4)
    A = rng.uniform(-1, 1, 40 * 30).astype(np.float32)
    B = rng.uniform(-1, 1, 30 * 20).astype(np.float32)
    c = np.full(40 * 20, np.nan, np.float32)
    mm.sgemm("N", "N", 40, 20, 30, 1.0, A, B, 0.0, c)
    assert rel(c, orc.sgemm("N", "N", 40, 20, 30, 1.0, A, B, 0.0, np.zeros(800, np.float32))) < TOL
    M, N, K = 256, 256, 512   # the same on the tensor-core path
    A = rng.uniform(-1, 1, M * K).astype(np.float32)
    B = rng.uniform(-1, 1, K * N).astype(np.float32)
    c = np.full(M * N, np.nan, np.float32)
    mm.sgemm("N", "N", M, N, K, 1.0, A, B, 0.0, c)
    assert rel(c, orc.sgemm("N", "N", M, N, K, 1.0, A, B, 0.0, np.zeros(M * N, np.float32))) < TOL


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


# The standalone SGEMM configuration (square M = N = K of 1024, 2048, 4096 in
# the three forms catseye.h calls, beta 0 and 1) through the host drop-in
# cats_sgemm, checked on 64 sampled rows of C: against the reference's own
# gemm_rnn / gemm_rnt / gemm_rtn run on those rows only (A's sampled rows,
# or A's sampled columns for TN, which give exactly those rows of C), and
# against a float64 product.  The reference accumulates in fp32 in K order,
# so its own error grows with K: the bar against it is 1e-5 plus that error.
@pytest.mark.parametrize("beta", [0.0, 1.0])
@pytest.mark.parametrize("ta,tb", [("N", "N"), ("N", "T"), ("T", "N")])
@pytest.mark.parametrize("n", [1024, 2048, 4096])
def test_sgemm_config_sizes_sampled_rows(mm, ref_cnn, ta, tb, n, beta):
    rng = np.random.default_rng(n * 7 + (ta == "T") * 3 + (tb == "T") + int(beta) * 11)
    A = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    B = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    C0 = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    c = C0.copy()
    mm.sgemm(ta, tb, n, n, n, 1.0, A, B, beta, c)
    rows = np.sort(rng.choice(n, 64, replace=False))
    a_rows = np.ascontiguousarray(A[:, rows] if ta == "T" else A[rows])   # [K][64] for TN, else [64][K]
    c_ref = ref_cnn.sgemm(ta, tb, 64, n, n, 1.0, a_rows.reshape(-1), B.reshape(-1), beta,
                          np.ascontiguousarray(C0[rows]).reshape(-1)).reshape(64, n)
    opA = (A.T if ta == "T" else A)[rows].astype(np.float64)
    opB = (B.T if tb == "T" else B).astype(np.float64)
    exact = opA @ opB + beta * C0[rows].astype(np.float64)
    got = c[rows]
    assert rel(got, exact) < TOL, (ta, tb, n, beta)
    assert rel(got, c_ref) < TOL + rel(c_ref, exact), (ta, tb, n, beta, rel(c_ref, exact))
