"""Batched quantized-weight product on the tensor cores (cats_gpu_qgemm):
y[T][d] = x[T][n] W^T against the exact product of the oracle's dequantized
weights, in float64.  fp16 operands with fp32 accumulation: normwise relative
error <= 1e-3, the bar for the tensor-core paths."""
import numpy as np
import pytest

from models import rel
from oracle.cpu import Q4_0, Q8_0

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def mm(gpu):
    from catseye_b200 import matmul
    return matmul


def _case(orc, t, n, d, T, seed):
    rng = np.random.default_rng(seed)
    w = orc.quantize_rows(t, (rng.standard_normal((d, n)) * 0.02).astype(np.float32))
    x = rng.standard_normal((T, n)).astype(np.float32)
    ref = x.astype(np.float64) @ orc.dequantize(t, w, n, d).astype(np.float64).T
    return w, x, ref


# (n, d, T): full 128 x 256 tiles; ragged rows and tokens; a partial last
# 64-block segment (11008 = 5 x 2048 + 768); the smallest shapes; grids small
# enough that K is split across CTAs (long K, few rows: 16 splits; the 7B w2
# shape at batch 16); 16 and 32 tokens, 17 (ragged tokens in a 32-wide
# tile), one token, and d = 1000 (a last 128-row tile that runs out).  These
# registered weights have fewer than 4736 rows, so their tile layout is not
# the 16-row one and they run on the kernel that loads weights itself.
SHAPES = [(4096, 4096, 512), (4096, 1000, 16), (11008, 4096, 100), (64, 128, 1), (8192, 256, 300),
          (2048, 11008, 33), (128, 17, 7), (28672, 256, 16), (11008, 4096, 16), (4096, 2048, 32),
          (8192, 640, 17), (4096, 256, 1)]


@pytest.mark.parametrize("t", [Q4_0, Q8_0])
@pytest.mark.parametrize("n,d,T", SHAPES)
def test_qgemm_matches_exact_product(mm, orc, t, n, d, T):
    w, x, ref = _case(orc, t, n, d, T, n * 7 + d * 3 + T)
    mm.register_weight(w, t, n, d)
    try:
        y = mm.qgemm(w, x, T, n, d)
    finally:
        mm.unregister_weight(w)
    assert rel(y, ref) < TOL, rel(y, ref)


def test_qgemm_rows_equal_matvecs(mm, orc):
    """Each token's row of the batched product is the matvec of that token
    (the matvec quantizes x to Q8 first, so the two agree to ~1e-3)."""
    n, d, T = 4096, 512, 8
    w, x, ref = _case(orc, Q4_0, n, d, T, 5)
    mm.register_weight(w, Q4_0, n, d)
    try:
        y = mm.qgemm(w, x, T, n, d)
        for i in range(T):
            out = np.zeros(d, np.float32)
            mm.matmul(Q4_0, out, mm.quantize(x[i]), w, n, d)
            assert rel(y[i], out) < 2e-2
    finally:
        mm.unregister_weight(w)


def test_qgemm_device_form(mm, orc):
    import torch
    n, d, T = 4096, 384, 64
    w, x, ref = _case(orc, Q4_0, n, d, T, 9)
    mm.register_weight(w, Q4_0, n, d)
    try:
        dx = torch.from_numpy(x).cuda()
        dy = torch.empty((T, d), device="cuda")
        mm.qgemm_dev(w, dx, dy, T)
        torch.cuda.synchronize()
        assert rel(dy.cpu().numpy(), ref) < TOL
    finally:
        mm.unregister_weight(w)


def test_qgemm_refuses_f32_weights(mm):
    from catseye_b200._lib import CatsGpuError
    w = np.zeros((16, 64), np.float32)
    mm.register_weight(w, 0, 64, 16)
    try:
        with pytest.raises(CatsGpuError):
            mm.qgemm(w, np.zeros((2, 64), np.float32), 2, 64, 16)
    finally:
        mm.unregister_weight(w)


# Q4_0 weights in 16-row tiles (registered weights of 4736 rows and more,
# and every model weight) take the path that brings raw weight bytes in with
# tensor-map copies (four K slices a stage): full segments; a short last
# segment of 24 units (11008) and of exactly 8 (4352); a last segment too
# short for it (4160: 2 units, the load-fed kernel); ragged rows past the
# last 128-row tile; K splits that start on four-slice boundaries; 1 to 512
# tokens.
TMA_SHAPES = [(4096, 8192, 16), (11008, 8192, 16), (4096, 5000, 512), (28672, 4736, 100), (4352, 4800, 40),
              (4160, 4800, 16), (11008, 4864, 1), (8192, 4736, 256), (2048, 6000, 33)]


@pytest.mark.parametrize("n,d,T", TMA_SHAPES)
def test_qgemm_tma_path_matches_exact_product(mm, orc, n, d, T):
    w, x, ref = _case(orc, Q4_0, n, d, T, n * 11 + d + T)
    mm.register_weight(w, Q4_0, n, d)
    try:
        y = mm.qgemm(w, x, T, n, d)
    finally:
        mm.unregister_weight(w)
    assert rel(y, ref) < TOL, rel(y, ref)


def test_qgemm_plan_and_slice_timeline(mm, orc):
    """The plan the library reports for a 16-row-tile Q4_0 weight (tensor-map
    fed, K splits on four-slice boundaries), and the per-slice timeline of
    one product: every stamped slice's events in their causal order (warp 0
    finds the stage free before it arrives, the MMA thread finds the
    operands ready after that and commits after that; each warp's own stamp
    follows its arrival, so it may trail the MMA thread's), the product's
    result still exact."""
    import torch
    n, d, T = 4096, 4736, 16
    w, x, ref = _case(orc, Q4_0, n, d, T, 77)
    mm.register_weight(w, Q4_0, n, d)
    try:
        bn, splits, resident, tma, kper, occ, occ_err = mm.qgemm_plan(w, T)
        assert (bn, tma) == (16, 1) and splits >= 1 and resident >= 1 and occ_err == 0
        assert kper % 4 == 0 and splits * kper >= n // 64 > (splits - 1) * kper
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty((T, d), device="cuda")
        torch.cuda.synchronize()
        slices = min(8, kper)
        tr = mm.qgemm_trace(w, xd, yd, T, slices).astype(np.int64)
        assert rel(yd.cpu().numpy(), ref) < TOL
        for k in range(slices):
            free, done0, ready, commit = tr[k, 3], tr[k, 4], tr[k, 12], tr[k, 13]
            assert 0 < free <= done0 and free < ready <= commit, (k, tr[k])
            assert tr[k, 4:12].min() > 0, (k, tr[k])
        assert tr[slices, 0] <= tr[0, 3] and tr[slices, 1] <= tr[slices, 2]
    finally:
        mm.unregister_weight(w)
