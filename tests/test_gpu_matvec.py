"""CUDA matvec / quantize / dequantize against the oracle and the golden
fixtures, through the C ABI (host-pointer drop-ins and device-pointer forms).

Bars: quantize_q8 and dequantize bit-exact; matvec normwise relative error
<= 1e-5 (fp32 accumulation order differs from the reference's 8-lane AVX sum,
the per-block integer dots are exact)."""
import os

import numpy as np
import pytest

from models import rel
from oracle.cpu import F32, Q4_0, Q8_0

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-5


def golden(name):
    return np.load(os.path.join(G, name + ".npz"))


@pytest.fixture(scope="module")
def mm(gpu):
    from catseye_b200 import matmul
    return matmul


def test_quantize_q8_matches_reference_bits(mm):
    g = golden("quant")
    assert np.array_equal(mm.quantize(g["q8_x"]), g["q8_avx"])


def test_quantize_q8_dev_both_roundings(mm):
    import torch
    g = golden("quant")
    x = torch.from_numpy(g["q8_x"]).cuda()
    for mode, key in ((False, "q8_avx"), (True, "q8_scalar")):
        q = torch.zeros(x.numel() // 32 * 36, dtype=torch.int8, device="cuda")
        mm.quantize_dev(q, x, scalar_mode=mode)
        torch.cuda.synchronize()
        assert np.array_equal(q.cpu().numpy(), g[key]), key


def test_dequantize_q4_0_bit_exact(mm):
    g = golden("quant")
    for r in range(16):
        y = mm.dequantize(Q4_0, g["q4_w"], r, 256)
        assert np.array_equal(y.view(np.uint32), g["q4_deq"][r].view(np.uint32))


def test_dequantize_q8_0_bit_exact(mm, orc):
    rng = np.random.default_rng(11)
    w = orc.quantize_rows(Q8_0, (rng.standard_normal((5, 1024)) * 0.02).astype(np.float32))
    want = orc.dequantize(Q8_0, w, 1024, rows=5)
    for r in range(5):
        assert np.array_equal(mm.dequantize(Q8_0, w, r, 1024).view(np.uint32), want[r].view(np.uint32))


def test_matmul_golden(mm, orc):
    g = golden("matvec")
    for key in sorted({k.rsplit("_", 1)[0] for k in g.files}):
        t, n, d = (int(v[1:]) for v in key.split("_"))
        x = g[key + "_x"]
        xin = x if t == F32 else orc.quantize_q8(x)
        out = np.zeros(d, np.float32)
        w = g[key + "_w"]
        mm.matmul(t, out, xin, w, n, d)
        mm.unregister_weight(w)   # the registry is keyed by address; this array is about to be freed
        assert rel(out, g[key + "_avx"]) < TOL, key


SHAPES = [(32, 1), (64, 7), (288, 288), (288, 768), (768, 288), (1024, 33), (1376, 17), (4096, 4096),
          (11008, 512), (4096, 1000), (96, 129)]


@pytest.mark.parametrize("t", [F32, Q4_0, Q8_0])
@pytest.mark.parametrize("n,d", SHAPES)
def test_matmul_dropin_shapes(mm, orc, t, n, d):
    rng = np.random.default_rng(n * 7 + d)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    w = orc.quantize_rows(t, (rng.standard_normal((d, n)) * 0.02).astype(np.float32))
    if t == F32:
        want = orc.matmul(F32, x, w, n, d)
        xin = x
    else:
        xin = orc.quantize_q8(x)
        fn = "oracle_matmul_q4_0_q8" if t == Q4_0 else "oracle_matmul_q8_0_q8"
        want = orc.matmul_prequant(fn, xin, w, n, d)
    out = np.full(d, np.nan, np.float32)
    mm.matmul(t, out, xin, w, n, d)
    assert np.all(np.isfinite(out))
    assert rel(out, want) < TOL, (t, n, d)
    mm.unregister_weight(w)


@pytest.mark.parametrize("t", [F32, Q4_0, Q8_0])
def test_matvec_dev_fp32_input(mm, orc, t):
    """Device form with fp32 x: the kernel quantizes x itself (AVX rounding)."""
    import torch
    rng = np.random.default_rng(99 + t)
    n, d = 4096, 2048
    x = rng.standard_normal(n).astype(np.float32)
    w = orc.quantize_rows(t, (rng.standard_normal((d, n)) * 0.02).astype(np.float32))
    mm.register_weight(w, t, n, d)
    xd = torch.from_numpy(x).cuda()
    out = torch.zeros(d, device="cuda")
    mm.matvec_dev(w, out, xd)
    torch.cuda.synchronize()
    assert rel(out.cpu().numpy(), orc.matmul(t, x, w, n, d)) < TOL
    if t != F32:   # and with a pre-quantized input
        q = torch.from_numpy(orc.quantize_q8(x)).cuda()
        out2 = torch.zeros(d, device="cuda")
        mm.matvec_dev(w, out2, q, x_is_q8=True)
        torch.cuda.synchronize()
        assert torch.equal(out, out2)
    mm.unregister_weight(w)


def test_matmul_repeat_is_deterministic(mm, orc):
    rng = np.random.default_rng(1)
    n, d = 4096, 4096
    w = orc.quantize_rows(Q4_0, (rng.standard_normal((d, n)) * 0.02).astype(np.float32))
    xq = orc.quantize_q8(rng.standard_normal(n).astype(np.float32))
    a = np.zeros(d, np.float32)
    b = np.zeros(d, np.float32)
    mm.matmul(Q4_0, a, xq, w, n, d)
    mm.matmul(Q4_0, b, xq, w, n, d)
    assert np.array_equal(a, b)
    mm.unregister_weight(w)


def test_reregistration_on_shape_change(mm, orc):
    rng = np.random.default_rng(2)
    buf = np.zeros(64 * 18 * 8, np.uint8)
    w1 = orc.quantize_rows(Q4_0, (rng.standard_normal((8, 2048)) * 0.02).astype(np.float32)).reshape(-1)
    buf[:w1.size] = w1
    x = rng.standard_normal(2048).astype(np.float32)
    out = np.zeros(8, np.float32)
    mm.matmul(Q4_0, out, orc.quantize_q8(x), buf, 2048, 8)
    assert rel(out, orc.matmul(Q4_0, x, w1, 2048, 8)) < TOL
    w2 = orc.quantize_rows(Q4_0, (rng.standard_normal((16, 1024)) * 0.02).astype(np.float32)).reshape(-1)
    buf[:w2.size] = w2
    x2 = rng.standard_normal(1024).astype(np.float32)
    out2 = np.zeros(16, np.float32)
    mm.matmul(Q4_0, out2, orc.quantize_q8(x2), buf, 1024, 16)
    assert rel(out2, orc.matmul(Q4_0, x2, w2, 1024, 16)) < TOL
    mm.unregister_weight(buf)


def test_bad_arguments_are_rejected(mm):
    from catseye_b200._lib import CatsGpuError
    x = np.zeros(40, np.int8)
    w = np.zeros(18, np.uint8)
    out = np.zeros(1, np.float32)
    with pytest.raises(CatsGpuError):
        mm.matmul(Q4_0, out, x, w, 33, 1)      # n not a multiple of 32
    with pytest.raises(CatsGpuError):
        mm.matmul(Q4_0, out, x, w, 32, 0)      # no rows
    with pytest.raises(CatsGpuError):
        mm.quantize(np.zeros(31, np.float32))  # partial block
