"""K-quant matvecs (Q3_K / Q6_K against Q8_K activations, quantize_q8_K, the
K-quant dequantizers) and the fp32-activation Q4_0 / Q8_0 matvec
(matmul_q4_0) on the GPU, against the golden fixtures recorded from the
reference and the oracle.

Bars: quantize_q8_K and the dequantizers bit-exact; matvecs normwise
relative error <= 1e-5 (integer block sums are exact; only the float
accumulation order differs)."""
import os

import numpy as np
import pytest

from models import rel
from oracle.cpu import Q3_K, Q4_0, Q6_K, Q8_0

pytestmark = pytest.mark.gpu
G = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def mm(gpu):
    from catseye_b200 import matmul
    return matmul


def _kquant_weight(t, n, d, seed):
    """Random K-quant rows (any bytes are a valid block) with small finite fp16 scales."""
    bs = 110 if t == Q3_K else 210
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 256, (d, n // 256, bs), dtype=np.uint8)
    sc = np.float16(rng.uniform(1e-4, 1e-3, (d, n // 256))).view(np.uint16)
    w[:, :, bs - 2] = sc & 0xff
    w[:, :, bs - 1] = sc >> 8
    return np.ascontiguousarray(w.reshape(d, -1))


def test_quantize_q8_K_bit_exact(mm, orc):
    g = np.load(os.path.join(G, "quant.npz"))
    assert np.array_equal(mm.quantize_q8_K(g["q8K_x"]), g["q8K"])
    rng = np.random.default_rng(4)
    for scale in (1e-6, 1.0, 1e4):
        x = (rng.standard_normal(4096) * scale).astype(np.float32)
        x[:256] = 0.0                                   # an all-zero block
        x[300], x[301] = 50 * scale, -50 * scale        # equal magnitudes: the first one sets the sign
        assert np.array_equal(mm.quantize_q8_K(x), orc.quantize_q8_K(x))


@pytest.mark.parametrize("t,name", [(Q3_K, "q3K"), (Q6_K, "q6K")])
def test_kquant_golden(mm, t, name):
    g = np.load(os.path.join(G, "quant.npz"))
    w = np.ascontiguousarray(g[name + "_w"])
    for r in range(8):
        got = mm.dequantize(t, w, r, 512)
        assert np.array_equal(got.view(np.uint32), g[name + "_deq"][r].view(np.uint32)), r
    out = np.zeros(8, np.float32)
    mm.matmul(t, out, g["q8K"], w, 512, 8)
    assert rel(out, g[name + "_mv"]) < 1e-5
    mm.unregister_weight(w)


@pytest.mark.parametrize("t", [Q3_K, Q6_K])
@pytest.mark.parametrize("n,d", [(4096, 4096), (11008, 333), (256, 1)])
def test_kquant_matvec_against_oracle(mm, orc, t, n, d):
    w = _kquant_weight(t, n, d, n + d + t)
    x = np.random.default_rng(d).standard_normal(n).astype(np.float32)
    xq = orc.quantize_q8_K(x)
    out = np.zeros(d, np.float32)
    mm.matmul(t, out, xq, w, n, d)
    fn = "oracle_matmul_q3_K_q8_K" if t == Q3_K else "oracle_matmul_q6_K_q8_K"
    assert rel(out, orc.matmul_prequant(fn, xq, w, n, d)) < 1e-5
    # the device form quantizes fp32 x on the device first
    import torch
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(d, device="cuda")
    mm.matvec_dev(w, dy, dx)
    torch.cuda.synchronize()
    assert np.array_equal(dy.cpu().numpy(), out)
    mm.unregister_weight(w)


@pytest.mark.parametrize("t", [Q4_0, Q8_0])
@pytest.mark.parametrize("n,d", [(4096, 4096), (11008, 4096), (64, 3)])
def test_matvec_f32_activations(mm, orc, t, n, d):
    rng = np.random.default_rng(n * 3 + d + t)
    w = orc.quantize_rows(t, (rng.standard_normal((d, n)) * 0.02).astype(np.float32))
    x = rng.standard_normal(n).astype(np.float32)
    ref = x.astype(np.float64) @ orc.dequantize(t, w, n, d).astype(np.float64).T
    out = np.zeros(d, np.float32)
    mm.matmul_f32act(t, out, x, w, n, d)
    assert rel(out, ref) < 1e-5
    import torch
    dy = torch.empty(d, device="cuda")
    mm.matvec_dev(w, dy, torch.from_numpy(x).cuda(), x_is_q8=2)
    torch.cuda.synchronize()
    assert rel(dy.cpu().numpy(), ref) < 1e-5
    mm.unregister_weight(w)
