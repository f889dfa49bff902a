"""The CPU oracle against the golden fixtures recorded from the reference
itself (tests/golden/make_golden.py), and live against the compiled reference
when oracle/_ref is present.  CPU only."""
import os

import numpy as np
import pytest

from models import rel
from oracle.cpu import F32, Q4_0, Q3_K, Q6_K, Q8_0

G = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(G, name + ".npz"))


def test_quantize_q8_bit_exact(orc):
    g = load("quant")
    assert np.array_equal(orc.quantize_q8(g["q8_x"], "avx"), g["q8_avx"])
    assert np.array_equal(orc.quantize_q8(g["q8_x"], "scalar"), g["q8_scalar"])


def test_avx_and_scalar_rounding_differ_only_by_one(orc):
    g = load("quant")
    a = g["q8_avx"].reshape(-1, 36)[:, :32].astype(int)
    s = g["q8_scalar"].reshape(-1, 36)[:, :32].astype(int)
    assert np.abs(a - s).max() <= 1


def test_fp16_conversions(orc):
    g = load("quant")
    got = np.array([orc.fp32_to_fp16(v) for v in g["f32"]], dtype=np.uint16)
    assert np.array_equal(got, g["f32_to_f16"])
    h = np.arange(0, 65536, 97, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([orc.fp16_to_fp32(x) for x in h], dtype=np.float32)
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin].view(np.uint32), ref[fin].view(np.uint32))


def test_dequantize_q4_0_bit_exact(orc):
    g = load("quant")
    got = orc.dequantize(Q4_0, g["q4_w"], 256, rows=16)
    assert np.array_equal(got.view(np.uint32), g["q4_deq"].view(np.uint32))


@pytest.mark.parametrize("t,name", [(Q3_K, "q3K"), (Q6_K, "q6K")])
def test_kquant_dequant_and_matvec(orc, t, name):
    g = load("quant")
    got = orc.dequantize(t, g[name + "_w"], 512, rows=8)
    assert np.array_equal(got.view(np.uint32), g[name + "_deq"].view(np.uint32))
    assert np.array_equal(orc.quantize_q8_K(g["q8K_x"]), g["q8K"])
    mv = orc.matmul_prequant(f"oracle_matmul_{'q3_K' if t == Q3_K else 'q6_K'}_q8_K", g["q8K"], g[name + "_w"], 512, 8)
    assert rel(mv, g[name + "_mv"]) < 1e-5


def test_matvec_golden(orc):
    g = load("matvec")
    for key in {k.rsplit("_", 1)[0] for k in g.files}:
        t, n, d = (int(v[1:]) for v in key.split("_"))
        got = orc.matmul(t, g[key + "_x"], g[key + "_w"], n, d)
        assert rel(got, g[key + "_avx"]) < 1e-5, key
        assert rel(got, g[key + "_scalar"]) < 1e-5, key


def test_sgemm_golden(orc):
    g = load("cnn")
    for k in g.files:
        if not k.endswith("_C") or k.startswith(("conv", "lin", "im2col")):
            continue
        base, b = k[:-2].rsplit("_b", 1)
        ta, tb = base[0], base[1]
        M, N, K = (int(v) for v in base.split("_")[1:])
        got = orc.sgemm(ta, tb, M, N, K, 1.0, g[base + "_A"], g[base + "_B"], float(b), g[base + "_C0"])
        assert rel(got, g[k]) < 1e-5, k


def test_im2col_conv_linear_golden(orc):
    g = load("cnn")
    assert np.array_equal(orc.im2col(g["im2col_x"], 3, 8, 8, 3, 3, 1, 1, 1, 1), g["im2col"])
    assert rel(orc.conv2d_forward(g["conv_x"], g["conv_w"], 2, 3, 8, 8, 4, 3, 1, 1), g["conv_z"]) < 1e-5
    assert rel(orc.linear_forward(g["lin_x"], g["lin_w"], 3, 20, 7), g["lin_z"]) < 1e-5


def test_cnn_training_layers_golden(orc):
    """col2im bit-exact; convolution / linear backward and update within 1e-5
    of the reference's layers (catseye.h:445-505, 533-556, 589-640)."""
    g = load("cnn_train")
    assert np.array_equal(orc.col2im(g["col2im_col"], 3, 8, 8, 3, 3, 1, 1, 1, 1), g["col2im"])
    for name, (b, ich, h, wd, ch, k, pad, st) in (("s1", (2, 3, 8, 8, 4, 3, 1, 1)), ("s2", (2, 5, 9, 7, 6, 3, 1, 2))):
        p = f"conv_{name}_"
        assert rel(orc.conv2d_backward(g[p + "dout"], g[p + "w"], b, ich, h, wd, ch, k, pad, st), g[p + "din"]) < 1e-5
        assert rel(orc.conv2d_update(g[p + "dout"], g[p + "x"], g[p + "dw0"], b, ich, h, wd, ch, k, pad, st),
                   g[p + "dw"]) < 1e-5
    assert rel(orc.linear_backward(g["lin_dout"], g["lin_w"], 3, 20, 7), g["lin_din"]) < 1e-5
    w1, dw = orc.linear_update(g["lin_dout"], g["lin_x"], g["lin_w"], g["lin_dw0"], 3, 20, 7, 0.01)
    assert rel(w1, g["lin_w1"]) < 1e-6 and rel(dw, g["lin_dw"]) < 1e-5


class _MW:
    def __init__(self, g):
        from catseye_b200.llm import LlmConfig
        c = [int(v) for v in g["cfg"]]
        self.cfg = LlmConfig(*c)
        for k in ("emb", "rms_att", "rms_ffn", "rms_final", "wq", "wk", "wv", "wo", "w1", "w2", "w3", "wcls"):
            setattr(self, k, np.ascontiguousarray(g[k]))


@pytest.mark.parametrize("name,tol", [("llm_f32", 1e-5), ("llm_q4_0", 1e-3)])
def test_llm_decode_golden(orc, name, tol):
    g = load(name)
    mw = _MW(g)
    m = orc.llm(mw)
    for pos, tok in enumerate(g["fed"]):
        lg = m.step(int(tok), pos)
        assert rel(lg, g["logits"][pos]) < tol, (name, pos)
        assert orc.argmax(lg) == g["argmax"][pos]


def test_llm_decode_f32_activations_golden(orc):
    """The oracle's fp32-activation mode (q8_mode=2) against the reference's
    Q4_0 tensors bound to matmul_q4_0 + quantize_null."""
    g = load("llm_q4_0_f32act")
    mw = _MW(g)
    m = orc.llm(mw, q8_mode=2)
    for pos, tok in enumerate(g["fed"]):
        lg = m.step(int(tok), pos)
        assert rel(lg, g["logits"][pos]) < 1e-5, pos
        assert orc.argmax(lg) == g["argmax"][pos]
    # and it is a different binding from the requantizing one
    assert rel(g["logits"], load("llm_q4_0")["logits"]) > 1e-4


def test_live_against_reference(orc, ref_llm):
    rng = np.random.default_rng(5)
    for n in (32, 4096, 11008):
        x = (rng.standard_normal(n) * rng.uniform(0.01, 50)).astype(np.float32)
        assert np.array_equal(orc.quantize_q8(x), ref_llm.quantize_q8(x))
    for t, n, d in ((F32, 256, 33), (Q4_0, 4096, 17)):
        x = rng.standard_normal(n).astype(np.float32)
        w = orc.quantize_rows(t, (rng.standard_normal((d, n)) * 0.02).astype(np.float32))
        assert rel(orc.matmul(t, x, w, n, d), ref_llm.matmul(t, x, w, n, d)) < 1e-5


def test_q8_0_roundtrip(orc):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((4, 256)) * 0.02).astype(np.float32)
    b = orc.quantize_rows(Q8_0, w)
    deq = orc.dequantize(Q8_0, b, 256, rows=4)
    d = np.abs(w).reshape(4, -1, 32).max(-1) / 127
    # half a step, plus 127 steps of the fp16 rounding of d (2^-11 relative)
    assert np.all(np.abs(deq - w).reshape(4, -1, 32) <= d[..., None] * (0.5 + 127 * 2.0 ** -11) + 1e-7)
