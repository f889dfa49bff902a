"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs the reference's own C functions, compiled from its headers by
oracle/Makefile into oracle/_ref/ (`make -C oracle ref`), on seeded inputs and
stores inputs and outputs as compressed .npz files.  The reference ships no
test vectors of its own, so these recorded outputs are what pins the oracle
and the CUDA path.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle.cpu import F32, Q4_0, Q3_K, Q6_K, Oracle, Reference  # noqa: E402
from catseye_b200.llm import LlmConfig  # noqa: E402
from models import ModelWeights, prompt  # noqa: E402


def quant(ref, refs, orc, rng):
    xs = []
    for k in range(8):
        x = (rng.standard_normal(1024) * 10.0 ** rng.uniform(-4, 3)).astype(np.float32)
        if k == 1:
            x[:96] = 0.0                       # all-zero blocks: d = 0, id = 0
        if k == 2:
            x = np.round(x * 2) / 2            # many exact .5 multiples of the step
        if k == 3:
            x[5::32] *= 1000                   # one dominant element per block
        xs.append(x)
    x = np.concatenate(xs).astype(np.float32)
    f = np.concatenate([rng.standard_normal(4000) * 10.0 ** rng.uniform(-8, 5, 4000),
                        [0.0, -0.0, 65504.0, 65520.0, 1e-8, 6.1e-5, 5.96e-8, 2.98e-8]]).astype(np.float32)
    h16 = np.array([ref.lib.ref_fp32_to_fp16(float(v)) for v in f], dtype=np.uint16)
    # Q4_0 matrix for dequantize
    w = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    wq = orc.quantize_rows(Q4_0, w)
    deq = np.stack([ref.dequantize(Q4_0, wq, r, 256) for r in range(16)])
    # K-quant blocks: any bytes are a valid block; keep the fp16 scale small and finite
    kq = {}
    for t, bs in ((Q3_K, 110), (Q6_K, 210)):
        blk = rng.integers(0, 256, (8, 2 * bs), dtype=np.uint8)   # 8 rows of n=512 (2 super-blocks)
        for r in range(8):
            for b in range(2):
                off = b * bs + bs - 2
                blk[r, off:off + 2] = np.frombuffer(np.float16(rng.uniform(1e-4, 1e-3)).tobytes(), np.uint8)
        kq[t] = blk
    xk = rng.standard_normal(512).astype(np.float32)
    out = dict(q8_x=x, q8_avx=ref.quantize_q8(x), q8_scalar=refs.quantize_q8(x),
               f32=f, f32_to_f16=h16, q4_w=wq, q4_deq=deq,
               q8K_x=xk, q8K=ref.quantize_q8_K(xk))
    for t, blk in kq.items():
        name = {Q3_K: "q3K", Q6_K: "q6K"}[t]
        out[name + "_w"] = blk
        out[name + "_deq"] = np.stack([ref.dequantize(t, blk, r, 512) for r in range(8)])
        out[name + "_mv"] = ref.matmul(t, xk, blk, 512, 8)
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **out)


def matvec(ref, refs, orc, rng):
    out = {}
    for t, n, d in ((F32, 288, 96), (F32, 1024, 40), (Q4_0, 512, 64), (Q4_0, 1376, 24)):
        x = rng.standard_normal(n).astype(np.float32)
        w = (rng.standard_normal((d, n)) * 0.02).astype(np.float32)
        wb = orc.quantize_rows(t, w)
        key = f"t{t}_n{n}_d{d}"
        out[key + "_x"] = x
        out[key + "_w"] = wb
        out[key + "_avx"] = ref.matmul(t, x, wb, n, d)
        out[key + "_scalar"] = refs.matmul(t, x, wb, n, d)
    np.savez_compressed(os.path.join(HERE, "matvec.npz"), **out)


def cnn(rc, rng):
    out = {}
    for ta, tb in (("N", "N"), ("N", "T"), ("T", "N")):
        for (M, N, K) in ((33, 17, 45), (64, 64, 64)):
            A = rng.uniform(-1, 1, M * K).astype(np.float32)
            B = rng.uniform(-1, 1, K * N).astype(np.float32)
            C0 = rng.uniform(-1, 1, M * N).astype(np.float32)
            base = f"{ta}{tb}_{M}_{N}_{K}"
            out[base + "_A"], out[base + "_B"], out[base + "_C0"] = A, B, C0
            for beta in (0.0, 1.0):
                out[f"{base}_b{int(beta)}_C"] = rc.sgemm(ta, tb, M, N, K, 1.0, A, B, beta, C0)
    im = rng.uniform(0, 1, 3 * 8 * 8).astype(np.float32)
    out["im2col_x"] = im
    out["im2col"] = rc.im2col(im, 3, 8, 8, 3, 3, 1, 1, 1, 1)
    x = rng.uniform(0, 1, 2 * 3 * 8 * 8).astype(np.float32)
    w = (rng.standard_normal(4 * 3 * 9) * np.sqrt(2 / 27)).astype(np.float32)
    out["conv_x"], out["conv_w"] = x, w
    out["conv_z"] = rc.conv2d_forward(x, w, 2, 3, 8, 8, 4, 3, 1, 1)
    xl = rng.uniform(0, 1, 3 * 20).astype(np.float32)
    wl = (rng.standard_normal(20 * 7 + 7) * 0.3).astype(np.float32)
    out["lin_x"], out["lin_w"] = xl, wl
    out["lin_z"] = rc.linear_forward(xl, wl, 3, 20, 7)
    np.savez_compressed(os.path.join(HERE, "cnn.npz"), **out)


def cnn_train(rc, rng):
    """The training layers: col2im, convolution backward / update (3x3 pad 1
    stride 1, and 3x3 pad 1 stride 2), linear backward / update."""
    out = {}
    col = rng.uniform(-1, 1, 3 * 9 * 8 * 8).astype(np.float32)
    out["col2im_col"] = col
    out["col2im"] = rc.col2im(col, 3, 8, 8, 3, 3, 1, 1, 1, 1)
    for name, (b, ich, h, wd, ch, k, pad, st) in (("s1", (2, 3, 8, 8, 4, 3, 1, 1)), ("s2", (2, 5, 9, 7, 6, 3, 1, 2))):
        oh, ow = (h + 2 * pad - k) // st + 1, (wd + 2 * pad - k) // st + 1
        x = rng.uniform(0, 1, b * ich * h * wd).astype(np.float32)
        w = (rng.standard_normal(ch * ich * k * k) * np.sqrt(2 / (ich * k * k))).astype(np.float32)
        dout = rng.uniform(-1, 1, b * ch * oh * ow).astype(np.float32)
        dw0 = rng.uniform(-0.1, 0.1, ch * ich * k * k).astype(np.float32)
        out[f"conv_{name}_x"], out[f"conv_{name}_w"], out[f"conv_{name}_dout"], out[f"conv_{name}_dw0"] = x, w, dout, dw0
        out[f"conv_{name}_din"] = rc.conv2d_backward(dout, w, b, ich, h, wd, ch, k, pad, st)
        out[f"conv_{name}_dw"] = rc.conv2d_update(dout, x, dw0, b, ich, h, wd, ch, k, pad, st)
    xl = rng.uniform(0, 1, 3 * 20).astype(np.float32)
    wl = (rng.standard_normal(20 * 7 + 7) * 0.3).astype(np.float32)
    dl = rng.uniform(-1, 1, 3 * 7).astype(np.float32)
    dwl = rng.uniform(-0.1, 0.1, 20 * 7).astype(np.float32)
    out["lin_x"], out["lin_w"], out["lin_dout"], out["lin_dw0"] = xl, wl, dl, dwl
    out["lin_din"] = rc.linear_backward(dl, wl, 3, 20, 7)
    out["lin_w1"], out["lin_dw"] = rc.linear_update(dl, xl, wl, dwl, 3, 20, 7, 0.01)
    np.savez_compressed(os.path.join(HERE, "cnn_train.npz"), **out)


TINY = LlmConfig(dim=64, hidden=96, n_layers=2, n_heads=4, n_kv_heads=2, vocab=128, seq_len=32)


def llm(ref, orc, t, name, f32_act=False):
    """f32_act: the Q4_0 tensors bound to matmul_q4_0 with quantize_null
    (fp32 activations), the reference's counterpart of the batched path."""
    cfg = TINY.with_type(t)
    mw = ModelWeights(cfg, 7, orc)
    toks = prompt(7, 4, cfg.vocab)
    m = ref.llm(mw, f32_act)
    logits, nxt, fed = [], [], []
    for pos in range(12):
        tok = int(toks[pos]) if pos < len(toks) else nxt[-1]   # prompt forcing, then greedy
        fed.append(tok)
        lg = m.step(tok, pos)
        logits.append(lg)
        nxt.append(ref.argmax(lg))
    out = {k: getattr(mw, k) for k in ("emb", "rms_att", "rms_ffn", "rms_final", "wq", "wk", "wv", "wo", "w1",
                                       "w2", "w3", "wcls")}
    out.update(prompt=toks, fed=np.array(fed, np.int32), logits=np.stack(logits), argmax=np.array(nxt, np.int32),
               cfg=np.array([cfg.dim, cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.vocab,
                             cfg.seq_len, cfg.wtype], np.int32))
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)


def main(only=None):
    """Writes every fixture, or only the named ones (argv)."""
    rng = np.random.default_rng(20240601)
    orc = Oracle()
    ref, refs, rc = Reference("llm"), Reference("llm_scalar"), Reference("cnn")
    assert ref.is_avx() and not refs.is_avx()
    want = (lambda n: not only or n in only)
    # quant, matvec and cnn draw from one stream in this order
    if want("quant") or want("matvec") or want("cnn"):
        quant(ref, refs, orc, rng)
        matvec(ref, refs, orc, rng)
        cnn(rc, rng)
    if want("cnn_train"):
        cnn_train(rc, np.random.default_rng(20241202))
    if want("llm_f32"):
        llm(ref, orc, F32, "llm_f32")
    if want("llm_q4_0"):
        llm(ref, orc, Q4_0, "llm_q4_0")
    if want("llm_q4_0_f32act"):
        llm(ref, orc, Q4_0, "llm_q4_0_f32act", f32_act=True)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main(sys.argv[1:])
