"""Model files straight to the device (cats_gpu_llm_load) against the same
weights uploaded as host blobs (cats_gpu_llm_set_weights) and against the
reference's own loader + step on the same file (oracle/_ref).

Loading only moves bytes: the loaded model's logits equal the set_weights
model's bit for bit.  Against the reference: fp32 <= 1e-4 with equal greedy
tokens, Q4_0 within the Q8 flip amplitude (3e-2)."""
import numpy as np
import pytest

from model_files import write_bin, write_ggjt, write_gguf
from models import ModelWeights, rel
from oracle.cpu import F32, Q4_0, Q8_0

pytestmark = pytest.mark.gpu
FEED = [3, 17, 200, 5, 99, 1, 42, 7]


@pytest.fixture(scope="module")
def llm(gpu):
    from catseye_b200 import llm
    return llm


def _cfg(llm, **kw):
    base = dict(dim=256, hidden=704, n_layers=2, n_heads=8, n_kv_heads=4, vocab=512, seq_len=64, wtype=Q4_0)
    base.update(kw)
    return llm.LlmConfig(**base)


def _run(m):
    return [m.step(t, p).copy() for p, t in enumerate(FEED)]


@pytest.mark.parametrize("fmt,t", [(1, Q4_0), (1, Q8_0), (1, F32), (2, Q4_0), (3, F32)])
def test_loaded_model_matches_set_weights_and_reference(llm, orc, tmp_path, fmt, t):
    if fmt == 2:   # the legacy format: kv heads = heads, context 2048, hidden from n_mult
        cfg = _cfg(llm, wtype=t, n_kv_heads=8, seq_len=2048, hidden=(2 * 4 * 256 // 3 + 31) // 32 * 32)
    else:
        cfg = _cfg(llm, wtype=t)
    mw = ModelWeights(cfg, 40 + fmt + t, orc)
    path = tmp_path / "model"
    if fmt == 1:
        write_gguf(path, mw)
    elif fmt == 2:
        emb_q = orc.quantize_rows(Q4_0, mw.emb)
        write_ggjt(path, mw, 32, emb_q.tobytes())
        mw.emb = orc.dequantize(Q4_0, emb_q.reshape(-1), cfg.dim, cfg.vocab).reshape(cfg.vocab, cfg.dim)
    else:
        write_bin(path, mw)
    a = llm.GpuLLM.load(path)
    assert a.cfg == cfg
    got = _run(a)
    a.close()
    b = llm.GpuLLM(cfg)
    b.set_weights(mw)
    want = _run(b)
    b.close()
    for g, w in zip(got, want):
        assert np.array_equal(g, w)
    from oracle.cpu import Reference, ref_available
    if t == Q8_0 or not ref_available("llm"):
        return   # the reference has no Q8_0 matmul
    r, _ = Reference("llm").load(path, fmt)
    errs = [rel(g, r.step(tok, p)) for p, (g, tok) in enumerate(zip(got, FEED))]
    assert max(errs) < (1e-4 if t == F32 else 3e-2), errs


def test_loaded_gguf_with_quantized_embedding_and_no_classifier(llm, orc, tmp_path):
    """A GGUF whose embedding is Q4_0 and which has no output.weight: the
    classifier is the embedding (shared), the embedding rows fp32 exactly."""
    cfg = _cfg(llm)
    mw = ModelWeights(cfg, 77, orc)
    emb_q = orc.quantize_rows(Q4_0, mw.emb)
    path = tmp_path / "m.gguf"
    write_gguf(path, mw, with_output=False, emb=(Q4_0, emb_q.tobytes()))
    a = llm.GpuLLM.load(path)
    got = _run(a)
    a.close()
    mw.emb = orc.dequantize(Q4_0, emb_q.reshape(-1), cfg.dim, cfg.vocab).reshape(cfg.vocab, cfg.dim)
    mw.wcls = emb_q.reshape(-1)
    b = llm.GpuLLM(cfg)
    b.set_weights(mw)
    for g, w in zip(got, _run(b)):
        assert np.array_equal(g, w)
    b.close()


def test_unsupported_mix_is_refused(llm, orc, tmp_path):
    from catseye_b200._lib import CatsGpuError
    cfg = _cfg(llm)
    mw = ModelWeights(cfg, 78, orc)
    path = tmp_path / "m.gguf"
    # classifier of another type than the layers (fp32 classifier bytes, Q4_0 layers) is refused
    write_gguf(path, mw, with_output=False, emb=(F32, mw.emb.astype(np.float32).tobytes()))
    with pytest.raises(CatsGpuError):
        llm.GpuLLM.load(path)
    m = llm.GpuLLM(cfg)   # the library stays usable
    m.set_weights(mw)
    assert np.isfinite(m.step(1, 0)).all()
    m.close()
