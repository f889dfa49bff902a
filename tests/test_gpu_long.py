"""Long runs of the decode and prefill paths at the benchmark configurations'
own lengths, against the reference's own step (oracle/_ref, all cores) or the
oracle where the reference is not built.

* Decode attention past position 256, where the persistent kernel leaves its
  one-CTA-per-head form for the split form (and the graph engine's attention
  kernel runs long caches): fp32 weights, so every step's logits are held to
  1e-4 and the greedy token must match (cats_llama2_transformer's attention
  loops t = 0..pos over the whole cache, llm/catseye_llm.h:1685-1723).
* The 512-token prefill of the 70B-shape model (and a 300-token prefill of
  the 7B shape) through the batched tensor-core step against the reference's
  fp32-activation binding (matmul_q4_0 with quantize_null, :880-914), then
  decode steps of both single-token engines over the prefilled cache against
  the reference's default Q8 binding.
* The stories-shape fp32 model at its full length: 8 prompt tokens and 248
  greedy steps, equal token ids at every step (sample_argmax, :1944-1956).
* The full 32-layer 7B Q4_0 model over the positions the benchmark times:
  greedy token agreement with the reference step by step.

Models with 1 layer keep the benchmark shapes of everything attention sees
(dim, heads, kv heads, head size); their vocabulary and, for the fp32
attention runs, the hidden width are cut so the reference finishes in
seconds."""
from dataclasses import replace

import numpy as np
import pytest

from models import ModelWeights, prompt, rel
from oracle.cpu import F32, Q4_0

pytestmark = pytest.mark.gpu
ENGINES = [0, 1]   # persistent cooperative kernel, CUDA graph of per-phase kernels


@pytest.fixture(scope="module")
def llm(gpu):
    from catseye_b200 import llm
    return llm


def _reference(orc, mw, f32_act=False):
    """The reference's own step on all host cores, else the oracle."""
    from oracle.cpu import Reference, ref_available
    if ref_available("llm_allcores") and mw.cfg.wtype in (F32, Q4_0):
        return Reference("llm_allcores").llm(mw, f32_act=f32_act)
    return orc.llm(mw, 2 if f32_act else 0)


_REF_CACHE = {}


def _long_case(llm, orc, name):
    """(model weights, fed tokens, the reference's logits per step), shared by both engines."""
    if name in _REF_CACHE:
        return _REF_CACHE[name]
    base = {"7b": llm.LLAMA2_7B, "70b": llm.LLAMA2_70B}[name]
    steps = {"7b": 600, "70b": 400}[name]
    cfg = replace(base, n_layers=1, hidden=1024, vocab=1024, seq_len=1024, wtype=F32)
    mw = ModelWeights(cfg, 300 + len(name), orc)
    toks = prompt(300 + len(name), steps, cfg.vocab)
    r = _reference(orc, mw)
    logits = np.stack([r.step(int(t), p) for p, t in enumerate(toks)])
    del r
    _REF_CACHE[name] = (mw, toks, logits)
    return _REF_CACHE[name]


@pytest.mark.parametrize("engine", ENGINES)
@pytest.mark.parametrize("name", ["7b", "70b"])
def test_long_context_decode_fp32(llm, orc, name, engine):
    """Teacher-forced decode to position 599 (7B heads: 32 x 128) and 399
    (70B heads: 64 query heads over 8 kv heads), fp32 weights: logits within
    1e-4 and the same greedy token at every step, on both sides of the
    position-256 switch of the persistent kernel's attention."""
    mw, toks, want = _long_case(llm, orc, name)
    m = llm.GpuLLM(mw.cfg)
    m.set_engine(engine)
    m.set_weights(mw)
    errs = np.zeros(len(toks))
    for p, t in enumerate(toks):
        lg = m.step(int(t), p)
        errs[p] = rel(lg, want[p])
        assert int(np.argmax(lg)) == int(np.argmax(want[p])), (name, engine, p)
    m.close()
    assert errs[:256].max() < 1e-4, errs[:256].max()
    assert errs[256:].max() < 1e-4, (int(np.argmax(errs)), errs.max())


@pytest.mark.parametrize("name,T", [("7b", 300), ("70b", 512)])
def test_long_prefill_then_decode_q4_0(llm, orc, name, T):
    """A T-token prompt in one batched step (tcgen05 products, fp16 operands)
    against the reference's fp32-activation binding, logits per token within
    3e-3; then 8 greedy decode steps of each single-token engine over that
    cache (positions T..T+7) against the reference switched back to its Q8
    binding, within the Q8 flip amplitude (3e-2).

    The step's logits carry the fp16 rounding of the operands of its five
    chained products (qkv, attention, wo, w1/w3, w2, classifier), each within
    1e-3 of its exact product (test_gpu_qgemm): measured 0.7-2.0e-3 at the
    70B shapes (dim 8192, hidden 28672), 3e-3 is the bar."""
    base = {"7b": llm.LLAMA2_7B, "70b": llm.LLAMA2_70B}[name]
    cfg = replace(base, n_layers=1, vocab=2048, seq_len=1024, wtype=Q4_0)
    seed = 500 + T
    mw = ModelWeights(cfg, seed, orc)
    toks = prompt(seed, T, cfg.vocab)
    r = _reference(orc, mw, f32_act=True)
    want = np.stack([r.step(int(t), p) for p, t in enumerate(toks)])
    if not hasattr(r, "use_q8_activations"):
        pytest.skip("switching bindings after the prompt needs the compiled reference")
    r.use_q8_activations()
    feed, ref_dec = [int(np.argmax(want[-1]))], []
    for i in range(8):
        lr = r.step(feed[-1], T + i)
        ref_dec.append(lr)
        feed.append(int(np.argmax(lr)))
    del r
    for engine in ENGINES:
        m = llm.GpuLLM(cfg)
        m.set_engine(engine)
        m.set_weights(mw)
        m.batch_reserve(T, 1)
        _, lg = m.forward_batch(toks, np.arange(T, dtype=np.int32), logits=True)
        perr = [rel(lg[p], want[p]) for p in range(T)]
        assert max(perr) < 3e-3, (name, int(np.argmax(perr)), max(perr))
        derr = [rel(m.step(feed[i], T + i), ref_dec[i]) for i in range(8)]
        assert max(derr) < 3e-2, (name, engine, derr)
        m.close()


@pytest.mark.parametrize("engine", ENGINES)
def test_stories_full_length_greedy(llm, orc, engine):
    """The fp32 llama2.c-shape model (dim 288, 6 layers, vocab 32000,
    seq_len 256) for its whole context: 8 seeded prompt tokens, then 248
    greedy steps.  Every step's greedy token equals the reference's and the
    logits are within 1e-4; the device-fed greedy loop (argmax on the GPU, one
    launch for all 248 steps) gives the same ids."""
    cfg = llm.STORIES_F32
    mw = ModelWeights(cfg, 1, orc)
    toks = prompt(1, 8, cfg.vocab)
    r = _reference(orc, mw)
    m = llm.GpuLLM(cfg)
    m.set_engine(engine)
    m.set_weights(mw)
    tok, ids, errs = int(toks[0]), [], []
    for pos in range(cfg.seq_len):
        lg, lr = m.step(tok, pos), r.step(tok, pos)
        errs.append(rel(lg, lr))
        nxt = int(np.argmax(lr))
        assert int(np.argmax(lg)) == nxt, pos
        if pos >= 7:
            ids.append(nxt)
        tok = int(toks[pos + 1]) if pos + 1 < len(toks) else nxt
    assert max(errs) < 1e-4, (int(np.argmax(errs)), max(errs))
    assert len(ids) == 249
    # device-fed: after the prompt, the steps at positions 8..255 from the last prompt token's argmax
    g = llm.GpuLLM(cfg)
    g.set_engine(engine)
    g.set_weights(mw)
    for pos in range(7):
        g.step(int(toks[pos]), pos)
    dev = g.generate(int(toks[7]), 7, cfg.seq_len - 7)
    assert list(dev) == ids, [i for i, (a, b) in enumerate(zip(dev, ids)) if a != b][:5]
    m.close()
    g.close()


def test_llama7b_q4_0_token_agreement(llm, orc):
    """Full 32-layer 7B Q4_0 model, 8 prompt tokens then 128 greedy steps (the
    benchmark's decode), the reference fed the GPU's tokens.  Every step's
    logits stay within max(6e-2, 2x the reference's own AVX / plain-C spread)
    - the amplitude of a Q8 activation code rounding the other way (the
    spread measured on the first 4 steps), which stays bounded over the whole
    run instead of growing through the cache.  On these random weights the
    top logits are close (measured agreement 85%), so where the greedy tokens
    differ the GPU's token must be a near tie: the reference scores it within
    that step's largest logit difference of its own best.  Agreement >= 75%."""
    from oracle.cpu import Reference, ref_available
    if not ref_available("llm_scalar"):
        pytest.skip("compiled reference (oracle/_ref) not built here")
    from test_gpu_llm import _synth_weights
    cfg = replace(llm.LLAMA2_7B.with_type(Q4_0), seq_len=256)
    m = llm.GpuLLM(cfg)
    m.init_random(2024)
    w = _synth_weights(llm, cfg, 2024)
    avx = _reference(orc, w)
    plain = Reference("llm_scalar").llm(w)
    toks = list(prompt(2024, 8, cfg.vocab))
    agree, errs, spread, unexplained = 0, [], [], []
    tok = int(toks[0])
    n = 8 + 128
    for pos in range(n):
        lg, la = m.step(tok, pos).copy(), avx.step(tok, pos)
        errs.append(rel(lg, la))
        if pos < 4:   # the plain-C build is slow: its spread is measured on the first steps
            spread.append(rel(plain.step(tok, pos), la))
        g, gr = int(np.argmax(lg)), int(np.argmax(la))
        agree += g == gr
        if g != gr and la[gr] - la[g] > float(np.max(np.abs(lg - la))):
            unexplained.append(pos)
        tok = int(toks[pos + 1]) if pos + 1 < len(toks) else g
    m.close()
    bar = max(6e-2, 2 * max(spread))
    assert max(errs) < bar, (max(errs), bar)
    assert not unexplained, unexplained
    assert agree >= 0.75 * n, (agree, n)
