"""Batched step on the tensor cores (prefill and batched decode,
cats_gpu_llm_forward_batch / _generate_batch) against the oracle's
fp32-activation mode: cats_llama2_transformer with the Q4_0 tensors bound to
matmul_q4_0 + quantize_null (llm/catseye_llm.h:880-914), which
tests/golden/llm_q4_0_f32act.npz pins to the reference itself.

The batched products take fp16 operands (weights dequantized to fp16,
activations rounded to fp16, relative rounding <= 2^-11 each) and accumulate
in fp32, so each product is within ~5e-4 of the exact one; head-size-128
prefill attention also runs on the tensor cores with fp16 operands.  Measured
on B200: logits 4e-4 .. 1.2e-3 from the oracle (tiny GQA, 7B and 70B shapes),
against ~1e-2 between the oracle's fp32- and Q8-activation modes; TOL is 1.6x
the largest."""
from dataclasses import replace

import numpy as np
import pytest

from models import ModelWeights, prompt, rel
from oracle.cpu import Q4_0, Q8_0

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.fixture(scope="module")
def llm(gpu):
    from catseye_b200 import llm
    return llm


def _tiny(llm, t):
    # GQA (kv_mul 2), head_size 32, every product's n a multiple of 64
    return llm.LlmConfig(dim=128, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, vocab=512, seq_len=64, wtype=t)


@pytest.mark.parametrize("t", [Q4_0, Q8_0])
def test_prefill_matches_stepwise_oracle(llm, orc, t):
    cfg = _tiny(llm, t)
    mw = ModelWeights(cfg, 11, orc)
    toks = prompt(11, 12, cfg.vocab)
    m = llm.GpuLLM(cfg)
    m.set_weights(mw)
    m.batch_reserve(16, 1)
    nxt, lg = m.forward_batch(toks, np.arange(12), logits=True)
    r = orc.llm(mw, q8_mode=2)
    errs = []
    for p, tok in enumerate(toks):
        ref = r.step(int(tok), p)
        errs.append(rel(lg[p], ref))
        assert int(nxt[p]) == int(np.argmax(lg[p]))
    print("prefill rel errors", t, ["%.2e" % e for e in errs])
    assert max(errs) < TOL, errs
    m.close()


def test_prefill_in_pieces_equals_one_call(llm, orc):
    """The KV cache written by one call is what the next call attends to:
    12 tokens in one call or as 7 + 5 give the same logits for the last 5."""
    cfg = _tiny(llm, Q4_0)
    mw = ModelWeights(cfg, 5, orc)
    toks = prompt(5, 12, cfg.vocab)
    a = llm.GpuLLM(cfg)
    a.set_weights(mw)
    a.batch_reserve(16, 1)
    _, la = a.forward_batch(toks, np.arange(12), logits=True)
    b = llm.GpuLLM(cfg)
    b.set_weights(mw)
    b.batch_reserve(16, 1)
    b.forward_batch(toks[:7], np.arange(7))
    _, lb = b.forward_batch(toks[7:], np.arange(7, 12), logits=True)
    assert rel(lb, la[7:]) < 1e-6
    a.close()
    b.close()


def test_several_sequences_prefill_and_decode(llm, orc):
    """Three sequences of different lengths prefilled in one call, then
    decoded one token of each per step: every row against its own oracle
    sequence; then the device-resident greedy loop reproduces the ids."""
    cfg = _tiny(llm, Q4_0)
    mw = ModelWeights(cfg, 21, orc)
    lens = [5, 8, 3]
    prompts = [prompt(100 + i, n, cfg.vocab) for i, n in enumerate(lens)]
    toks = np.concatenate(prompts)
    pos = np.concatenate([np.arange(n) for n in lens])
    seqs = np.concatenate([np.full(n, i) for i, n in enumerate(lens)])
    refs = [orc.llm(mw, q8_mode=2) for _ in lens]

    m = llm.GpuLLM(cfg)
    m.set_weights(mw)
    m.batch_reserve(16, 3)
    nxt, lg = m.forward_batch(toks, pos, seqs, logits=True)
    for row in range(toks.size):
        ref = refs[seqs[row]].step(int(toks[row]), int(pos[row]))
        assert rel(lg[row], ref) < TOL, row
    last = np.cumsum(lens) - 1
    cur = nxt[last].copy()
    cur_pos = np.array(lens)
    first, first_pos = cur.copy(), cur_pos.copy()
    ids = []
    for step in range(6):
        nx, lg = m.forward_batch(cur, cur_pos, np.arange(3), logits=True)
        for i in range(3):
            ref = refs[i].step(int(cur[i]), int(cur_pos[i]))
            assert rel(lg[i], ref) < TOL, (step, i)
        ids.append(nx.copy())
        cur, cur_pos = nx, cur_pos + 1
    m.close()

    g = llm.GpuLLM(cfg)
    g.set_weights(mw)
    g.batch_reserve(16, 3)
    g.forward_batch(toks, pos, seqs)
    out = g.generate_batch(first, first_pos, 6)
    assert np.array_equal(out, np.stack(ids))
    g.close()


def test_llama7b_shape_two_layers(llm, orc):
    """Every 7B-shaped product (qkv 4096->12288, wo, w1/w3 4096->2x11008,
    w2 11008->4096, classifier 4096->32000) at T=16 tokens of one prompt."""
    from test_gpu_llm import _synth_weights
    cfg = replace(llm.LLAMA2_7B, n_layers=2, seq_len=64, wtype=Q4_0)
    m = llm.GpuLLM(cfg)
    m.init_random(2024)
    m.batch_reserve(16, 1)
    toks = prompt(3, 16, cfg.vocab)
    _, lg = m.forward_batch(toks, np.arange(16), logits=True)
    r = orc.llm(_synth_weights(llm, cfg, 2024), q8_mode=2)
    errs = [rel(lg[p], r.step(int(tok), p)) for p, tok in enumerate(toks)]
    print("7B-shape rel errors", ["%.2e" % e for e in errs])
    assert max(errs) < TOL, errs
    m.close()


def test_llama70b_shape_one_layer_gqa(llm, orc):
    """70B shapes (dim 8192, 64 heads over 8 kv heads: 64-row query blocks of
    8 tokens x 8 heads, hidden 28672) at T=8."""
    from test_gpu_llm import _synth_weights
    cfg = replace(llm.LLAMA2_70B, n_layers=1, seq_len=32, wtype=Q4_0)
    m = llm.GpuLLM(cfg)
    m.init_random(70)
    m.batch_reserve(8, 1)
    toks = prompt(4, 8, cfg.vocab)
    _, lg = m.forward_batch(toks, np.arange(8), logits=True)
    r = orc.llm(_synth_weights(llm, cfg, 70), q8_mode=2)
    errs = [rel(lg[p], r.step(int(tok), p)) for p, tok in enumerate(toks)]
    print("70B-shape rel errors", ["%.2e" % e for e in errs])
    assert max(errs) < TOL, errs
    m.close()


def test_batch_refuses_bad_input(llm, orc):
    from catseye_b200._lib import CatsGpuError
    cfg = _tiny(llm, Q4_0)
    m = llm.GpuLLM(cfg)
    m.set_weights(ModelWeights(cfg, 1, orc))
    with pytest.raises(CatsGpuError):
        m.forward_batch([1, 2], [0, 1])          # nothing reserved
    m.batch_reserve(4, 2)
    for toks, pos, seqs in (([1] * 5, range(5), None),            # more tokens than reserved
                            ([1, 2], [0, 64], None),              # position beyond the cache
                            ([1, 2], [0, 1], [0, 2]),             # no such sequence
                            ([1, 512], [0, 1], None)):            # token outside the vocabulary
        with pytest.raises(CatsGpuError):
            m.forward_batch(toks, list(pos), seqs)
    m.close()
    f = llm.GpuLLM(cfg.with_type(0))                                # fp32 weights: the matvec engines only
    f.set_weights(ModelWeights(cfg.with_type(0), 1, orc))
    with pytest.raises(CatsGpuError):
        f.batch_reserve(4, 1)
    f.close()


@pytest.mark.parametrize("engine", [0, 1])
def test_prefill_then_single_token_decode(llm, orc, engine):
    """A prompt prefilled by one batched step is continued by the single-token
    engines (persistent kernel, graph): the oracle runs the prompt in its
    fp32-activation mode and the next steps with quantize_q8, as the two
    device paths do.  The prefilled cache differs from the oracle's by the
    fp16 rounding (~5e-4), enough to flip a few Q8 activation codes in the
    decode steps: their bar is the flip amplitude of the single-token tests
    (3e-2; measured 0.8-1.1e-2).  A model whose cache never saw the prompt
    lands far outside it, so the bar still shows the cache is the one read."""
    cfg = _tiny(llm, Q4_0)
    mw = ModelWeights(cfg, 31, orc)
    toks = prompt(31, 8, cfg.vocab)
    m = llm.GpuLLM(cfg)
    m.set_engine(engine)
    m.set_weights(mw)
    m.batch_reserve(8, 1)
    nxt, lg = m.forward_batch(toks, np.arange(8), logits=True)
    cold = llm.GpuLLM(cfg)               # same weights, empty cache
    cold.set_engine(engine)
    cold.set_weights(mw)
    r = orc.llm(mw, q8_mode=2)
    pre = [rel(lg[p], r.step(int(tok), p)) for p, tok in enumerate(toks)]
    r.s.q8_mode = 0                      # the decode steps quantize their activations
    tok = int(nxt[-1])
    dec, unprimed = [], []
    for p in range(8, 12):
        got = m.step(tok, p).copy()
        ref = r.step(tok, p)
        dec.append(rel(got, ref))
        unprimed.append(rel(cold.step(tok, p).copy(), ref))
        tok = int(np.argmax(got))
    print("prefill", ["%.1e" % e for e in pre], "decode", ["%.1e" % e for e in dec],
          "empty cache", ["%.1e" % e for e in unprimed])
    assert max(pre) < TOL
    assert max(dec) < 3e-2
    assert min(unprimed) > 3 * 3e-2
    m.close()
    cold.close()
