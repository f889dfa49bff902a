"""Tensor-parallel decode over NCCL: a model sharded over 2 GPUs (one
process per GPU) against the same seeded model on one GPU.

Each rank quantizes the same 32-blocks the unsharded model does; only the
allreduce's summation order differs.  Bars: fp32 logits <= 1e-4 per step and
equal greedy tokens; Q4_0 within the Q8 flip amplitude (3e-2).  Needs two
visible GPUs (skipped on one)."""
import os
import socket

import numpy as np
import pytest

from models import rel

pytestmark = pytest.mark.gpu

CFG = dict(dim=512, hidden=1408, n_layers=2, n_heads=8, n_kv_heads=2, vocab=4096, seq_len=64)
FEED = [3, 17, 400, 4095, 5, 123, 77, 9]
SEED = 31


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _decode_run(m):
    """Per-step logits of FEED and 12 greedy tokens after it (single-token engines)."""
    logits = [m.step(t, p).copy() for p, t in enumerate(FEED)]
    toks = m.generate(int(np.argmax(logits[-1])), len(FEED), 12)
    return logits, [int(t) for t in toks]


def _batch_run(m):
    """FEED prefilled in one batched step (logits of every token), then 6
    batched greedy steps of two sequences: FEED's continuation and a second
    sequence started from token 5 at position 0."""
    m.batch_reserve(16, 2)
    nxt, lg = m.forward_batch(FEED, np.arange(len(FEED)), logits=True)
    gen = m.generate_batch([int(nxt[-1]), 5], [len(FEED), 0], 6)
    return [row.copy() for row in lg], [int(t) for t in np.asarray(gen).reshape(-1)]


def _rank(rank, world, port, wtype, batched, out):
    import torch.distributed as dist
    from catseye_b200 import _lib, llm
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _lib.init(rank)
        m = llm.GpuLLM(llm.LlmConfig(**CFG, wtype=wtype), rank, world)
        m.tp_connect(llm.tp_share_id())
        m.init_random(SEED)
        logits, toks = (_batch_run if batched else _decode_run)(m)
        m.close()
        out.put((rank, logits, toks))
    except Exception as e:   # reported to the parent, which fails the test
        out.put((rank, repr(e), None))
    finally:
        dist.destroy_process_group()


def _sharded(wtype, world=2, batched=False):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, wtype, batched, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, logits, toks = q.get(timeout=600)
        res[r] = (logits, toks)
    for p in procs:
        p.join(timeout=120)
    for r, (logits, toks) in res.items():
        assert toks is not None, (r, logits)
    return res


@pytest.fixture(scope="module")
def two_gpus(gpu):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallel needs two visible GPUs")


@pytest.mark.parametrize("wtype,tol", [(0, 1e-4), (2, 3e-2)])
def test_two_rank_decode_matches_one_gpu(two_gpus, wtype, tol):
    from catseye_b200 import llm
    one = llm.GpuLLM(llm.LlmConfig(**CFG, wtype=wtype))
    one.set_engine(llm.ENGINE_GRAPH)
    one.init_random(SEED)
    ref, ref_toks = _decode_run(one)
    one.close()
    res = _sharded(wtype)
    for r, (logits, toks) in res.items():
        errs = [rel(a, b) for a, b in zip(logits, ref)]
        assert max(errs) < tol, (r, errs)
        if wtype == 0:
            assert [int(np.argmax(a)) for a in logits] == [int(np.argmax(b)) for b in ref]
            assert toks == ref_toks, r
    # every rank holds the full logits and decodes the same tokens
    assert res[0][1] == res[1][1]
    assert all(np.array_equal(a, b) for a, b in zip(res[0][0], res[1][0]))


def test_two_rank_batched_step_matches_one_gpu(two_gpus):
    """The batched step sharded over 2 GPUs (wo/w2 partial products
    sum-allreduced, classifier slices allgathered) against the same model on
    one GPU.  Only fp32 summation orders differ, but a residual that differs
    in its last bits can round to the neighbouring fp16 value when it becomes
    the next product's operand, so the logits carry that flip (measured
    <= 2.1e-4; bar 1e-3, half the batched step's bar against the oracle) and
    the greedy tokens of both sequences are equal."""
    from catseye_b200 import llm
    one = llm.GpuLLM(llm.LlmConfig(**CFG, wtype=2))
    one.init_random(SEED)
    ref, ref_toks = _batch_run(one)
    one.close()
    res = _sharded(2, batched=True)
    for r, (logits, toks) in res.items():
        errs = [rel(a, b) for a, b in zip(logits, ref)]
        print("rank", r, "logit errors", ["%.1e" % e for e in errs], "tokens", toks, "one GPU", ref_toks)
        assert max(errs) < 1e-3, (r, errs)
        assert toks == ref_toks, r
    assert res[0][1] == res[1][1]
