"""Seeded synthetic llama models in the reference's host layouts (test infrastructure:
tests and the CPU-baseline leg of bench.py).

Weights are N(0, std) from numpy's PCG64 stream, norms are 1.0, the embedding
is fp32; layer matrices and the classifier are block-quantized with the
oracle's synthetic quantizer.  fp32 models share the classifier with the
embedding, as llama2.c checkpoints do (llm/catseye_llm.h:2924).
"""
import numpy as np

from .cpu import F32, row_bytes


class ModelWeights:
    def __init__(self, cfg, seed, orc, std=0.02):
        self.cfg = cfg
        rng = np.random.default_rng(seed)
        t, L, dim, hid, kvd = cfg.wtype, cfg.n_layers, cfg.dim, cfg.hidden, cfg.kv_dim

        def mats(d, n):
            out = []
            for _ in range(L):
                w = rng.standard_normal((d, n), dtype=np.float32) * np.float32(std)
                out.append(orc.quantize_rows(t, w).reshape(-1))
            return np.concatenate(out)

        self.emb = (rng.standard_normal((cfg.vocab, dim), dtype=np.float32) * np.float32(std))
        self.rms_att = np.ones((L, dim), np.float32)
        self.rms_ffn = np.ones((L, dim), np.float32)
        self.rms_final = np.ones(dim, np.float32)
        self.wq = mats(dim, dim)
        self.wk = mats(kvd, dim)
        self.wv = mats(kvd, dim)
        self.wo = mats(dim, dim)
        self.w1 = mats(hid, dim)
        self.w2 = mats(dim, hid)
        self.w3 = mats(hid, dim)
        if t == F32:
            self.wcls = self.emb.view(np.uint8).reshape(-1).copy()
        else:
            w = rng.standard_normal((cfg.vocab, dim), dtype=np.float32) * np.float32(std)
            self.wcls = orc.quantize_rows(t, w).reshape(-1)
        assert self.wq.size == L * row_bytes(t, dim) * dim


def prompt(seed, n, vocab):
    return np.random.default_rng(seed + 1).integers(0, vocab, n).astype(np.int32)


def rel(a, b):
    """normwise relative error ||a-b|| / ||b||"""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
