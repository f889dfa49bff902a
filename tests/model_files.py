"""Writes seeded synthetic models (oracle/models.py ModelWeights) as model
files in the three formats the reference's runtime loads, for the loader
tests: GGUF v2/v3 (llm/catseye_llm.h:2678-2895), the legacy llama.cpp 'ggjt'
v3 files (:2326-2550) and llama2.c .bin checkpoints (:2900-2993).

The files carry what the reference's own loaders need to read them (a
tokenizer vocabulary of short strings, output.weight), so the same file can be
loaded by the reference and by the library."""
import struct

import numpy as np

from oracle.cpu import F32, Q4_0, row_bytes

# GGUF value types
G_U32, G_F32, G_STR, G_ARR = 4, 6, 8, 9


def _layer_blob(mw, name, l):
    """Layer l's matrix `name` (wq .. w3) of a ModelWeights: bytes of [d][row]."""
    c = mw.cfg
    kvd = c.kv_dim
    n, d = {"wq": (c.dim, c.dim), "wk": (c.dim, kvd), "wv": (c.dim, kvd), "wo": (c.dim, c.dim),
            "w1": (c.dim, c.hidden), "w2": (c.hidden, c.dim), "w3": (c.dim, c.hidden)}[name]
    sz = row_bytes(c.wtype, n) * d
    blob = np.ascontiguousarray(getattr(mw, name)).view(np.uint8).reshape(-1)
    return blob[l * sz:(l + 1) * sz].tobytes(), n, d


def _tensors(mw, emb_bytes, emb_type, with_output, names):
    """(name, [ne0, ne1], type, bytes) of every tensor, in the GGUF naming
    (`names` maps them to another naming)."""
    c = mw.cfg
    out = [(names("token_embd.weight"), [c.dim, c.vocab], emb_type, emb_bytes)]
    for l in range(c.n_layers):
        out.append((names(f"blk.{l}.attn_norm.weight"), [c.dim], F32, mw.rms_att[l].astype(np.float32).tobytes()))
        for key, gg in (("wq", "attn_q"), ("wk", "attn_k"), ("wv", "attn_v"), ("wo", "attn_output"),
                        ("w1", "ffn_gate"), ("w2", "ffn_down"), ("w3", "ffn_up")):
            b, n, d = _layer_blob(mw, key, l)
            out.append((names(f"blk.{l}.{gg}.weight"), [n, d], c.wtype, b))
        out.append((names(f"blk.{l}.ffn_norm.weight"), [c.dim], F32, mw.rms_ffn[l].astype(np.float32).tobytes()))
    out.append((names("output_norm.weight"), [c.dim], F32, mw.rms_final.astype(np.float32).tobytes()))
    if with_output:
        out.append((names("output.weight"), [c.dim, c.vocab], c.wtype, np.ascontiguousarray(mw.wcls).tobytes()))
    return out


def _gstr(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, mw, version=3, with_output=True, alignment=32, extra_kv=(), emb=None):
    """emb: (type, bytes) of token_embd.weight (default: the fp32 embedding)."""
    c = mw.cfg
    emb_type, emb_bytes = emb if emb else (F32, mw.emb.astype(np.float32).tobytes())
    kv = [("general.architecture", G_STR, "llama"), ("general.alignment", G_U32, alignment),
          ("llama.context_length", G_U32, c.seq_len), ("llama.embedding_length", G_U32, c.dim),
          ("llama.block_count", G_U32, c.n_layers), ("llama.feed_forward_length", G_U32, c.hidden),
          ("llama.attention.head_count", G_U32, c.n_heads), ("llama.attention.head_count_kv", G_U32, c.n_kv_heads),
          ("llama.rope.dimension_count", G_U32, c.head_size)] + list(extra_kv)
    tensors = _tensors(mw, emb_bytes, emb_type, with_output, lambda n: n)
    body = bytearray()
    body += struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(kv) + 2)
    for key, t, v in kv:
        body += _gstr(key) + struct.pack("<I", t)
        body += _gstr(v) if t == G_STR else struct.pack("<I", v)
    body += _gstr("tokenizer.ggml.tokens") + struct.pack("<IIQ", G_ARR, G_STR, c.vocab)
    for i in range(c.vocab):
        body += _gstr(f"t{i}")
    body += _gstr("tokenizer.ggml.scores") + struct.pack("<IIQ", G_ARR, G_F32, c.vocab)
    body += np.zeros(c.vocab, np.float32).tobytes()
    off = 0
    offsets = []
    for name, ne, t, b in tensors:
        offsets.append(off)
        off = (off + len(b) + alignment - 1) // alignment * alignment
    for (name, ne, t, b), o in zip(tensors, offsets):
        body += _gstr(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne) + struct.pack("<IQ", t, o)
    body += b"\0" * ((-len(body)) % alignment)
    base = len(body)
    for (name, ne, t, b), o in zip(tensors, offsets):
        body += b"\0" * (base + o - len(body))
        body += b
    open(path, "wb").write(bytes(body))
    return tensors


def write_ggjt(path, mw, n_mult, emb_q4_0):
    """A ggjt v3 file; every matrix Q4_0 (the reference's legacy loader binds
    matmul_q4_0_q8 and _dequantize_q4_0 for all of them).  emb_q4_0: the
    embedding as Q4_0 blocks."""
    c = mw.cfg
    assert c.wtype == Q4_0 and c.hidden == (2 * (4 * c.dim) // 3 + n_mult - 1) // n_mult * n_mult
    legacy = {"token_embd.weight": "tok_embeddings.weight", "output_norm.weight": "norm.weight",
              "output.weight": "output.weight"}
    parts = {"attn_q": "attention.wq", "attn_k": "attention.wk", "attn_v": "attention.wv",
             "attn_output": "attention.wo", "attn_norm": "attention_norm", "ffn_gate": "feed_forward.w1",
             "ffn_down": "feed_forward.w2", "ffn_up": "feed_forward.w3", "ffn_norm": "ffn_norm"}

    def names(n):
        if n in legacy:
            return legacy[n]
        _, l, part, _w = n.split(".")
        return f"layers.{l}.{parts[part]}.weight"

    tensors = _tensors(mw, emb_q4_0, Q4_0, True, names)
    body = bytearray(struct.pack("<II", 0x67676a74, 3))
    body += struct.pack("<7I", c.vocab, c.dim, n_mult, c.n_heads, c.n_layers, c.head_size, 2)
    for i in range(c.vocab):
        w = f"t{i}".encode()
        body += struct.pack("<I", len(w)) + w + struct.pack("<f", 0.0)
    for name, ne, t, b in tensors:
        nb = name.encode()
        body += struct.pack("<III", len(ne), len(nb), t) + struct.pack(f"<{len(ne)}I", *ne) + nb
        body += b"\0" * ((-len(body)) % 32)
        body += b
    open(path, "wb").write(bytes(body))
    return tensors


def write_bin(path, mw):
    """A llama2.c checkpoint: fp32, classifier shared with the embedding."""
    c = mw.cfg
    assert c.wtype == F32
    out = [struct.pack("<7i", c.dim, c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab, c.seq_len),
           mw.emb.astype(np.float32).tobytes(), mw.rms_att.astype(np.float32).tobytes()]
    for k in ("wq", "wk", "wv", "wo"):
        out.append(np.ascontiguousarray(getattr(mw, k)).tobytes())
    out.append(mw.rms_ffn.astype(np.float32).tobytes())
    for k in ("w1", "w2", "w3"):
        out.append(np.ascontiguousarray(getattr(mw, k)).tobytes())
    out.append(mw.rms_final.astype(np.float32).tobytes())
    open(path, "wb").write(b"".join(out))
