"""Model-file parsing on the CPU: the library's loader (cats_gpu_llm_file_config,
no GPU) reads the hyperparameters of synthetic GGUF v2/v3, ggjt v3 and
llama2.c .bin files written by tests/model_files.py, the same ones the
reference's own loaders read from those files (oracle/_ref); damaged files
are refused with an error instead of being read past their end, and a long
metadata string (which the reference would copy into a 64-byte buffer,
llm/catseye_llm.h:2714) is parsed safely."""
import ctypes as C

import numpy as np
import pytest

from model_files import write_bin, write_ggjt, write_gguf
from models import ModelWeights
from oracle.cpu import F32, Q4_0


@pytest.fixture(scope="module")
def lib():
    from catseye_b200 import _lib
    return _lib.load()


def cfg_of(lib, path):
    from catseye_b200 import _lib
    c = _lib.LlmConfigC()
    rc = lib.cats_gpu_llm_file_config(str(path).encode(), C.byref(c))
    lib.cats_gpu_clear_error()
    return rc, [c.dim, c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab, c.seq_len, c.wtype]


def _cfg(**kw):
    from catseye_b200.llm import LlmConfig
    base = dict(dim=128, hidden=352, n_layers=2, n_heads=4, n_kv_heads=2, vocab=256, seq_len=64, wtype=Q4_0)
    base.update(kw)
    return LlmConfig(**base)


def _want(cfg):
    return [cfg.dim, cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.vocab, cfg.seq_len, cfg.wtype]


@pytest.mark.parametrize("version", [2, 3])
def test_gguf_config(lib, orc, tmp_path, version):
    cfg = _cfg()
    mw = ModelWeights(cfg, 5, orc)
    p = tmp_path / "m.gguf"
    write_gguf(p, mw, version=version)
    rc, got = cfg_of(lib, p)
    assert rc == 0 and got == _want(cfg)


def test_ggjt_config(lib, orc, tmp_path):
    cfg = _cfg(n_kv_heads=4, seq_len=2048)   # the legacy format has no kv-head count or context: heads, 2048
    mw = ModelWeights(cfg, 6, orc)
    emb_q = orc.quantize_rows(Q4_0, mw.emb).tobytes()
    p = tmp_path / "m.ggjt"
    write_ggjt(p, mw, 32, emb_q)
    rc, got = cfg_of(lib, p)
    assert rc == 0 and got == _want(cfg)


def test_bin_config(lib, orc, tmp_path):
    cfg = _cfg(wtype=F32)
    mw = ModelWeights(cfg, 7, orc)
    p = tmp_path / "m.bin"
    write_bin(p, mw)
    rc, got = cfg_of(lib, p)
    assert rc == 0 and got == _want(cfg)


@pytest.mark.parametrize("fmt", [1, 2, 3])
def test_same_hyperparameters_as_the_reference_loader(lib, orc, ref_llm, tmp_path, fmt):
    """The reference's own loader reads the same file to the same model shape."""
    if fmt == 2:
        cfg = _cfg(n_kv_heads=4, seq_len=2048)
        mw = ModelWeights(cfg, 8, orc)
        p = tmp_path / "m.ggjt"
        write_ggjt(p, mw, 32, orc.quantize_rows(Q4_0, mw.emb).tobytes())
    elif fmt == 1:
        cfg = _cfg()
        mw = ModelWeights(cfg, 8, orc)
        p = tmp_path / "m.gguf"
        write_gguf(p, mw)
    else:
        cfg = _cfg(wtype=F32)
        mw = ModelWeights(cfg, 8, orc)
        p = tmp_path / "m.bin"
        write_bin(p, mw)
    _, hp = ref_llm.load(p, fmt)
    rc, got = cfg_of(lib, p)
    assert rc == 0
    assert got[:7] == hp, (got, hp)


def test_long_metadata_string_is_read_safely(lib, orc, tmp_path):
    cfg = _cfg()
    mw = ModelWeights(cfg, 9, orc)
    p = tmp_path / "m.gguf"
    write_gguf(p, mw, extra_kv=[("general.description", 8, "x" * 5000), ("general.name", 8, "y" * 300)])
    rc, got = cfg_of(lib, p)
    assert rc == 0 and got == _want(cfg)


def test_damaged_files_are_refused(lib, orc, tmp_path):
    cfg = _cfg()
    mw = ModelWeights(cfg, 10, orc)
    p = tmp_path / "m.gguf"
    write_gguf(p, mw)
    data = p.read_bytes()
    cases = {
        "truncated_table": data[:400],
        "truncated_data": data[:len(data) - 1000],
        "bad_version": data[:4] + (7).to_bytes(4, "little") + data[8:],
        "huge_count": data[:8] + (1 << 40).to_bytes(8, "little") + data[16:],
        "empty": b"",
        "garbage": bytes(np.random.default_rng(0).integers(0, 256, 4096, dtype=np.uint8)),
    }
    for name, blob in cases.items():
        q = tmp_path / f"{name}.gguf"
        q.write_bytes(blob)
        rc, _ = cfg_of(lib, q)
        assert rc == 2, name   # CATS_ERR_ARG
    rc, _ = cfg_of(lib, tmp_path / "missing.gguf")
    assert rc == 2
