"""Device-resident llama decode over libcatsgpu (cats_llama2_transformer on a B200).

`GpuLLM` owns a cats_gpu_llm: weights uploaded from host blobs in the
reference's layouts (what cats_checkpoint_load / cats_gguf_load bind,
llm/catseye_llm.h:2897-2993) or generated on the device, a fp32 KV cache, and
a CUDA graph of one decode step.
"""
import ctypes as C
from dataclasses import dataclass, replace

import numpy as np

from . import _lib

F32, Q4_0, Q8_0 = 0, 2, 8
ENGINE_PERSISTENT, ENGINE_GRAPH = 0, 1


@dataclass(frozen=True)
class LlmConfig:
    dim: int
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab: int
    seq_len: int
    wtype: int = F32

    @property
    def head_size(self):
        return self.dim // self.n_heads

    @property
    def kv_dim(self):
        return self.dim * self.n_kv_heads // self.n_heads

    def with_type(self, t):
        return replace(self, wtype=t)


# the model shapes the benchmarks are quoted on
STORIES_F32 = LlmConfig(dim=288, hidden=768, n_layers=6, n_heads=6, n_kv_heads=6, vocab=32000, seq_len=256, wtype=F32)
LLAMA2_7B = LlmConfig(dim=4096, hidden=11008, n_layers=32, n_heads=32, n_kv_heads=32, vocab=32000, seq_len=2048,
                      wtype=Q4_0)
LLAMA2_70B = LlmConfig(dim=8192, hidden=28672, n_layers=80, n_heads=64, n_kv_heads=8, vocab=32000, seq_len=2048,
                       wtype=Q4_0)


def weight_bytes(cfg):
    """Bytes of layer + classifier weights one decode step reads (the reference layout)."""
    def rb(n):
        return {F32: n * 4, Q4_0: n // 32 * 18, Q8_0: n // 32 * 34}[cfg.wtype]
    per_layer = rb(cfg.dim) * (2 * cfg.dim + 2 * cfg.kv_dim + 2 * cfg.hidden) + rb(cfg.hidden) * cfg.dim
    return cfg.n_layers * per_layer + rb(cfg.dim) * cfg.vocab


class GpuLLM:
    def __init__(self, cfg: LlmConfig, tp_rank=0, tp_size=1):
        self.lib = _lib.init()
        self.cfg = cfg
        c = _lib.LlmConfigC(cfg.dim, cfg.hidden, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.vocab, cfg.seq_len,
                            cfg.wtype, tp_rank, tp_size)
        self.h = self.lib.cats_gpu_llm_create(C.byref(c))
        if not self.h:
            _lib.check(None, "cats_gpu_llm_create")
            raise _lib.CatsGpuError("cats_gpu_llm_create failed")
        self._logits = np.zeros(cfg.vocab, dtype=np.float32)
        self._view, self._view_ptr = None, None

    @classmethod
    def load(cls, path, tp_rank=0, tp_size=1, seq_len=0):
        """A model straight from a GGUF v2/v3, ggjt v3 or llama2.c .bin file
        (cats_gpu_llm_load): this rank's slices uploaded a layer at a time."""
        lib = _lib.init()
        c = _lib.LlmConfigC()
        _lib.check(lib.cats_gpu_llm_file_config(str(path).encode(), C.byref(c)), "file_config")
        self = cls.__new__(cls)
        self.lib = lib
        self.cfg = LlmConfig(c.dim, c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab,
                             seq_len or c.seq_len, c.wtype)
        self.h = lib.cats_gpu_llm_load(str(path).encode(), tp_rank, tp_size, seq_len)
        if not self.h:
            _lib.check(None, "cats_gpu_llm_load")
            raise _lib.CatsGpuError("cats_gpu_llm_load failed")
        self._logits = np.zeros(self.cfg.vocab, dtype=np.float32)
        self._view, self._view_ptr = None, None
        return self

    def set_weights(self, mw):
        """mw: object with numpy blobs emb, rms_att, rms_ffn, rms_final, wq, wk, wv, wo, w1, w2, w3, wcls."""
        ptrs = [C.c_void_p(np.ascontiguousarray(getattr(mw, n)).ctypes.data)
                for n in ("emb", "rms_att", "rms_ffn", "rms_final", "wq", "wk", "wv", "wo", "w1", "w2", "w3", "wcls")]
        _lib.check(self.lib.cats_gpu_llm_set_weights(self.h, *ptrs), "set_weights")

    def init_random(self, seed, std=0.02):
        _lib.check(self.lib.cats_gpu_llm_init_random(self.h, seed, std), "init_random")

    def tp_connect(self, unique_id):
        """Join this rank's NCCL communicator (every rank calls it with the same id)."""
        _framework_nccl_first()
        buf = C.create_string_buffer(bytes(unique_id), len(unique_id))
        _lib.check(self.lib.cats_gpu_llm_tp_connect(self.h, buf), "tp_connect")

    def step(self, token, pos, out=None):
        """cats_llama2_transformer(token, pos): logits of this step (host numpy).
        Into `out` when given; otherwise a view of the model's own page-locked
        copy, which the model's next step overwrites (copy it to keep it), as
        the reference returns its state's logits array."""
        p = self.lib.cats_gpu_llama2_transformer(token, pos, self.h,
                                                 None if out is None else C.c_void_p(out.ctypes.data))
        if not p:
            _lib.check(None, "llama2_transformer")
            raise _lib.CatsGpuError("llama2_transformer failed")
        if out is not None:
            return out
        if self._view is None or self._view_ptr != p:
            self._view = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), shape=(self.cfg.vocab,))
            self._view_ptr = p
        return self._view

    def generate(self, token, pos, steps):
        """Greedy decode fully on the device; returns the argmax ids of the steps."""
        toks = np.zeros(max(steps, 1), dtype=np.int32)
        _lib.check(self.lib.cats_gpu_llm_generate(self.h, token, pos, steps, C.c_void_p(toks.ctypes.data)), "generate")
        return toks[:steps]

    # ---- batched step on the tensor cores (prefill, batched decode)
    def batch_reserve(self, max_tokens, n_seqs=1):
        """Room for max_tokens per batched step and n_seqs KV sequences."""
        _lib.check(self.lib.cats_gpu_llm_batch_reserve(self.h, max_tokens, n_seqs), "batch_reserve")

    def forward_batch(self, tokens, pos, seqs=None, logits=False):
        """T tokens through the model at once (token t at pos[t] of sequence
        seqs[t]); returns the greedy argmax per token, and the [T][vocab]
        logits when asked."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        T = tokens.size
        sp = None
        if seqs is not None:
            seqs = np.ascontiguousarray(seqs, np.int32)
            sp = C.c_void_p(seqs.ctypes.data)
        nxt = np.zeros(T, np.int32)
        lg = np.zeros((T, self.cfg.vocab), np.float32) if logits else None
        _lib.check(self.lib.cats_gpu_llm_forward_batch(
            self.h, C.c_void_p(tokens.ctypes.data), C.c_void_p(pos.ctypes.data), sp, T,
            C.c_void_p(nxt.ctypes.data), C.c_void_p(lg.ctypes.data) if logits else None), "forward_batch")
        return (nxt, lg) if logits else nxt

    def generate_batch(self, tokens, pos, steps):
        """Greedy decoding of len(tokens) sequences (sequence i from tokens[i]
        at pos[i]), one token of each per step; returns [steps][n] ids."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        n = tokens.size
        out = np.zeros((max(steps, 1), n), np.int32)
        _lib.check(self.lib.cats_gpu_llm_generate_batch(self.h, C.c_void_p(tokens.ctypes.data),
                                                        C.c_void_p(pos.ctypes.data), n, steps,
                                                        C.c_void_p(out.ctypes.data)), "generate_batch")
        return out[:steps]

    def batch_set(self, tokens, pos, seqs=None):
        """Upload a batch for batch_enqueue (timing)."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        sp = None
        if seqs is not None:
            seqs = np.ascontiguousarray(seqs, np.int32)
            sp = C.c_void_p(seqs.ctypes.data)
        _lib.check(self.lib.cats_gpu_llm_batch_set(self.h, C.c_void_p(tokens.ctypes.data),
                                                   C.c_void_p(pos.ctypes.data), sp, tokens.size), "batch_set")

    def batch_enqueue(self):
        """Enqueue one batched step of the batch set last on the model's stream."""
        _lib.check(self.lib.cats_gpu_llm_batch_enqueue(self.h), "batch_enqueue")

    def batch_enqueue_decode(self, steps):
        """Enqueue `steps` greedy steps of the batch set last (one token per sequence)."""
        _lib.check(self.lib.cats_gpu_llm_batch_enqueue_decode(self.h, steps), "batch_enqueue_decode")

    def time_product(self, kind, T, reps=2):
        """(ms, FLOPs, weight bytes) per launch of one batched product kind at
        T tokens: 0 qkv, 1 wo, 2 w13, 3 w2, 4 classifier."""
        ms, fl, wb = C.c_float(), C.c_double(), C.c_double()
        _lib.check(self.lib.cats_gpu_llm_time_product(self.h, kind, T, reps, C.byref(ms), C.byref(fl), C.byref(wb)),
                   "time_product")
        return ms.value, fl.value, wb.value

    def tp_loopback(self):
        """Failure-detection check on one GPU: every rank's exchange buffer is
        this rank's own, so the first exchange of a step waits for ranks that
        never arrive and the step raises CatsGpuError (CATS_ERR_TIMEOUT)."""
        _lib.check(self.lib.cats_gpu_llm_tp_loopback(self.h), "tp_loopback")

    def tp_persistent(self):
        """Select the persistent kernel for this model; False (engine unchanged)
        when this build runs the model only in the per-phase graph engine."""
        if self.lib.cats_gpu_llm_set_engine(self.h, ENGINE_PERSISTENT) != 0:
            self.lib.cats_gpu_clear_error()
            return False
        return True

    def set_engine(self, engine):
        """ENGINE_PERSISTENT (default): one cooperative kernel runs whole tokens;
        ENGINE_GRAPH: a CUDA graph of per-phase kernels."""
        _lib.check(self.lib.cats_gpu_llm_set_engine(self.h, engine), "set_engine")

    def set_position(self, token, pos):
        _lib.check(self.lib.cats_gpu_llm_set_position(self.h, token, pos), "set_position")

    def enqueue(self, steps):
        _lib.check(self.lib.cats_gpu_llm_enqueue(self.h, steps), "enqueue")

    def synchronize(self):
        _lib.check(self.lib.cats_gpu_llm_synchronize(self.h), "synchronize")

    @property
    def stream(self):
        return self.lib.cats_gpu_llm_stream(self.h)

    def logits(self):
        out = np.zeros(self.cfg.vocab, dtype=np.float32)
        _lib.check(self.lib.cats_gpu_llm_logits(self.h, C.c_void_p(out.ctypes.data)), "logits")
        return out

    def next_token(self):
        return self.lib.cats_gpu_llm_next_token(self.h)

    def weight_bytes(self):
        return self.lib.cats_gpu_llm_weight_bytes(self.h)

    def time_matvec(self, kind, reps=3):
        """(ms per launch, algorithmic bytes per launch) of one matvec kind:
        0 qkv, 1 wo, 2 w13, 3 w2, 4 classifier."""
        ms, by = C.c_float(), C.c_double()
        _lib.check(self.lib.cats_gpu_llm_time_matvec(self.h, kind, reps, C.byref(ms), C.byref(by)), "time_matvec")
        return ms.value, by.value

    def trace_step(self, token, pos, per_cta=1024):
        """One traced step of the persistent engine: ([ctas][per_cta] globaltimer
        ns, [ctas][per_cta] SM clock64) stamps."""
        buf = np.zeros(2 * 148 * per_cta, dtype=np.uint64)
        ctas = C.c_int()
        _lib.check(self.lib.cats_gpu_llm_trace_step(self.h, token, pos, C.c_void_p(buf.ctypes.data), per_cta,
                                                    C.byref(ctas)), "trace_step")
        n = ctas.value * per_cta
        return buf[:n].reshape(ctas.value, per_cta), buf[n:2 * n].reshape(ctas.value, per_cta)

    def close(self):
        if self.h:
            self.lib.cats_gpu_llm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def synth_tensor(t, n, d, seed, tensor_id, std=0.02, constant=0.0):
    """The device generator's tensor `tensor_id` in GGUF layout (host bytes)."""
    lib = _lib.init()
    rb = {F32: n * 4, Q4_0: n // 32 * 18, Q8_0: n // 32 * 34}[t]
    out = np.zeros(rb * d, dtype=np.uint8)
    _lib.check(lib.cats_gpu_synth_tensor(C.c_void_p(out.ctypes.data), t, n, d, seed, tensor_id, std, constant),
               "synth_tensor")
    return out


# tensor ids of the device generator (csrc/llm.cu)
T_EMB, T_RMS_ATT, T_RMS_FFN, T_RMS_FINAL, T_WCLS, T_LAYER0 = 0, 1, 2, 3, 4, 16


def layer_tensor_id(layer, k):
    """k: 0 wq, 1 wk, 2 wv, 3 wo, 4 w1, 5 w2, 6 w3."""
    return T_LAYER0 + layer * 8 + k


def _framework_nccl_first():
    """The library opens NCCL at first use and takes a libnccl.so.2 that is
    already loaded; importing torch first makes that torch's own copy, so the
    process holds one NCCL."""
    import torch  # noqa: F401


def tp_unique_id():
    """A fresh NCCL unique id for a tensor-parallel model (bytes)."""
    _framework_nccl_first()
    lib = _lib.init()
    n = lib.cats_gpu_tp_unique_id_bytes()
    buf = C.create_string_buffer(n)
    _lib.check(lib.cats_gpu_tp_unique_id(buf, n), "tp_unique_id")
    return buf.raw


def tp_share_id(group=None, make_id=tp_unique_id):
    """Rank 0 of the torch.distributed group makes the unique id, every rank
    gets the same bytes back (broadcast over the group's backend, gloo or nccl)."""
    import torch.distributed as dist
    box = [make_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    return box[0]
