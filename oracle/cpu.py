"""ctypes bindings for the C oracle (libcatsoracle.so) and the compiled reference
(oracle/_ref/libcatsref_*.so).  Test infrastructure only.

The oracle restates catseye's algorithms (oracle/cats_oracle.c, each function
cites the reference file:line it follows).  The reference libraries are the
reference's own headers compiled from their sources by oracle/Makefile; they are
used to pin the oracle and as the timed CPU baseline.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

F32, Q4_0, Q8_0, Q3_K, Q6_K = 0, 2, 8, 11, 14

_fp = C.POINTER(C.c_float)
_vp = C.c_void_p


def row_bytes(t, n):
    return {F32: n * 4, Q4_0: n // 32 * 18, Q8_0: n // 32 * 34,
            Q3_K: n // 256 * 110, Q6_K: n // 256 * 210}[t]


def _ptr(a):
    return a.ctypes.data_as(_vp)


def aligned(a, align=256):
    """`a` itself when its address is a multiple of `align` bytes, else a copy
    in such a buffer: the reference allocates everything 256-byte aligned
    (llm/catseye_llm.h:36-46) and its AVX code uses aligned loads."""
    a = np.ascontiguousarray(a)
    if a.ctypes.data % align == 0:
        return a
    raw = np.empty(a.nbytes + align, dtype=np.uint8)
    off = (-raw.ctypes.data) % align
    out = raw[off:off + a.nbytes].view(a.dtype).reshape(a.shape)
    out[...] = a
    return out


def build_oracle():
    """Compile libcatsoracle.so with the system gcc if it is missing."""
    so = os.path.join(HERE, "libcatsoracle.so")
    if not os.path.exists(so):
        subprocess.check_call(["make", "-s", "-C", HERE, "libcatsoracle.so"])
    return so


def ref_available(name="llm"):
    return os.path.exists(os.path.join(REF_DIR, f"libcatsref_{name}.so"))


class _LLMState(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("dim", "hidden", "n_layers", "n_heads", "n_kv_heads",
                                       "vocab", "seq_len", "wtype", "q8_mode")] + \
               [(n, _vp) for n in ("emb", "rms_att", "rms_ffn", "rms_final", "wq", "wk", "wv",
                                   "wo", "w1", "w2", "w3", "wcls")] + \
               [(n, _fp) for n in ("x", "xb", "xb2", "hb", "hb2", "q", "att", "logits",
                                   "key_cache", "value_cache")]


class Oracle:
    """The C restatement.  All arrays are numpy; outputs are returned."""

    def __init__(self):
        self.lib = C.CDLL(build_oracle())
        L = self.lib
        L.oracle_fp16_to_fp32.restype = C.c_float
        L.oracle_fp16_to_fp32.argtypes = [C.c_uint16]
        L.oracle_fp32_to_fp16.restype = C.c_uint16
        L.oracle_fp32_to_fp16.argtypes = [C.c_float]
        L.oracle_llm_step.restype = _fp
        L.oracle_argmax.argtypes = [_vp, C.c_int]
        L.oracle_sgemm.argtypes = [C.c_char, C.c_char, C.c_int, C.c_int, C.c_int, C.c_float,
                                   _vp, _vp, C.c_float, _vp]
        for fn in ("oracle_quantize_q8_avx", "oracle_quantize_q8_scalar", "oracle_quantize_q8_K",
                   "oracle_quantize_row_q4_0", "oracle_quantize_row_q8_0"):
            getattr(L, fn).argtypes = [_vp, _vp, C.c_int]
        L.oracle_dequantize_row.argtypes = [C.c_int, _vp, _vp, C.c_int]
        L.oracle_matmul.argtypes = [C.c_int, _vp, _vp, _vp, C.c_int, C.c_int]
        for fn in ("oracle_matmul_f32", "oracle_matmul_q4_0_q8", "oracle_matmul_q8_0_q8",
                   "oracle_matmul_q4_0_f32", "oracle_matmul_q3_K_q8_K", "oracle_matmul_q6_K_q8_K"):
            getattr(L, fn).argtypes = [_vp, _vp, _vp, C.c_int, C.c_int]
        L.oracle_im2col.argtypes = [_vp] + [C.c_int] * 9 + [_vp]
        L.oracle_conv2d_forward.argtypes = [_vp, _vp, _vp] + [C.c_int] * 8
        L.oracle_linear_forward.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int]
        L.oracle_col2im.argtypes = [_vp] + [C.c_int] * 9 + [_vp]
        L.oracle_conv2d_backward.argtypes = [_vp, _vp, _vp] + [C.c_int] * 8
        L.oracle_conv2d_update.argtypes = [_vp, _vp, _vp] + [C.c_int] * 8
        L.oracle_linear_backward.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int]
        L.oracle_linear_update.argtypes = [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_float]

    # --- conversions / quantizers -------------------------------------------
    def fp16_to_fp32(self, h):
        return self.lib.oracle_fp16_to_fp32(int(h))

    def fp32_to_fp16(self, f):
        return self.lib.oracle_fp32_to_fp16(float(f))

    def quantize_q8(self, x, mode="avx"):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q = np.zeros(x.size // 32 * 36, dtype=np.int8)
        fn = self.lib.oracle_quantize_q8_avx if mode == "avx" else self.lib.oracle_quantize_q8_scalar
        fn(_ptr(q), _ptr(x), x.size)
        return q

    def quantize_q8_K(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q = np.zeros(x.size // 256 * 260, dtype=np.int8)
        self.lib.oracle_quantize_q8_K(_ptr(q), _ptr(x), x.size)
        return q

    def quantize_rows(self, t, w):
        """Quantize a float matrix [d][n] into GGUF blocks of type t (bytes, [d][row_bytes])."""
        w = np.ascontiguousarray(w, dtype=np.float32)
        d, n = w.shape
        if t == F32:
            return w.view(np.uint8).reshape(d, n * 4).copy()
        out = np.zeros((d, row_bytes(t, n)), dtype=np.uint8)
        fn = self.lib.oracle_quantize_row_q4_0 if t == Q4_0 else self.lib.oracle_quantize_row_q8_0
        fn(_ptr(out), _ptr(w), d * n)   # rows are whole blocks, so one call covers the matrix
        return out

    def dequantize(self, t, wbytes, n, rows=1):
        wbytes = np.ascontiguousarray(wbytes).view(np.uint8)
        y = np.zeros(rows * n, dtype=np.float32)
        self.lib.oracle_dequantize_row(t, _ptr(y), _ptr(wbytes), rows * n)
        return y.reshape(rows, n)

    # --- matvecs ------------------------------------------------------------
    def matmul(self, t, x, w, n, d):
        """matmul as the runtime calls it: quantize x (AVX rounding) then W x."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w)
        out = np.zeros(d, dtype=np.float32)
        self.lib.oracle_matmul(t, _ptr(out), _ptr(x), _ptr(w), n, d)
        return out

    def matmul_prequant(self, fn, xq, w, n, d):
        out = np.zeros(d, dtype=np.float32)
        getattr(self.lib, fn)(_ptr(out), _ptr(np.ascontiguousarray(xq)), _ptr(np.ascontiguousarray(w)), n, d)
        return out

    def sgemm(self, ta, tb, M, N, K, alpha, A, B, beta, C0):
        Cm = np.array(C0, dtype=np.float32, copy=True)
        self.lib.oracle_sgemm(ta.encode(), tb.encode(), M, N, K, alpha, _ptr(np.ascontiguousarray(A, np.float32)),
                              _ptr(np.ascontiguousarray(B, np.float32)), beta, _ptr(Cm))
        return Cm

    def im2col(self, im, c, h, w, kh, kw, ph, pw, sh, sw):
        hc, wc = (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1
        col = np.zeros(c * kh * kw * hc * wc, dtype=np.float32)
        self.lib.oracle_im2col(_ptr(np.ascontiguousarray(im, np.float32)), c, h, w, kh, kw, ph, pw, sh, sw, _ptr(col))
        return col

    def conv2d_forward(self, x, w, batch, ich, h, wd, ch, k, pad, stride):
        oh, ow = (h + 2 * pad - k) // stride + 1, (wd + 2 * pad - k) // stride + 1
        z = np.zeros(batch * ch * oh * ow, dtype=np.float32)
        self.lib.oracle_conv2d_forward(_ptr(np.ascontiguousarray(x, np.float32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                       _ptr(z), batch, ich, h, wd, ch, k, pad, stride)
        return z

    def linear_forward(self, x, w, batch, n_in, n_out):
        z = np.zeros(batch * n_out, dtype=np.float32)
        self.lib.oracle_linear_forward(_ptr(np.ascontiguousarray(x, np.float32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                       _ptr(z), batch, n_in, n_out)
        return z

    # --- CNN training layers (catseye.h:445-505, 533-556, 589-640) ------------
    def col2im(self, col, c, h, w, kh, kw, ph, pw, sh, sw):
        im = np.zeros(c * h * w, dtype=np.float32)
        self.lib.oracle_col2im(_ptr(np.ascontiguousarray(col, np.float32)), c, h, w, kh, kw, ph, pw, sh, sw, _ptr(im))
        return im

    def conv2d_backward(self, dout, w, batch, ich, h, wd, ch, k, pad, stride):
        din = np.zeros(batch * ich * h * wd, dtype=np.float32)
        self.lib.oracle_conv2d_backward(_ptr(np.ascontiguousarray(dout, np.float32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                    _ptr(din), batch, ich, h, wd, ch, k, pad, stride)
        return din

    def conv2d_update(self, dout, x, dw0, batch, ich, h, wd, ch, k, pad, stride):
        dw = np.array(dw0, dtype=np.float32, copy=True)
        self.lib.oracle_conv2d_update(_ptr(np.ascontiguousarray(dout, np.float32)), _ptr(np.ascontiguousarray(x, np.float32)),
                                  _ptr(dw), batch, ich, h, wd, ch, k, pad, stride)
        return dw

    def linear_backward(self, dout, w, batch, n_in, n_out):
        din = np.zeros(batch * n_in, dtype=np.float32)
        self.lib.oracle_linear_backward(_ptr(np.ascontiguousarray(dout, np.float32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                    _ptr(din), batch, n_in, n_out)
        return din

    def linear_update(self, dout, x, w0, dw0, batch, n_in, n_out, eta):
        w = np.array(w0, dtype=np.float32, copy=True)
        dw = np.array(dw0, dtype=np.float32, copy=True)
        self.lib.oracle_linear_update(_ptr(np.ascontiguousarray(dout, np.float32)), _ptr(np.ascontiguousarray(x, np.float32)),
                                  _ptr(w), _ptr(dw), batch, n_in, n_out, float(eta))
        return w, dw

    def argmax(self, v):
        v = np.ascontiguousarray(v, np.float32)
        return self.lib.oracle_argmax(_ptr(v), v.size)

    # --- decode step ----------------------------------------------------------
    def llm(self, model, q8_mode=0):
        """q8_mode 0/1: quantize_q8 with the AVX / plain-C rounding before each
        quantized matmul; 2: fp32 activations (matmul_q4_0 and its Q8_0 form)."""
        return OracleLLM(self, model, q8_mode)


class OracleLLM:
    """cats_llama2_transformer restated; `model` is a catseye_b200.llm.ModelWeights."""

    def __init__(self, orc, mw, q8_mode=0):
        self.orc, self.mw = orc, mw
        c = mw.cfg
        s = _LLMState()
        s.dim, s.hidden, s.n_layers, s.n_heads = c.dim, c.hidden, c.n_layers, c.n_heads
        s.n_kv_heads, s.vocab, s.seq_len, s.wtype, s.q8_mode = c.n_kv_heads, c.vocab, c.seq_len, c.wtype, q8_mode
        for name in ("emb", "rms_att", "rms_ffn", "rms_final", "wq", "wk", "wv", "wo", "w1", "w2", "w3", "wcls"):
            setattr(s, name, _ptr(getattr(mw, name)))
        self.s = s
        self.lib = orc.lib
        self.lib.oracle_llm_alloc.argtypes = [C.POINTER(_LLMState)]
        self.lib.oracle_llm_step.argtypes = [C.POINTER(_LLMState), C.c_int, C.c_int]
        self.lib.oracle_llm_free.argtypes = [C.POINTER(_LLMState)]
        if self.lib.oracle_llm_alloc(C.byref(s)) != 0:
            raise MemoryError("oracle_llm_alloc")

    def step(self, token, pos):
        p = self.lib.oracle_llm_step(C.byref(self.s), token, pos)
        return np.ctypeslib.as_array(p, shape=(self.mw.cfg.vocab,)).copy()

    def __del__(self):
        try:
            self.lib.oracle_llm_free(C.byref(self.s))
        except Exception:
            pass


class Reference:
    """The reference's own functions compiled from its headers (oracle/_ref)."""

    def __init__(self, name="llm"):
        path = os.path.join(REF_DIR, f"libcatsref_{name}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.name = name
        self.lib = L = C.CDLL(path)
        if name.startswith("llm"):
            L.ref_fp16_to_fp32.restype = C.c_float
            L.ref_fp16_to_fp32.argtypes = [C.c_uint16]
            L.ref_fp32_to_fp16.restype = C.c_uint16
            L.ref_fp32_to_fp16.argtypes = [C.c_float]
            L.ref_quantize_q8.argtypes = [_vp, _vp, C.c_int]
            L.ref_quantize_q8_K.argtypes = [_vp, _vp, C.c_int]
            L.ref_dequantize.argtypes = [C.c_int, _vp, _vp, C.c_int, C.c_int]
            L.ref_matmul.argtypes = [C.c_int, _vp, _vp, _vp, C.c_int, C.c_int]
            L.ref_sample_argmax.argtypes = [_vp, C.c_int]
            L.ref_llm_create.restype = _vp
            L.ref_llm_create.argtypes = [C.c_int] * 8 + [_vp] * 12
            L.ref_llm_step.restype = _fp
            L.ref_llm_step.argtypes = [_vp, C.c_int, C.c_int]
            L.ref_llm_destroy.argtypes = [_vp]
            if hasattr(L, "ref_llm_use_f32_activations"):   # AVX builds only (matmul_q4_0)
                L.ref_llm_use_f32_activations.argtypes = [_vp]
            if hasattr(L, "ref_llm_use_q8_activations"):
                L.ref_llm_use_q8_activations.argtypes = [_vp]
            if hasattr(L, "ref_llm_dropin_tables"):   # libcatsgpu dropped into the reference runtime
                L.ref_llm_dropin_tables.argtypes = []
                L.ref_llm_dropin_tables()
            if hasattr(L, "ref_llm_load"):
                L.ref_llm_load.restype = _vp
                L.ref_llm_load.argtypes = [C.c_char_p, C.c_int, _vp]
        else:
            L.ref_sgemm.argtypes = [C.c_char, C.c_char, C.c_int, C.c_int, C.c_int, C.c_float,
                                    _vp, _vp, C.c_float, _vp]
            L.ref_im2col.argtypes = [_vp] + [C.c_int] * 9 + [_vp]
            L.ref_conv2d_forward.argtypes = [_vp, _vp, _vp] + [C.c_int] * 8
            L.ref_linear_forward.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int]
            L.ref_col2im.argtypes = [_vp] + [C.c_int] * 9 + [_vp]
            L.ref_conv2d_backward.argtypes = [_vp, _vp, _vp] + [C.c_int] * 8
            L.ref_conv2d_update.argtypes = [_vp, _vp, _vp] + [C.c_int] * 8 + [_vp]
            L.ref_linear_backward.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int]
            L.ref_linear_update.argtypes = [_vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_float]
            if hasattr(L, "ref_cnn_init"):   # the OpenCL backend over libcatsgpu: sgemm_init first
                L.ref_cnn_init.argtypes = []
                L.ref_cnn_init()

    def is_avx(self):
        return bool(self.lib.ref_is_avx())

    def quantize_q8(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q = np.zeros(x.size // 32 * 36, dtype=np.int8)
        self.lib.ref_quantize_q8(_ptr(q), _ptr(x), x.size)
        return q

    def quantize_q8_K(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).copy()
        q = np.zeros(x.size // 256 * 260, dtype=np.int8)
        self.lib.ref_quantize_q8_K(_ptr(q), _ptr(x), x.size)
        return q

    def dequantize(self, t, wbytes, row, n):
        y = np.zeros(n, dtype=np.float32)
        y = aligned(y)
        self.lib.ref_dequantize(t, _ptr(y), _ptr(aligned(wbytes)), row, n)
        return y

    def matmul_raw(self, t, xq, w, n, d):
        out = np.zeros(d, dtype=np.float32)
        out = aligned(out)
        self.lib.ref_matmul(t, _ptr(out), _ptr(aligned(xq)), _ptr(aligned(w)), n, d)
        return out

    def matmul(self, t, x, w, n, d):
        """quantize (the tensor's quantizer) then matmul, as the runtime does."""
        if t == F32:
            return self.matmul_raw(t, np.ascontiguousarray(x, np.float32), w, n, d)
        if t in (Q3_K, Q6_K):
            return self.matmul_raw(t, self.quantize_q8_K(x), w, n, d)
        return self.matmul_raw(t, self.quantize_q8(x), w, n, d)

    # --- CNN training layers (catseye.h:445-505, 533-556, 589-640) ------------
    def col2im(self, col, c, h, w, kh, kw, ph, pw, sh, sw):
        im = np.zeros(c * h * w, dtype=np.float32)
        self.lib.ref_col2im(_ptr(np.ascontiguousarray(col, np.float32)), c, h, w, kh, kw, ph, pw, sh, sw, _ptr(im))
        return im

    def conv2d_backward(self, dout, w, batch, ich, h, wd, ch, k, pad, stride):
        din = np.zeros(batch * ich * h * wd, dtype=np.float32)
        self.lib.ref_conv2d_backward(_ptr(np.ascontiguousarray(dout, np.float32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                    _ptr(din), batch, ich, h, wd, ch, k, pad, stride)
        return din

    def conv2d_update(self, dout, x, dw0, batch, ich, h, wd, ch, k, pad, stride):
        dw = np.array(dw0, dtype=np.float32, copy=True)
        self.lib.ref_conv2d_update(_ptr(np.ascontiguousarray(dout, np.float32)), _ptr(np.ascontiguousarray(x, np.float32)),
                                  _ptr(dw), batch, ich, h, wd, ch, k, pad, stride, _ptr(np.zeros(ch * ich * k * k, np.float32)))
        return dw

    def linear_backward(self, dout, w, batch, n_in, n_out):
        din = np.zeros(batch * n_in, dtype=np.float32)
        self.lib.ref_linear_backward(_ptr(np.ascontiguousarray(dout, np.float32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                    _ptr(din), batch, n_in, n_out)
        return din

    def linear_update(self, dout, x, w0, dw0, batch, n_in, n_out, eta):
        w = np.array(w0, dtype=np.float32, copy=True)
        dw = np.array(dw0, dtype=np.float32, copy=True)
        self.lib.ref_linear_update(_ptr(np.ascontiguousarray(dout, np.float32)), _ptr(np.ascontiguousarray(x, np.float32)),
                                  _ptr(w), _ptr(dw), batch, n_in, n_out, float(eta))
        return w, dw

    def argmax(self, v):
        v = np.ascontiguousarray(v, np.float32)
        return self.lib.ref_sample_argmax(_ptr(v), v.size)

    def sgemm(self, ta, tb, M, N, K, alpha, A, B, beta, C0):
        Cm = np.array(C0, dtype=np.float32, copy=True)
        self.lib.ref_sgemm(ta.encode(), tb.encode(), M, N, K, alpha, _ptr(np.ascontiguousarray(A, np.float32)),
                           _ptr(np.ascontiguousarray(B, np.float32)), beta, _ptr(Cm))
        return Cm

    def im2col(self, im, c, h, w, kh, kw, ph, pw, sh, sw):
        hc, wc = (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1
        col = np.zeros(c * kh * kw * hc * wc, dtype=np.float32)
        self.lib.ref_im2col(_ptr(np.ascontiguousarray(im, np.float32)), c, h, w, kh, kw, ph, pw, sh, sw, _ptr(col))
        return col

    def conv2d_forward(self, x, w, batch, ich, h, wd, ch, k, pad, stride):
        oh, ow = (h + 2 * pad - k) // stride + 1, (wd + 2 * pad - k) // stride + 1
        z = np.zeros(batch * ch * oh * ow, dtype=np.float32)
        self.lib.ref_conv2d_forward(_ptr(np.ascontiguousarray(x, np.float32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                    _ptr(z), batch, ich, h, wd, ch, k, pad, stride)
        return z

    def linear_forward(self, x, w, batch, n_in, n_out):
        z = np.zeros(batch * n_out, dtype=np.float32)
        self.lib.ref_linear_forward(_ptr(np.ascontiguousarray(x, np.float32)), _ptr(np.ascontiguousarray(w, np.float32)),
                                    _ptr(z), batch, n_in, n_out)
        return z

    def llm(self, mw, f32_act=False):
        return RefLLM(self, mw, f32_act)

    def load(self, path, fmt):
        """The reference's own loader on a model file (fmt 1 GGUF, 2 ggjt, 3
        llama2.c .bin): (a stepper, [dim, hidden, layers, heads, kv_heads,
        vocab, seq_len])."""
        hp = np.zeros(7, np.int32)
        h = self.lib.ref_llm_load(str(path).encode(), fmt, _ptr(hp))
        if not h:
            raise ValueError(f"the reference's loader refused {path}")
        return RefLoaded(self, h, int(hp[5])), [int(v) for v in hp]


class RefLLM:
    """cats_llama2_transformer itself, on a model bound to the given weight blobs.
    f32_act: Q4_0 tensors bound to matmul_q4_0 with quantize_null (fp32 activations)."""

    def __init__(self, ref, mw, f32_act=False):
        c = mw.cfg
        self.ref, self.mw = ref, mw
        # the reference's AVX matvecs use aligned loads: give it 256-byte aligned copies
        self._blobs = [aligned(getattr(mw, n)) for n in ("emb", "rms_att", "rms_ffn", "rms_final", "wq", "wk",
                                                          "wv", "wo", "w1", "w2", "w3", "wcls")]
        self.h = ref.lib.ref_llm_create(c.dim, c.hidden, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab,
                                        c.seq_len, c.wtype, *[_ptr(b) for b in self._blobs])
        if not self.h:
            raise ValueError(f"reference has no matmul for weight type {c.wtype}")
        if f32_act:
            if not hasattr(ref.lib, "ref_llm_use_f32_activations"):
                raise ValueError("this reference build has no matmul_q4_0 (AVX builds only)")
            ref.lib.ref_llm_use_f32_activations(self.h)

    def use_q8_activations(self):
        """Rebind the Q4_0 tensors to the default quantize_q8 + matmul_q4_0_q8
        (after a prompt went through the fp32-activation binding)."""
        self.ref.lib.ref_llm_use_q8_activations(self.h)

    def step(self, token, pos):
        p = self.ref.lib.ref_llm_step(self.h, token, pos)
        return np.ctypeslib.as_array(p, shape=(self.mw.cfg.vocab,)).copy()

    def __del__(self):
        try:
            self.ref.lib.ref_llm_destroy(self.h)
        except Exception:
            pass


class RefLoaded:
    """cats_llama2_transformer on a model the reference's own loader read."""

    def __init__(self, ref, h, vocab):
        self.ref, self.h, self.vocab = ref, h, vocab

    def step(self, token, pos):
        p = self.ref.lib.ref_llm_step(self.h, token, pos)
        return np.ctypeslib.as_array(p, shape=(self.vocab,)).copy()
