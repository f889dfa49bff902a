"""Host mirror of catseye's hot-path operator interface over libcatsgpu.

The names and argument meanings follow the reference:
  matmul(xout, x, w, n, d)         llm/catseye_llm.h:1519-1533 (gguf_matmul[] :2583)
  matmul_f32act(...)               matmul_q4_0 (fp32 x, quantize_null), :880-914
  quantize(q, x, n)                quantize_q8, :155-225; quantize_q8_K :262-296
  dequantize(y, w, row, n)         _dequantize_q4_0, :483-486; Q3_K / Q6_K :349-426
  sgemm(ta, tb, m, n, k, ...)      sgemm_ocl, sgemm_ocl2.h:208 / gemm_rnn|rnt|rtn, catseye.h:78-129
Inputs are numpy arrays (host memory, copied per call like the reference's
GPU backends) or torch CUDA tensors for the device-pointer forms.
"""
import ctypes as C

import numpy as np

from . import _lib

F32, Q4_0, Q8_0, Q3_K, Q6_K = 0, 2, 8, 11, 14

# the type-indexed tables of the reference (gguf_matmul / gguf_quantize / gguf_dequantize)
_MATMUL = {F32: "cats_gpu_matmul_f32", Q4_0: "cats_gpu_matmul_q4_0_q8", Q8_0: "cats_gpu_matmul_q8_0_q8",
           Q3_K: "cats_gpu_matmul_q3_K_q8_K", Q6_K: "cats_gpu_matmul_q6_K_q8_K"}
_MATMUL_F32ACT = {Q4_0: "cats_gpu_matmul_q4_0_f32", Q8_0: "cats_gpu_matmul_q8_0_f32"}
_DEQUANT = {Q4_0: "cats_gpu_dequantize_q4_0", Q8_0: "cats_gpu_dequantize_q8_0", Q3_K: "cats_gpu_dequantize_q3_K",
            Q6_K: "cats_gpu_dequantize_q6_K"}


def row_bytes(t, n):
    return {F32: n * 4, Q4_0: n // 32 * 18, Q8_0: n // 32 * 34, Q3_K: n // 256 * 110, Q6_K: n // 256 * 210}[t]


def _p(a):
    return C.c_void_p(a.ctypes.data)


def _dp(t):
    return C.c_void_p(t.data_ptr())


def register_weight(w, t, n, d):
    """Upload a weight (bytes of [d][n] in GGUF layout) before its first matmul."""
    lib = _lib.init()
    _lib.check(lib.cats_gpu_register_weight(_p(w), t, n, d), "register_weight")


def unregister_weight(w):
    _lib.init().cats_gpu_unregister_weight(_p(w))


def matmul(t, xout, x, w, n, d):
    """xout[:d] = W x; x is fp32 (F32), Q8 blocks (Q4_0, Q8_0) or Q8_K blocks
    (Q3_K, Q6_K) as quantize() / quantize_q8_K() made them."""
    lib = _lib.init()
    _lib.call_void(getattr(lib, _MATMUL[t]), _p(xout), _p(x), _p(w), n, d, what=_MATMUL[t])
    return xout


def matmul_f32act(t, xout, x, w, n, d):
    """xout[:d] = W x with fp32 x against Q4_0 / Q8_0 weights (matmul_q4_0)."""
    lib = _lib.init()
    x = np.ascontiguousarray(x, dtype=np.float32)
    _lib.call_void(getattr(lib, _MATMUL_F32ACT[t]), _p(xout), _p(x), _p(w), n, d, what=_MATMUL_F32ACT[t])
    return xout


def quantize_q8_K(x):
    """quantize_q8_K of fp32 x -> n/256 blocks of 260 bytes (int8 array)."""
    lib = _lib.init()
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.zeros(x.size // 256 * 260, dtype=np.int8)
    _lib.call_void(lib.cats_gpu_quantize_q8_K, _p(q), _p(x), x.size, what="quantize_q8_K")
    return q


def quantize(x):
    """quantize_q8 of fp32 x -> n/32 blocks of 36 bytes (int8 array)."""
    lib = _lib.init()
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.zeros(x.size // 32 * 36, dtype=np.int8)
    _lib.call_void(lib.cats_gpu_quantize_q8, _p(q), _p(x), x.size, what="quantize_q8")
    return q


def dequantize(t, w, row, n):
    lib = _lib.init()
    y = np.zeros(n, dtype=np.float32)
    _lib.call_void(getattr(lib, _DEQUANT[t]), _p(y), _p(np.ascontiguousarray(w)), row, n, what=_DEQUANT[t])
    return y


def matvec_dev(w, out, x, x_is_q8=False, stream=None):
    """Device form: out (cuda tensor, d floats) = W x for a registered weight w (host key)."""
    lib = _lib.init()
    _lib.check(lib.cats_gpu_matvec_dev(_p(w), _dp(out), _dp(x), int(x_is_q8), stream), "matvec_dev")
    return out


def quantize_dev(q, x, scalar_mode=False, stream=None):
    lib = _lib.init()
    _lib.check(lib.cats_gpu_quantize_q8_dev(_dp(q), _dp(x), x.numel(), int(scalar_mode), stream), "quantize_dev")
    return q


def dequantize_dev(t, y, w, n, rows, stream=None):
    lib = _lib.init()
    _lib.check(lib.cats_gpu_dequantize_dev(t, _dp(y), _dp(w), n, rows, stream), "dequantize_dev")
    return y


def sgemm(ta, tb, m, n, k, alpha, a, b, beta, c):
    """C = alpha*op(A)*op(B) + beta*C on host arrays (C updated in place and returned)."""
    lib = _lib.init()
    _lib.call_void(lib.cats_sgemm, ta.encode(), tb.encode(), m, n, k, alpha, _p(np.ascontiguousarray(a, np.float32)),
                   _p(np.ascontiguousarray(b, np.float32)), beta, _p(c), what="cats_sgemm")
    return c


def sgemm_dev(ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc, stream=None):
    lib = _lib.init()
    _lib.check(lib.cats_sgemm_dev(ta.encode(), tb.encode(), m, n, k, alpha, _dp(a), lda, _dp(b), ldb, beta,
                                  _dp(c), ldc, stream), "cats_sgemm_dev")
    return c


# ---------------------------------------------------------------- CNN forward
def conv_out(n, k, pad, stride):
    """Output length of a convolution axis (0 for a geometry the library refuses)."""
    if stride <= 0 or k <= 0 or pad < 0:
        return 0
    return max(0, (n + 2 * pad - k) // stride + 1)


def im2col(im, channels, height, width, kh, kw, ph, pw, sh, sw):
    """im2col (catseye.h:508-532) of one host image -> host [c*kh*kw][oh*ow]."""
    lib = _lib.init()
    col = np.empty(channels * kh * kw * conv_out(height, kh, ph, sh) * conv_out(width, kw, pw, sw), np.float32)
    _lib.call_void(lib.cats_im2col, _p(np.ascontiguousarray(im, np.float32)), channels, height, width, kh, kw, ph,
                   pw, sh, sw, _p(col), what="cats_im2col")
    return col


def conv2d_forward(x, w, batch, ich, h, wd, ch, ksize, pad, stride):
    """Batched convolution forward (CatsEye_convolutional_forward) on host arrays -> z[b][ch][oh*ow]."""
    lib = _lib.init()
    z = np.empty(batch * ch * conv_out(h, ksize, pad, stride) * conv_out(wd, ksize, pad, stride), np.float32)
    _lib.call_void(lib.cats_conv2d_forward, _p(np.ascontiguousarray(x, np.float32)),
                   _p(np.ascontiguousarray(w, np.float32)), _p(z), batch, ich, h, wd, ch, ksize, pad, stride,
                   what="cats_conv2d_forward")
    return z


def conv2d_forward_dev(x, w, z, batch, ich, h, wd, ch, ksize, pad, stride, stream=None):
    lib = _lib.init()
    _lib.check(lib.cats_conv2d_forward_dev(_dp(x), _dp(w), _dp(z), batch, ich, h, wd, ch, ksize, pad, stride,
                                           stream), "cats_conv2d_forward_dev")
    return z


def linear_forward(x, w, batch, n_in, n_out):
    """Linear forward (CatsEye_linear_forward): w holds [out][in] weights then out biases."""
    lib = _lib.init()
    z = np.empty(batch * n_out, np.float32)
    _lib.call_void(lib.cats_linear_forward, _p(np.ascontiguousarray(x, np.float32)),
                   _p(np.ascontiguousarray(w, np.float32)), _p(z), batch, n_in, n_out, what="cats_linear_forward")
    return z


def linear_forward_dev(x, w, z, batch, n_in, n_out, stream=None):
    lib = _lib.init()
    _lib.check(lib.cats_linear_forward_dev(_dp(x), _dp(w), _dp(z), batch, n_in, n_out, stream),
               "cats_linear_forward_dev")
    return z


# ------------------------------------------------------------ CNN training
def col2im(col, channels, height, width, kh, kw, ph, pw, sh, sw):
    """col2im (catseye.h:533-556) of one image's columns -> im[c][h][w]."""
    lib = _lib.init()
    im = np.empty(channels * height * width, np.float32)
    _lib.call_void(lib.cats_col2im, _p(np.ascontiguousarray(col, np.float32)), channels, height, width, kh, kw,
                   ph, pw, sh, sw, _p(im), what="cats_col2im")
    return im


def conv2d_backward(dout, w, batch, ich, h, wd, ch, ksize, pad, stride):
    """CatsEye_convolutional_backward for a batch -> dIn[b][ich][h][wd]."""
    lib = _lib.init()
    din = np.empty(batch * ich * h * wd, np.float32)
    _lib.call_void(lib.cats_conv2d_backward, _p(np.ascontiguousarray(dout, np.float32)),
                   _p(np.ascontiguousarray(w, np.float32)), _p(din), batch, ich, h, wd, ch, ksize, pad, stride,
                   what="cats_conv2d_backward")
    return din


def conv2d_update(dout, x, dw, batch, ich, h, wd, ch, ksize, pad, stride):
    """CatsEye_convolutional_update for a batch: dw (updated in place and returned)."""
    lib = _lib.init()
    _lib.call_void(lib.cats_conv2d_update, _p(np.ascontiguousarray(dout, np.float32)),
                   _p(np.ascontiguousarray(x, np.float32)), _p(dw), batch, ich, h, wd, ch, ksize, pad, stride,
                   what="cats_conv2d_update")
    return dw


def linear_backward(dout, w, batch, n_in, n_out):
    """CatsEye_linear_backward -> dIn[b][in]."""
    lib = _lib.init()
    din = np.empty(batch * n_in, np.float32)
    _lib.call_void(lib.cats_linear_backward, _p(np.ascontiguousarray(dout, np.float32)),
                   _p(np.ascontiguousarray(w, np.float32)), _p(din), batch, n_in, n_out, what="cats_linear_backward")
    return din


def linear_update(dout, x, w, dw, batch, n_in, n_out, eta):
    """CatsEye_linear_update: dw += dOut^T x, biases in w -= eta * dOut (w, dw updated in place)."""
    lib = _lib.init()
    _lib.call_void(lib.cats_linear_update, _p(np.ascontiguousarray(dout, np.float32)),
                   _p(np.ascontiguousarray(x, np.float32)), _p(w), _p(dw), batch, n_in, n_out, float(eta),
                   what="cats_linear_update")
    return w, dw


def conv2d_backward_dev(dout, w, din, batch, ich, h, wd, ch, ksize, pad, stride, stream=None):
    lib = _lib.init()
    _lib.check(lib.cats_conv2d_backward_dev(_dp(dout), _dp(w), _dp(din), batch, ich, h, wd, ch, ksize, pad, stride,
                                            stream), "cats_conv2d_backward_dev")
    return din


def conv2d_update_dev(dout, x, dw, batch, ich, h, wd, ch, ksize, pad, stride, stream=None):
    lib = _lib.init()
    _lib.check(lib.cats_conv2d_update_dev(_dp(dout), _dp(x), _dp(dw), batch, ich, h, wd, ch, ksize, pad, stride,
                                          stream), "cats_conv2d_update_dev")
    return dw


# ------------------------------------------------ batched product (tensor cores)
def qgemm(w, x, T, n, d):
    """y[T][d] = x[T][n] * W^T for a registered Q4_0/Q8_0 weight w (host arrays)."""
    lib = _lib.init()
    y = np.empty(T * d, np.float32)
    _lib.check(lib.cats_gpu_qgemm(_p(w), _p(np.ascontiguousarray(x, np.float32)), _p(y), T), "cats_gpu_qgemm")
    return y.reshape(T, d)


def qgemm_dev(w, x, y, T, stream=None):
    lib = _lib.init()
    _lib.check(lib.cats_gpu_qgemm_dev(_p(w), _dp(x), _dp(y), T, stream), "cats_gpu_qgemm_dev")
    return y


def qgemm_plan(w, T):
    """(token tile, K splits, CTAs resident per SM, tensor-map-fed, K slices per split,
    occupancy asked afresh, its CUDA error)."""
    lib = _lib.init()
    plan = np.zeros(7, np.int32)
    _lib.check(lib.cats_gpu_qgemm_plan(_p(w), T, _p(plan)), "cats_gpu_qgemm_plan")
    return tuple(int(v) for v in plan)


def qgemm_trace(w, x, y, T, slices):
    """Runs the product once on device tensors x (T x n) and y (T x d);
    returns CTA (0, 0, 0)'s clock64 stamps, (slices + 1) x 16 (see
    cats_gpu_qgemm_trace)."""
    lib = _lib.init()
    tr = np.zeros((slices + 1) * 16, np.uint64)
    _lib.check(lib.cats_gpu_qgemm_trace(_p(w), _dp(x), _dp(y), T, _p(tr), slices), "cats_gpu_qgemm_trace")
    return tr.reshape(slices + 1, 16)
