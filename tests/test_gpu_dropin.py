"""The drop-in in place: the reference's own C code, compiled from its
sources, with libcatsgpu bound where a catseye program binds a backend.

* LLM (oracle/_ref/libcatsref_llm_dropin.so): the runtime's dispatch tables
  gguf_matmul[] / gguf_quantize[] / gguf_dequantize[] (llm/catseye_llm.h:
  2583-2607) rebound to cats_gpu_matmul_f32, cats_gpu_matmul_q4_0_q8,
  cats_gpu_quantize_q8 and cats_gpu_dequantize_q4_0 before the model is
  bound; the reference's own cats_llama2_transformer (:1625-1772) then runs
  every matmul on the GPU.  Against the unmodified reference: fp32 <= 1e-4
  with equal greedy tokens; Q4_0 within the Q8 flip amplitude (3e-2): the
  quantizer is bit-exact, but a float-order difference in a matvec sum can
  round one activation code the other way in a later layer.
* CNN (oracle/_ref/libcatsref_cnn_ocl.so): catseye.h's unchanged OpenCL
  backend (sgemm_ocl2.h, built with -DCATS_OPENCL) over include/
  cats_ocl_cuda.h, driving the reference's own CatsEye_convolutional_forward
  / _backward / _update and CatsEye_linear_forward / _backward / _update.
  Against the CPU build of the same layers: normwise <= 1e-5."""
import numpy as np
import pytest

from models import ModelWeights, prompt, rel
from oracle.cpu import F32, Q4_0

pytestmark = pytest.mark.gpu


def _lib(name):
    from oracle.cpu import Reference, ref_available
    if not ref_available(name):
        pytest.skip(f"oracle/_ref/libcatsref_{name}.so not built here")
    return Reference(name)


@pytest.fixture(scope="module")
def dropin(gpu):
    return _lib("llm_dropin")


@pytest.fixture(scope="module")
def cnn_ocl(gpu):
    return _lib("cnn_ocl")


@pytest.mark.parametrize("t,tol", [(F32, 1e-4), (Q4_0, 3e-2)])
def test_reference_transformer_on_gpu_matmuls(dropin, ref_llm, orc, t, tol):
    from catseye_b200.llm import STORIES_F32
    cfg = STORIES_F32.with_type(t)
    mw = ModelWeights(cfg, 21, orc)
    gpu_side, cpu_side = dropin.llm(mw), ref_llm.llm(mw)
    toks = prompt(21, 8, cfg.vocab)
    tok = int(toks[0])
    for pos in range(24):
        lg, lr = gpu_side.step(tok, pos), cpu_side.step(tok, pos)
        assert rel(lg, lr) < tol, (t, pos, rel(lg, lr))
        if t == F32:
            assert int(np.argmax(lg)) == int(np.argmax(lr)), pos
        tok = int(toks[pos + 1]) if pos + 1 < len(toks) else int(np.argmax(lr))


def test_reference_cnn_layers_on_the_opencl_backend_over_the_gpu(cnn_ocl, ref_cnn):
    rng = np.random.default_rng(3)
    for (b, ich, h, w, ch, k, pad, st) in ((4, 3, 32, 32, 64, 3, 1, 1), (4, 64, 16, 16, 128, 3, 1, 1),
                                           (2, 5, 11, 9, 6, 3, 1, 2)):
        oh, ow = (h + 2 * pad - k) // st + 1, (w + 2 * pad - k) // st + 1
        x = rng.uniform(0, 1, b * ich * h * w).astype(np.float32)
        wt = (rng.standard_normal(ch * ich * k * k) * np.sqrt(2 / (ich * k * k))).astype(np.float32)
        dout = rng.uniform(-1, 1, b * ch * oh * ow).astype(np.float32)
        dw0 = rng.uniform(-0.1, 0.1, ch * ich * k * k).astype(np.float32)
        args = (b, ich, h, w, ch, k, pad, st)
        assert rel(cnn_ocl.conv2d_forward(x, wt, *args), ref_cnn.conv2d_forward(x, wt, *args)) < 1e-5
        assert rel(cnn_ocl.conv2d_backward(dout, wt, *args), ref_cnn.conv2d_backward(dout, wt, *args)) < 1e-5
        assert rel(cnn_ocl.conv2d_update(dout, x, dw0, *args), ref_cnn.conv2d_update(dout, x, dw0, *args)) < 1e-5
    for (b, n_in, n_out) in ((16, 8192, 256), (16, 256, 10), (3, 37, 11)):
        x = rng.uniform(0, 1, b * n_in).astype(np.float32)
        wt = (rng.standard_normal(n_in * n_out + n_out) * 0.05).astype(np.float32)
        dout = rng.uniform(-1, 1, b * n_out).astype(np.float32)
        dw0 = rng.uniform(-0.1, 0.1, n_in * n_out).astype(np.float32)
        assert rel(cnn_ocl.linear_forward(x, wt, b, n_in, n_out), ref_cnn.linear_forward(x, wt, b, n_in, n_out)) < 1e-5
        assert rel(cnn_ocl.linear_backward(dout, wt, b, n_in, n_out),
                   ref_cnn.linear_backward(dout, wt, b, n_in, n_out)) < 1e-5
        w1, d1 = cnn_ocl.linear_update(dout, x, wt, dw0, b, n_in, n_out, 0.01)
        w2, d2 = ref_cnn.linear_update(dout, x, wt, dw0, b, n_in, n_out, 0.01)
        assert rel(d1, d2) < 1e-5 and rel(w1, w2) < 1e-6
    # the plain sgemm through the backend: NN, NT, TN with beta 0 and 1
    for ta, tb in (("N", "N"), ("N", "T"), ("T", "N")):
        M, N, K = 300, 200, 500
        A = rng.uniform(-1, 1, M * K).astype(np.float32)
        B = rng.uniform(-1, 1, K * N).astype(np.float32)
        C0 = rng.uniform(-1, 1, M * N).astype(np.float32)
        for beta in (0.0, 1.0):
            assert rel(cnn_ocl.sgemm(ta, tb, M, N, K, 1.0, A, B, beta, C0),
                       ref_cnn.sgemm(ta, tb, M, N, K, 1.0, A, B, beta, C0)) < 1e-5
