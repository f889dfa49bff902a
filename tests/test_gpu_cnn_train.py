"""CNN training callers of the GEMM on the GPU: col2im, convolution backward
(dIn) and update (dw), linear backward and update, against the golden
fixtures recorded from the compiled reference's layers and live against the
reference (oracle/_ref) at the CNN benchmark's layer shapes.

col2im is a gather in the reference's summation order: bit-exact.  The
GEMM-backed layers sum in fp32 in another order than the reference's loops
(one GEMM over the batch instead of one per sample): normwise relative
error <= 1e-5."""
import os

import numpy as np
import pytest

from models import rel

pytestmark = pytest.mark.gpu
TOL = 1e-5
G = os.path.join(os.path.dirname(__file__), "golden", "cnn_train.npz")


@pytest.fixture(scope="module")
def mm(gpu):
    from catseye_b200 import matmul
    return matmul


def test_golden(mm):
    g = np.load(G)
    assert np.array_equal(mm.col2im(g["col2im_col"], 3, 8, 8, 3, 3, 1, 1, 1, 1), g["col2im"])
    for name, (b, ich, h, wd, ch, k, pad, st) in (("s1", (2, 3, 8, 8, 4, 3, 1, 1)), ("s2", (2, 5, 9, 7, 6, 3, 1, 2))):
        p = f"conv_{name}_"
        assert rel(mm.conv2d_backward(g[p + "dout"], g[p + "w"], b, ich, h, wd, ch, k, pad, st), g[p + "din"]) < TOL
        dw = g[p + "dw0"].copy()
        assert rel(mm.conv2d_update(g[p + "dout"], g[p + "x"], dw, b, ich, h, wd, ch, k, pad, st), g[p + "dw"]) < TOL
    assert rel(mm.linear_backward(g["lin_dout"], g["lin_w"], 3, 20, 7), g["lin_din"]) < TOL
    w, dw = g["lin_w"].copy(), g["lin_dw0"].copy()
    mm.linear_update(g["lin_dout"], g["lin_x"], w, dw, 3, 20, 7, 0.01)
    assert rel(w, g["lin_w1"]) < 1e-6 and rel(dw, g["lin_dw"]) < TOL


@pytest.mark.parametrize("c,h,w,kh,kw,ph,pw,sh,sw", [
    (3, 32, 32, 3, 3, 1, 1, 1, 1), (64, 16, 16, 3, 3, 1, 1, 1, 1), (5, 7, 9, 3, 3, 0, 0, 1, 1),
    (4, 11, 13, 5, 3, 2, 1, 2, 1), (2, 8, 8, 1, 1, 0, 0, 1, 1), (3, 9, 9, 3, 3, 1, 1, 2, 2), (2, 10, 10, 4, 4, 1, 1, 3, 3)])
def test_col2im_exact(mm, ref_cnn, c, h, w, kh, kw, ph, pw, sh, sw):
    rng = np.random.default_rng(c * 131 + h * 7 + w + kh)
    hc, wc = (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1
    col = rng.uniform(-1, 1, c * kh * kw * hc * wc).astype(np.float32)
    assert np.array_equal(mm.col2im(col, c, h, w, kh, kw, ph, pw, sh, sw),
                          ref_cnn.col2im(col, c, h, w, kh, kw, ph, pw, sh, sw))


# (batch, ich, h, w, ch, k, pad, stride): the CNN benchmark's four 3x3
# convolutions at batch 8 (the reference's per-sample loops at batch 128
# take minutes), a strided and a 1x1 layer
CONVS = [(8, 3, 32, 32, 64, 3, 1, 1), (8, 64, 32, 32, 64, 3, 1, 1), (8, 64, 16, 16, 128, 3, 1, 1),
         (8, 128, 16, 16, 128, 3, 1, 1), (4, 5, 13, 11, 7, 3, 1, 2), (4, 16, 8, 8, 32, 1, 0, 1)]


@pytest.mark.parametrize("b,ich,h,w,ch,k,pad,st", CONVS)
def test_conv_backward_and_update_against_reference(mm, ref_cnn, b, ich, h, w, ch, k, pad, st):
    rng = np.random.default_rng(b * 1009 + ich * 31 + ch + k)
    oh, ow = (h + 2 * pad - k) // st + 1, (w + 2 * pad - k) // st + 1
    x = rng.uniform(0, 1, b * ich * h * w).astype(np.float32)
    wt = (rng.standard_normal(ch * ich * k * k) * np.sqrt(2 / (ich * k * k))).astype(np.float32)
    dout = rng.uniform(-1, 1, b * ch * oh * ow).astype(np.float32)
    dw0 = rng.uniform(-0.1, 0.1, ch * ich * k * k).astype(np.float32)
    assert rel(mm.conv2d_backward(dout, wt, b, ich, h, w, ch, k, pad, st),
               ref_cnn.conv2d_backward(dout, wt, b, ich, h, w, ch, k, pad, st)) < TOL
    dw = dw0.copy()
    mm.conv2d_update(dout, x, dw, b, ich, h, w, ch, k, pad, st)
    assert rel(dw, ref_cnn.conv2d_update(dout, x, dw0, b, ich, h, w, ch, k, pad, st)) < TOL


@pytest.mark.parametrize("b,n_in,n_out", [(128, 8192, 256), (128, 256, 10), (3, 37, 11), (64, 1000, 333)])
def test_linear_backward_and_update_against_reference(mm, ref_cnn, b, n_in, n_out):
    rng = np.random.default_rng(b + n_in + n_out)
    x = rng.uniform(0, 1, b * n_in).astype(np.float32)
    wt = (rng.standard_normal(n_in * n_out + n_out) * 0.05).astype(np.float32)
    dout = rng.uniform(-1, 1, b * n_out).astype(np.float32)
    dw0 = rng.uniform(-0.1, 0.1, n_in * n_out).astype(np.float32)
    assert rel(mm.linear_backward(dout, wt, b, n_in, n_out), ref_cnn.linear_backward(dout, wt, b, n_in, n_out)) < TOL
    w, dw = wt.copy(), dw0.copy()
    mm.linear_update(dout, x, w, dw, b, n_in, n_out, 0.01)
    w_ref, dw_ref = ref_cnn.linear_update(dout, x, wt, dw0, b, n_in, n_out, 0.01)
    assert rel(dw, dw_ref) < TOL
    assert rel(w[n_in * n_out:], w_ref[n_in * n_out:]) < 1e-6      # the biases
    assert np.array_equal(w[:n_in * n_out], wt[:n_in * n_out])     # the weights themselves are not touched


def test_conv_backward_dev_full_batch_against_oracle(mm, orc):
    """Device pointers at the benchmark's batch of 128 (conv 64->64 on 32x32):
    the whole batch's column matrix (302 MB) in one GEMM, then col2im."""
    import torch
    b, ich, h, w, ch, k, pad, st = 128, 64, 32, 32, 64, 3, 1, 1
    g = torch.Generator(device="cuda").manual_seed(5)
    dout = torch.rand(b * ch * h * w, device="cuda", generator=g) * 2 - 1
    wt = torch.randn(ch * ich * k * k, device="cuda", generator=g) * (2 / (ich * k * k)) ** 0.5
    din = torch.empty(b * ich * h * w, device="cuda")
    mm.conv2d_backward_dev(dout, wt, din, b, ich, h, w, ch, k, pad, st)
    torch.cuda.synchronize()
    # the oracle on 4 samples of the batch (per-sample results are independent)
    sel = [0, 37, 90, 127]
    d = dout.view(b, -1)[sel].cpu().numpy().reshape(-1)
    want = orc.conv2d_backward(d, wt.cpu().numpy(), len(sel), ich, h, w, ch, k, pad, st)
    got = din.view(b, -1)[sel].cpu().numpy().reshape(-1)
    assert rel(got, want) < TOL
