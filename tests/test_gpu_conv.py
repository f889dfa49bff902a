"""CNN forward callers of the GEMM on the GPU (im2col, batched convolution
forward as one implicit GEMM, linear forward) against the golden fixtures
recorded from the compiled reference and against the oracle.

im2col is a copy: bit-exact.  Convolution and linear outputs are fp32 sums
in a different order than the reference's loops: normwise relative error
<= 1e-5."""
import os

import numpy as np
import pytest

from models import rel

pytestmark = pytest.mark.gpu
TOL = 1e-5
G = os.path.join(os.path.dirname(__file__), "golden", "cnn.npz")


@pytest.fixture(scope="module")
def mm(gpu):
    from catseye_b200 import matmul
    return matmul


def test_golden(mm):
    g = np.load(G)
    assert np.array_equal(mm.im2col(g["im2col_x"], 3, 8, 8, 3, 3, 1, 1, 1, 1), g["im2col"])
    assert rel(mm.conv2d_forward(g["conv_x"], g["conv_w"], 2, 3, 8, 8, 4, 3, 1, 1), g["conv_z"]) < TOL
    assert rel(mm.linear_forward(g["lin_x"], g["lin_w"], 3, 20, 7), g["lin_z"]) < TOL


@pytest.mark.parametrize("c,h,w,kh,kw,ph,pw,sh,sw", [
    (3, 32, 32, 3, 3, 1, 1, 1, 1), (64, 16, 16, 3, 3, 1, 1, 1, 1), (5, 7, 9, 3, 3, 0, 0, 1, 1),
    (4, 11, 13, 5, 3, 2, 1, 2, 1), (2, 8, 8, 1, 1, 0, 0, 1, 1), (3, 9, 9, 3, 3, 1, 1, 2, 2)])
def test_im2col_exact(mm, orc, c, h, w, kh, kw, ph, pw, sh, sw):
    rng = np.random.default_rng(c * 131 + h * 7 + w)
    im = rng.uniform(0, 1, c * h * w).astype(np.float32)
    assert np.array_equal(mm.im2col(im, c, h, w, kh, kw, ph, pw, sh, sw),
                          orc.im2col(im, c, h, w, kh, kw, ph, pw, sh, sw))


# (batch, ich, h, w, ch, ksize, pad, stride): the four convolutions of the
# 32x32x3 CNN at batch 4, then strides, no padding, 1x1, 5x5, odd sizes and
# channel counts that need two 128-row tiles or a ragged one
CONVS = [(4, 3, 32, 32, 64, 3, 1, 1), (4, 64, 32, 32, 64, 3, 1, 1), (4, 64, 16, 16, 128, 3, 1, 1),
         (4, 128, 16, 16, 128, 3, 1, 1), (3, 8, 15, 17, 24, 3, 1, 2), (2, 6, 12, 10, 40, 3, 0, 1),
         (5, 16, 9, 9, 32, 1, 0, 1), (2, 5, 13, 11, 20, 5, 2, 1), (3, 7, 10, 10, 200, 3, 1, 1),
         (1, 1, 1, 1, 1, 1, 0, 1), (7, 3, 5, 5, 96, 3, 1, 1),
         # tensor-core (3xTF32) shapes: ch * N * K >= 2^24 with K a multiple of 4.  A
         # 256-channel tile with 200 channels, stride 2 without padding and 96
         # channels, 5x5 with 128-pixel tiles that straddle samples (oh * ow = 900),
         # odd image sizes (255 pixels per sample), 1x1, and K = 99 and 117 (weight
         # rows not 16-byte aligned: scalar weight loads)
         (8, 32, 12, 12, 200, 3, 1, 1), (16, 16, 33, 33, 96, 3, 0, 2), (8, 4, 30, 30, 64, 5, 2, 1),
         (8, 20, 15, 17, 48, 3, 1, 1), (16, 64, 16, 16, 128, 1, 0, 1), (16, 11, 20, 20, 40, 3, 1, 1),
         (8, 13, 24, 24, 72, 3, 1, 1)]


@pytest.mark.parametrize("batch,ich,h,w,ch,ks,pad,stride", CONVS)
def test_conv2d_forward(mm, orc, batch, ich, h, w, ch, ks, pad, stride):
    rng = np.random.default_rng(batch * 1009 + ich * 31 + ch)
    x = rng.uniform(0, 1, batch * ich * h * w).astype(np.float32)
    wt = (rng.standard_normal(ch * ich * ks * ks) * np.sqrt(2.0 / (ich * ks * ks))).astype(np.float32)
    z = mm.conv2d_forward(x, wt, batch, ich, h, w, ch, ks, pad, stride)
    assert rel(z, orc.conv2d_forward(x, wt, batch, ich, h, w, ch, ks, pad, stride)) < TOL


def test_conv2d_forward_reference_full_batch(mm, ref_cnn):
    """The CNN's second convolution (64 -> 64 channels, 32x32) at batch 16
    against the compiled reference (per-sample im2col + gemm_rnn)."""
    rng = np.random.default_rng(11)
    x = rng.uniform(0, 1, 16 * 64 * 32 * 32).astype(np.float32)
    wt = (rng.standard_normal(64 * 576) * np.sqrt(2.0 / 576)).astype(np.float32)
    z = mm.conv2d_forward(x, wt, 16, 64, 32, 32, 64, 3, 1, 1)
    assert rel(z, ref_cnn.conv2d_forward(x, wt, 16, 64, 32, 32, 64, 3, 1, 1)) < TOL


@pytest.mark.parametrize("batch,n_in,n_out", [(128, 8192, 256), (128, 256, 10), (3, 20, 7), (1, 1, 1),
                                              (33, 100, 65)])
def test_linear_forward(mm, orc, batch, n_in, n_out):
    rng = np.random.default_rng(batch + n_in + n_out)
    x = rng.uniform(-1, 1, batch * n_in).astype(np.float32)
    w = rng.uniform(-0.1, 0.1, n_in * n_out + n_out).astype(np.float32)
    assert rel(mm.linear_forward(x, w, batch, n_in, n_out), orc.linear_forward(x, w, batch, n_in, n_out)) < TOL


def test_device_forms_match_host_forms(mm, orc):
    import torch
    rng = np.random.default_rng(5)
    x = rng.uniform(0, 1, 2 * 3 * 10 * 10).astype(np.float32)
    wt = rng.standard_normal(16 * 27).astype(np.float32)
    dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda()
    dz = torch.empty(2 * 16 * 100, device="cuda")
    mm.conv2d_forward_dev(dx, dw, dz, 2, 3, 10, 10, 16, 3, 1, 1)
    torch.cuda.synchronize()
    assert rel(dz.cpu().numpy(), orc.conv2d_forward(x, wt, 2, 3, 10, 10, 16, 3, 1, 1)) < TOL
    xl = rng.uniform(-1, 1, 4 * 30).astype(np.float32)
    wl = rng.uniform(-1, 1, 30 * 9 + 9).astype(np.float32)
    dzl = torch.empty(4 * 9, device="cuda")
    mm.linear_forward_dev(torch.from_numpy(xl).cuda(), torch.from_numpy(wl).cuda(), dzl, 4, 30, 9)
    torch.cuda.synchronize()
    assert rel(dzl.cpu().numpy(), orc.linear_forward(xl, wl, 4, 30, 9)) < TOL


def test_bad_geometry_is_refused(mm):
    from catseye_b200._lib import CatsGpuError
    with pytest.raises(CatsGpuError):
        mm.conv2d_forward(np.zeros(16, np.float32), np.zeros(9, np.float32), 1, 1, 4, 4, 1, 5, 0, 1)
    with pytest.raises(CatsGpuError):
        mm.conv2d_forward(np.zeros(16, np.float32), np.zeros(9, np.float32), 1, 1, 4, 4, 1, 3, 1, 0)
