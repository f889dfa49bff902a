/*
 * ref_cnn.c — exports the reference's own CPU sgemm (gemm_rnn/rnt/rtn), im2col
 * and the conv / linear forward layers from a shared library.
 *
 * TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile from REF_DIR/catseye.h
 * with -DCATS_USE_FLOAT into oracle/_ref/; nothing here adds arithmetic.
 */
#include "catseye.h"

void ref_sgemm(char ta, char tb, int m, int n, int k, float alpha, float *a, float *b,
               float beta, float *c)
{
    if (ta == 'N' && tb == 'N') gemm_rnn(m, n, k, alpha, a, b, beta, c);
    else if (ta == 'N' && tb == 'T') gemm_rnt(m, n, k, alpha, a, b, beta, c);
    else if (ta == 'T' && tb == 'N') gemm_rtn(m, n, k, alpha, a, b, beta, c);
}

void ref_im2col(const float *im, int channels, int height, int width, int kh, int kw, int ph,
                int pw, int sh, int sw, float *col)
{
    im2col(im, channels, height, width, kh, kw, ph, pw, sh, sw, col);
}

/* CatsEye_convolutional_forward on a hand-filled layer (catseye.h:557-574). */
void ref_conv2d_forward(float *x, float *w, float *z, int batch, int ich, int h, int wd, int ch,
                        int k, int pad, int stride)
{
    CatsEye p;
    CatsEye_layer l;
    memset(&p, 0, sizeof(p));
    memset(&l, 0, sizeof(l));
    p.batch = batch;
    l.p = &p;
    l.ksize = k; l.kw = k; l.kh = k; l.stride = stride; l.padding = pad; l.pw = pad; l.ph = pad;
    l.ich = ich; l.ch = ch; l.sx = wd; l.sy = h;
    l.ox = (wd + 2 * pad - k) / stride + 1;
    l.oy = (h + 2 * pad - k) / stride + 1;
    l.inputs = ich * h * wd;
    l.outputs = ch * l.ox * l.oy;
    l.x = x; l.w = w; l.z = z;
    l.workspace = malloc(sizeof(real) * (size_t)l.ox * l.oy * k * k * ich * batch);
    CatsEye_convolutional_forward(&l);
    free(l.workspace);
}

/* CatsEye_linear_forward (catseye.h:416-444): bias lives at w[inputs*outputs]. */
void ref_linear_forward(float *x, float *w, float *z, int batch, int in, int out)
{
    CatsEye p;
    CatsEye_layer l;
    memset(&p, 0, sizeof(p));
    memset(&l, 0, sizeof(l));
    p.batch = batch;
    l.p = &p;
    l.inputs = in; l.outputs = out;
    l.x = x; l.w = w; l.z = z;
    CatsEye_linear_forward(&l);
}
