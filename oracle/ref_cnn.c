/*
 * ref_cnn.c — exports the reference's own CPU sgemm (gemm_rnn/rnt/rtn), im2col
 * and the conv / linear forward layers from a shared library.
 *
 * TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile from REF_DIR/catseye.h
 * with -DCATS_USE_FLOAT into oracle/_ref/; nothing here adds arithmetic.
 */
#include "catseye.h"

#ifdef CATS_OPENCL
/* The OpenCL backend built over libcatsgpu (include/cats_ocl_cuda.h is
 * force-included): sgemm_init as catseye's network constructor calls it. */
void ref_cnn_init(void) { sgemm_init(0); }
#endif

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

/* col2im itself (catseye.h:533-556). */
void ref_col2im(const float *col, int channels, int height, int width, int kh, int kw, int ph, int pw, int sh,
                int sw, float *im)
{
    col2im(col, channels, height, width, kh, kw, ph, pw, sh, sw, im);
}

static void conv_layer(CatsEye *p, CatsEye_layer *l, int batch, int ich, int h, int wd, int ch, int k, int pad,
                       int stride)
{
    memset(p, 0, sizeof(*p));
    memset(l, 0, sizeof(*l));
    p->batch = batch;
    l->p = p;
    l->ksize = k; l->kw = k; l->kh = k; l->stride = stride; l->padding = pad; l->pw = pad; l->ph = pad;
    l->ich = ich; l->ch = ch; l->sx = wd; l->sy = h;
    l->ox = (wd + 2 * pad - k) / stride + 1;
    l->oy = (h + 2 * pad - k) / stride + 1;
    l->inputs = ich * h * wd;
    l->outputs = ch * l->ox * l->oy;
}

/* CatsEye_convolutional_backward (catseye.h:589-620): its col2im workspace is
 * the network's shared scratch p->mem. */
void ref_conv2d_backward(float *dout, float *w, float *din, int batch, int ich, int h, int wd, int ch, int k,
                         int pad, int stride)
{
    CatsEye p;
    CatsEye_layer l;
    conv_layer(&p, &l, batch, ich, h, wd, ch, k, pad, stride);
    l.w = w; l.dOut = dout; l.dIn = din;
    p.mem = malloc(sizeof(real) * (size_t)l.ox * l.oy * k * k * ich);
    CatsEye_convolutional_backward(&l);
    free(p.mem);
}

/* CatsEye_convolutional_update (catseye.h:622-640) reads the im2col workspace
 * the forward pass left: the forward runs first, into a scratch z. */
void ref_conv2d_update(float *dout, float *x, float *dw, int batch, int ich, int h, int wd, int ch, int k, int pad,
                       int stride, float *w)
{
    CatsEye p;
    CatsEye_layer l;
    conv_layer(&p, &l, batch, ich, h, wd, ch, k, pad, stride);
    l.x = x; l.w = w; l.dOut = dout; l.dw = dw;
    l.z = malloc(sizeof(real) * (size_t)l.outputs * batch);
    l.workspace = malloc(sizeof(real) * (size_t)l.ox * l.oy * k * k * ich * batch);
    CatsEye_convolutional_forward(&l);
    CatsEye_convolutional_update(&l);
    free(l.workspace);
    free(l.z);
}

/* CatsEye_linear_backward (catseye.h:445-477). */
void ref_linear_backward(float *dout, float *w, float *din, int batch, int in, int out)
{
    CatsEye p;
    CatsEye_layer l;
    memset(&p, 0, sizeof(p));
    memset(&l, 0, sizeof(l));
    p.batch = batch;
    l.p = &p;
    l.inputs = in; l.outputs = out;
    l.w = w; l.dOut = dout; l.dIn = din;
    CatsEye_linear_backward(&l);
}

/* CatsEye_linear_update (catseye.h:478-505): dw += dOut^T x, and the biases
 * kept after the weights step by -eta * dOut. */
void ref_linear_update(float *dout, float *x, float *w, float *dw, int batch, int in, int out, float eta)
{
    CatsEye p;
    CatsEye_layer l;
    memset(&p, 0, sizeof(p));
    memset(&l, 0, sizeof(l));
    p.batch = batch;
    l.p = &p;
    l.inputs = in; l.outputs = out;
    l.x = x; l.w = w; l.dw = dw; l.dOut = dout; l.eta = eta;
    CatsEye_linear_update(&l);
}
