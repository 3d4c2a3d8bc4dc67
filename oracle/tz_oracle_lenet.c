/*
 * tz_oracle_lenet.c -- CPU restatement of the reference LeNet-5 forward (lenet.zig).
 *
 * TEST INFRASTRUCTURE ONLY (see tz_oracle.h): the checker for the sm_100a LeNet kernels.
 *
 * Follows, operation for operation in f32 (compiled with -ffp-contract=off):
 *   conv2dForward        conv2d.zig:30-110   output = bias; sum over (kh, kw, ic) in that order
 *                                             from 0, then output += sum; zero padding skipped
 *   applyRelu            lenet.zig:859-863    max(v, 0)
 *   maxPool2dForward     maxpool.zig:25-78    running max from -inf, strict '>' (first max wins)
 *   linearForward        lenet.zig:874-898    sum = bias[j]; sum += x[k] * w[j, k] for k ascending
 *   forwardSequential    lenet.zig:270-321    conv1 -> ReLU -> pool -> conv2 -> ReLU -> pool ->
 *                                             flatten (NHWC) -> FC1 -> ReLU -> FC2 -> ReLU -> FC3
 * Two variants: TZO_LENET_REF is lenet.zig itself (conv1 valid, FC1 in = 256, logits out);
 * TZO_LENET_PAD2 is the benchmark configuration (conv1 zero padding 2, FC1 in = 400, and a
 * softmax over the 10 logits: max, exp(x - max), divide by the sum, softmax.zig:20-47).
 *
 * Parity status: the reference ships no LeNet forward fixtures (its tests check training
 * behaviour only), so this restatement is cross-checked against an independent PyTorch forward
 * (torch.nn.functional.conv2d / max_pool2d / linear) in the tests.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "tz_oracle.h"

static void conv2d_nhwc(const float* in, const float* w, const float* b, float* out, int ih, int iw, int ic, int oc,
                        int k, int pad) {
    const int oh = ih + 2 * pad - k + 1, ow = iw + 2 * pad - k + 1;
    for (int y = 0; y < oh; ++y)
        for (int x = 0; x < ow; ++x)
            for (int o = 0; o < oc; ++o) {
                float sum = 0.0f;
                for (int kh = 0; kh < k; ++kh)
                    for (int kw = 0; kw < k; ++kw) {
                        const int yy = y + kh - pad, xx = x + kw - pad;
                        if (yy < 0 || yy >= ih || xx < 0 || xx >= iw) continue;
                        for (int c = 0; c < ic; ++c)
                            sum += in[(yy * iw + xx) * ic + c] * w[((o * k + kh) * k + kw) * ic + c];
                    }
                out[(y * ow + x) * oc + o] = b[o] + sum;
            }
}

static void relu(float* v, int n) {
    for (int i = 0; i < n; ++i) v[i] = v[i] > 0.0f ? v[i] : 0.0f;
}

static void maxpool2(const float* in, float* out, int ih, int iw, int c) {
    const int oh = ih / 2, ow = iw / 2;
    for (int y = 0; y < oh; ++y)
        for (int x = 0; x < ow; ++x)
            for (int ch = 0; ch < c; ++ch) {
                float m = -INFINITY;
                for (int py = 0; py < 2; ++py)
                    for (int px = 0; px < 2; ++px) {
                        const float v = in[((2 * y + py) * iw + (2 * x + px)) * c + ch];
                        if (v > m) m = v;
                    }
                out[(y * ow + x) * c + ch] = m;
            }
}

static void linear(const float* x, const float* w, const float* b, float* y, int in, int out) {
    for (int j = 0; j < out; ++j) {
        float sum = b[j];
        for (int k = 0; k < in; ++k) sum += x[k] * w[j * in + k];
        y[j] = sum;
    }
}

void tzo_lenet_forward_one(const tzo_lenet_weights* w, int variant, const float* img, float* out) {
    const int pad = variant == TZO_LENET_PAD2 ? 2 : 0;
    const int c1 = 28 + 2 * pad - 4;      /* 24 or 28 */
    const int p1 = c1 / 2;                /* 12 or 14 */
    const int c2 = p1 - 4;                /* 8 or 10 */
    const int p2 = c2 / 2;                /* 4 or 5 */
    const int feat = p2 * p2 * 16;        /* 256 or 400 */
    float a1[28 * 28 * 6], q1[14 * 14 * 6], a2[10 * 10 * 16], q2[400], f1[120], f2[84];
    conv2d_nhwc(img, w->conv1_w, w->conv1_b, a1, 28, 28, 1, 6, 5, pad);
    relu(a1, c1 * c1 * 6);
    maxpool2(a1, q1, c1, c1, 6);
    conv2d_nhwc(q1, w->conv2_w, w->conv2_b, a2, p1, p1, 6, 16, 5, 0);
    relu(a2, c2 * c2 * 16);
    maxpool2(a2, q2, c2, c2, 16);
    linear(q2, w->fc1_w, w->fc1_b, f1, feat, 120);
    relu(f1, 120);
    linear(f1, w->fc2_w, w->fc2_b, f2, 120, 84);
    relu(f2, 84);
    linear(f2, w->fc3_w, w->fc3_b, out, 84, 10);
    if (variant == TZO_LENET_PAD2) {
        float m = out[0];
        for (int i = 1; i < 10; ++i) m = out[i] > m ? out[i] : m;
        float s = 0.0f;
        for (int i = 0; i < 10; ++i) {
            out[i] = expf(out[i] - m);
            s += out[i];
        }
        for (int i = 0; i < 10; ++i) out[i] = out[i] / s;
    }
}

/* Batch forward: images [n, 28, 28, 1] -> out [n, 10]; images are independent (OpenMP over the
 * batch when built with -fopenmp, nthreads <= 0 = all cores). */
void tzo_lenet_forward(const tzo_lenet_weights* w, int variant, const float* images, int64_t n, float* out,
                       int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) {
#pragma omp parallel for schedule(static) num_threads(nthreads)
        for (int64_t i = 0; i < n; ++i) tzo_lenet_forward_one(w, variant, images + i * 784, out + i * 10);
        return;
    }
#pragma omp parallel for schedule(static)
#endif
    for (int64_t i = 0; i < n; ++i) tzo_lenet_forward_one(w, variant, images + i * 784, out + i * 10);
    (void)nthreads;
}
