/* pk_oracle_preencode.c -- TEST INFRASTRUCTURE ONLY: plain-C restatement of
 * the reference's pre-encode subsampling and input scaling
 * (csrc/encoder.c:103-175, 578-593; pk_conv2d csrc/tensor_ops.c:439-475),
 * the checker of the pre-encode kernels. Evaluated in IEEE single precision
 * (built with -ffp-contract=off): each convolution output starts from its
 * bias and adds tap products as fused multiply-adds in (ic, kh, kw) order,
 * taps outside the input skipped, as the reference's loop does under its
 * build's contraction.
 *
 * The GEMM steps of the stage -- the two 1x1 convolutions and the output
 * projection -- are stand-ins supplied by the caller (y2, y3, proj: the GEMM
 * products without bias); the restatement adds the biases and captures their
 * inputs (s2d, s3d, flat). */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "pk_oracle.h"

#define PRE_C 256    /* subsampling channels (csrc/parakeet.h:23) */
#define PRE_MELS 128 /* mel bins (csrc/parakeet.h:22) */

/* pk_conv2d for groups == Cin (depthwise) or Cin == 1: out [Cout, Ho, Wo]. */
static void conv3x3_s2(const float *x, const float *w, const float *b, float *out, int Cout,
                       int H, int W, int per_channel_input)
{
    const int Ho = (H + 2 - 3) / 2 + 1, Wo = (W + 2 - 3) / 2 + 1;
    for (int oc = 0; oc < Cout; oc++) {
        const float *xc = x + (per_channel_input ? (size_t)oc * H * W : 0);
        const float *wc = w + (size_t)oc * 9;
        for (int oh = 0; oh < Ho; oh++)
            for (int ow = 0; ow < Wo; ow++) {
                float val = b[oc];
                for (int kh = 0; kh < 3; kh++)
                    for (int kw = 0; kw < 3; kw++) {
                        const int ih = 2 * oh - 1 + kh, iw = 2 * ow - 1 + kw;
                        if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                            val = fmaf(xc[(size_t)ih * W + iw], wc[kh * 3 + kw], val);
                    }
                out[((size_t)oc * Ho + oh) * Wo + ow] = val;
            }
    }
}

static float relu1(float v) { return v < 0.0f ? 0.0f : v; }

int or_pre_out_frames(int T)
{
    int h = T;
    for (int s = 0; s < 3; s++) h = (h + 2 - 3) / 2 + 1;
    return h;
}

int or_pre_encode(const float *mel, int T, const float *const *p, const float *y2,
                  const float *y3, const float *proj, float *s2d_cap, float *s3d_cap,
                  float *flat_cap, float *x_out)
{
    const int H1 = (T + 2 - 3) / 2 + 1, W1 = PRE_MELS / 2;
    const int H2 = (H1 + 2 - 3) / 2 + 1, W2 = W1 / 2;
    const int H3 = (H2 + 2 - 3) / 2 + 1, W3 = W2 / 2;
    const size_t P1 = (size_t)H1 * W1, P2 = (size_t)H2 * W2, P3 = (size_t)H3 * W3;
    float *mel_t = (float *)calloc((size_t)T * PRE_MELS, sizeof(float));
    float *s1 = (float *)malloc(PRE_C * P1 * sizeof(float));
    float *s2d = (float *)malloc(PRE_C * P2 * sizeof(float));
    float *s2 = (float *)malloc(PRE_C * P2 * sizeof(float));
    float *s3d = (float *)malloc(PRE_C * P3 * sizeof(float));
    float *s3 = (float *)malloc(PRE_C * P3 * sizeof(float));
    float *flat = (float *)malloc((size_t)H3 * PRE_C * W3 * sizeof(float));
    if (!mel_t || !s1 || !s2d || !s2 || !s3d || !s3 || !flat) {
        free(mel_t); free(s1); free(s2d); free(s2); free(s3d); free(s3); free(flat);
        return -1;
    }
    /* mel [128, T] -> [T, 128] (:111-114) */
    for (int t = 0; t < T; t++)
        for (int m = 0; m < PRE_MELS; m++) mel_t[(size_t)t * PRE_MELS + m] = mel[(size_t)m * T + t];
    /* conv 0 (1 -> 256, 3x3, stride 2) + ReLU (:116-121) */
    conv3x3_s2(mel_t, p[0], p[1], s1, PRE_C, T, PRE_MELS, 0);
    for (size_t i = 0; i < PRE_C * P1; i++) s1[i] = relu1(s1[i]);
    /* depthwise 3x3 stride 2, then the 1x1 conv: stand-in + bias, ReLU (:123-137) */
    conv3x3_s2(s1, p[2], p[3], s2d, PRE_C, H1, W1, 1);
    if (s2d_cap) memcpy(s2d_cap, s2d, PRE_C * P2 * sizeof(float));
    for (int c = 0; c < PRE_C; c++)
        for (size_t q = 0; q < P2; q++) s2[c * P2 + q] = relu1(y2[c * P2 + q] + p[4][c]);
    /* again, 32 -> 16 wide (:139-152) */
    conv3x3_s2(s2, p[5], p[6], s3d, PRE_C, H2, W2, 1);
    if (s3d_cap) memcpy(s3d_cap, s3d, PRE_C * P3 * sizeof(float));
    for (int c = 0; c < PRE_C; c++)
        for (size_t q = 0; q < P3; q++) s3[c * P3 + q] = relu1(y3[c * P3 + q] + p[7][c]);
    /* [256, T', 16] -> [T', 256 * 16] (:154-159) */
    for (int c = 0; c < PRE_C; c++)
        for (int h = 0; h < H3; h++)
            for (int w = 0; w < W3; w++)
                flat[(size_t)h * PRE_C * W3 + (size_t)c * W3 + w] = s3[((size_t)c * H3 + h) * W3 + w];
    if (flat_cap) memcpy(flat_cap, flat, (size_t)H3 * PRE_C * W3 * sizeof(float));
    /* projection stand-in + bias (:161-165), then x = result^T * sqrtf(1024) (:578-590) */
    const float scale = sqrtf(1024.0f);
    for (int t = 0; t < H3; t++)
        for (int d = 0; d < 1024; d++)
            x_out[(size_t)t * 1024 + d] = (proj[(size_t)t * 1024 + d] + p[8][d]) * scale;
    free(mel_t); free(s1); free(s2d); free(s2); free(s3d); free(s3); free(flat);
    return H3;
}
