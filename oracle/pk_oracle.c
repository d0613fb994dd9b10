/*  pk_oracle.c -- CPU restatement of the reference's non-GEMM encoder ops.
 *
 *  TEST INFRASTRUCTURE ONLY (see pk_oracle.h). Built with IEEE single
 *  precision semantics (-ffp-contract=off, no -ffast-math): every multiply-add
 *  the reference's AVX2 path fuses is an explicit fmaf() here, every other
 *  operation rounds on its own.
 *
 *  Where the reference's -ffast-math build substitutes approximations
 *  (vector division -> rcpps + one Newton step, 1/sqrtf -> rsqrtss + one
 *  Newton step, expf -> libmvec), this file evaluates the exact operation the
 *  source states; those results differ from the reference by a few ulp and
 *  the tests compare within 2e-6 absolute or 1e-5 relative.
 */
#include "pk_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Horizontal sum of 8 lanes in the order of pk_hsum_avx2
 * (csrc/tensor_ops.c:129-137): (l0+l4)+(l2+l6) + (l1+l5)+(l3+l7). */
static float hsum8(const float l[8])
{
    float s0 = l[0] + l[4], s1 = l[1] + l[5], s2 = l[2] + l[6], s3 = l[3] + l[7];
    return (s0 + s2) + (s1 + s3);
}

/* pk_exp_avx2 (csrc/tensor_ops.c:97-121): clamp to [-87,87], k = rint(x*log2e),
 * r = x - k*ln2 (fused: the reference build contracts it into one FMA),
 * degree-5 Taylor polynomial by Horner FMAs, times 2^k built in the exponent. */
float or_exp_poly(float x)
{
    x = (x > -87.0f) ? x : -87.0f;   /* _mm256_max_ps(x, -87): NaN -> -87 */
    x = (x < 87.0f) ? x : 87.0f;
    float kf = rintf(x * 1.44269504088896341f);
    int ki = (int)kf;
    float r = fmaf(-kf, 0.69314718055994529f, x);
    float y = 1.0f / 120.0f;
    y = fmaf(y, r, 1.0f / 24.0f);
    y = fmaf(y, r, 1.0f / 6.0f);
    y = fmaf(y, r, 0.5f);
    y = fmaf(y, r, 1.0f);
    y = fmaf(y, r, 1.0f);
    union { int32_t i; float f; } p;
    p.i = (int32_t)((uint32_t)(ki + 127) << 23);
    return y * p.f;
}

/* pk_layer_norm AVX2 path (csrc/tensor_ops.c:187-217): 8-lane sum, hsum,
 * scalar tail; mean; 8-lane FMA sum of squared deviations; biased variance;
 * inv_std = 1/sqrtf(var + 1e-5); out = fma((x-mean)*inv_std, gamma, beta). */
void or_layer_norm(const float *x, const float *g, const float *b, float *out, int len)
{
    float acc[8] = {0};
    int i = 0;
    for (; i + 8 <= len; i += 8)
        for (int j = 0; j < 8; j++) acc[j] += x[i + j];
    float sum = hsum8(acc);
    for (; i < len; i++) sum += x[i];
    float mean = sum / (float)len;

    float vacc[8] = {0};
    i = 0;
    for (; i + 8 <= len; i += 8)
        for (int j = 0; j < 8; j++) {
            float d = x[i + j] - mean;
            vacc[j] = fmaf(d, d, vacc[j]);
        }
    float var_sum = hsum8(vacc);
    for (; i < len; i++) { float d = x[i] - mean; var_sum += d * d; }
    float var = var_sum / (float)len;
    float inv_std = 1.0f / sqrtf(var + 1e-5f);

    i = 0;
    for (; i + 8 <= len; i += 8)
        for (int j = 0; j < 8; j++)
            out[i + j] = fmaf((x[i + j] - mean) * inv_std, g[i + j], b[i + j]);
    for (; i < len; i++)
        out[i] = (x[i] - mean) * inv_std * g[i] + b[i];
}

/* pk_layer_norm_rows (csrc/tensor_ops.c:249-254): the op applied per row. */
void or_layer_norm_rows(const float *x, const float *g, const float *b, float *out,
                        int n_rows, int D)
{
    for (int r = 0; r < n_rows; r++)
        or_layer_norm(x + (size_t)r * D, g, b, out + (size_t)r * D, D);
}

/* pk_layer_norm_rows_inplace (csrc/tensor_ops.c:262-280): row to a buffer, copy back. */
void or_layer_norm_rows_inplace(float *x, const float *g, const float *b, int n_rows, int D)
{
    float *row = (float *)malloc((size_t)D * sizeof(float));
    for (int r = 0; r < n_rows; r++) {
        or_layer_norm(x + (size_t)r * D, g, b, row, D);
        memcpy(x + (size_t)r * D, row, (size_t)D * sizeof(float));
    }
    free(row);
}

/* pk_softmax AVX2 path (csrc/tensor_ops.c:312-334): max; polynomial exp on the
 * first 8*floor(len/8) entries (8-lane sum + hsum), libm expf on the tail
 * (sequential sum); scale by 1/sum. */
void or_softmax(float *x, int len)
{
    float mx = x[0];
    for (int i = 1; i < len; i++) if (x[i] > mx) mx = x[i];
    float acc[8] = {0};
    int i = 0;
    for (; i + 8 <= len; i += 8)
        for (int j = 0; j < 8; j++) {
            float e = or_exp_poly(x[i + j] - mx);
            x[i + j] = e;
            acc[j] += e;
        }
    float sum = hsum8(acc);
    for (; i < len; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    float inv = 1.0f / sum;
    for (i = 0; i < len; i++) x[i] *= inv;
}

/* pk_softmax_rows (csrc/tensor_ops.c:359-363). */
void or_softmax_rows(float *x, int n_rows, int len)
{
    for (int r = 0; r < n_rows; r++) or_softmax(x + (size_t)r * len, len);
}

/* pk_swish AVX2 path (csrc/tensor_ops.c:380-389): v * (1/(1 + exp_poly(0 - v)))
 * on the first 8*floor(n/8) entries of the flat array; x/(1+expf(-x)) on the tail. */
void or_swish(float *x, long long n)
{
    long long n8 = (n / 8) * 8, i = 0;
    for (; i < n8; i++) {
        float v = x[i];
        float s = 1.0f / (1.0f + or_exp_poly(0.0f - v));
        x[i] = v * s;
    }
    for (; i < n; i++) x[i] = x[i] / (1.0f + expf(-x[i]));
}

/* pk_relu (csrc/tensor_ops.c:401-416): x < 0 ? 0 : x. The scalar tail states
 * this form; the reference's -ffast-math build (which may order the operands
 * of _mm256_max_ps freely) gives the vector body the same result for NaN and
 * -0, as the golden vectors record: both are kept. */
void or_relu(float *x, long long n)
{
    for (long long i = 0; i < n; i++) if (x[i] < 0.0f) x[i] = 0.0f;
}

/* pk_bias_add (csrc/tensor_ops.c:420-435). */
void or_bias_add(float *x, const float *b, int len)
{
    for (int i = 0; i < len; i++) x[i] += b[i];
}

/* pk_depthwise_conv1d (csrc/tensor_ops.c:481-575): per channel, symmetric
 * pad (K-1)/2, out[t] = bias + sum_k x[t-pad+k]*w[k] accumulated in k order
 * as a fused multiply-add chain starting from the bias (the order of the
 * vectorised interior, :518-523), zero outside [0,T). b may be NULL (:561).
 * For even K the reference's interior range [pad, T-pad) (:496-499) lets the
 * last tap read past the end of the channel row; this restatement (and the
 * kernels) skip taps outside [0,T) for every K. The model uses K = 9. */
void or_depthwise_conv1d(const float *x, const float *w, const float *b, float *out,
                         int C, int T, int K)
{
    int pad = (K - 1) / 2;
    for (int c = 0; c < C; c++) {
        const float *xc = x + (size_t)c * T;
        const float *wc = w + (size_t)c * K;
        float bias = b ? b[c] : 0.0f;
        for (int t = 0; t < T; t++) {
            float val = bias;
            for (int k = 0; k < K; k++) {
                int s = t - pad + k;
                if (s >= 0 && s < T) val = fmaf(xc[s], wc[k], val);
            }
            out[(size_t)c * T + t] = val;
        }
    }
}

/* relative_shift (csrc/encoder.c:230-254): pad each [T, 2T-1] row with a
 * leading zero column into [T, 2T], then read [T, T] starting T floats in with
 * row stride 2T-1. Equivalent closed form: out[h,i,j] = bd[h,i,T-1-i+j]. */
void or_relative_shift(const float *bd, float *out, int H, int T)
{
    int L = 2 * T - 1, Lp = 2 * T;
    float *padded = (float *)malloc((size_t)H * T * Lp * sizeof(float));
    for (int h = 0; h < H; h++)
        for (int r = 0; r < T; r++) {
            padded[(size_t)h * T * Lp + (size_t)r * Lp] = 0.0f;
            memcpy(padded + (size_t)h * T * Lp + (size_t)r * Lp + 1,
                   bd + (size_t)h * T * L + (size_t)r * L, (size_t)L * sizeof(float));
        }
    for (int h = 0; h < H; h++) {
        const float *src = padded + (size_t)h * T * Lp + T;
        for (int i = 0; i < T; i++)
            for (int j = 0; j < T; j++)
                out[(size_t)h * T * T + (size_t)i * T + j] = src[(size_t)i * L + j];
    }
    free(padded);
}

/* Score combine (csrc/encoder.c:383-400): ac = (ac + bd) * scale, in place. */
void or_relpos_combine(float *ac, const float *bd_shifted, long long n, float scale)
{
    for (long long i = 0; i < n; i++) ac[i] = (ac[i] + bd_shifted[i]) * scale;
}

/* Head gather with pos_bias_u/v (csrc/encoder.c:319-356) from a biased QKV
 * [T, 3D]: Qu/Qv [H,T,Dh] = Q + u/v[h], K/V [H,T,Dh] copies. */
void or_qkv_split_uv(const float *qkv, const float *u, const float *v,
                     float *Qu, float *Qv, float *K, float *V, int T)
{
    int D = OR_D, Dh = OR_DH;
    for (int h = 0; h < OR_H; h++)
        for (int t = 0; t < T; t++) {
            const float *row = qkv + (size_t)t * 3 * D;
            size_t o = (size_t)h * T * Dh + (size_t)t * Dh;
            for (int d = 0; d < Dh; d++) {
                float q = row[h * Dh + d];
                Qu[o + d] = q + u[h * Dh + d];
                Qv[o + d] = q + v[h * Dh + d];
                K[o + d] = row[D + h * Dh + d];
                V[o + d] = row[2 * D + h * Dh + d];
            }
        }
}

/* P head split (csrc/encoder.c:362-368): P [L, D] -> P_h [H, L, Dh]. */
void or_pos_head_split(const float *P, float *P_h, int L)
{
    for (int h = 0; h < OR_H; h++)
        for (int p = 0; p < L; p++)
            memcpy(P_h + (size_t)h * L * OR_DH + (size_t)p * OR_DH,
                   P + (size_t)p * OR_D + h * OR_DH, OR_DH * sizeof(float));
}

/* Head concat (csrc/encoder.c:410-415): attn_h [H, T, Dh] -> attn [T, D]. */
void or_head_concat(const float *attn_h, float *attn, int T)
{
    for (int h = 0; h < OR_H; h++)
        for (int t = 0; t < T; t++)
            memcpy(attn + (size_t)t * OR_D + h * OR_DH,
                   attn_h + (size_t)h * T * OR_DH + (size_t)t * OR_DH, OR_DH * sizeof(float));
}

/* Residual adds: macaron x += 0.5*out (csrc/encoder.c:202-216, an FMA in the
 * vector body) and attention x += out (:422-434). 0.5*y is exact, so the fused
 * and unfused forms agree for alpha in {0.5, 1}. */
void or_residual(float *x, const float *y, float alpha, long long n)
{
    for (long long i = 0; i < n; i++) x[i] = fmaf(y[i], alpha, x[i]);
}

/* [rows, cols] -> [cols, rows] (the LN -> channel-first copy, csrc/encoder.c:449-452). */
void or_transpose(const float *src, float *dst, int rows, int cols)
{
    for (int r = 0; r < rows; r++)
        for (int c = 0; c < cols; c++)
            dst[(size_t)c * rows + r] = src[(size_t)r * cols + c];
}

/* Pointwise-conv bias (csrc/tensor_ops.c:585-589), channel-first [C, T]. */
void or_pointwise_bias(float *out, const float *b, int C, int T)
{
    for (int c = 0; c < C; c++)
        for (int t = 0; t < T; t++) out[(size_t)c * T + t] += b[c];
}

/* GLU (csrc/encoder.c:457-465) on channel-first [2D, T] -> [D, T]. */
void or_glu_channel_first(const float *pw1, float *gated, int D, int T)
{
    for (int d = 0; d < D; d++)
        for (int t = 0; t < T; t++) {
            float va = pw1[(size_t)d * T + t];
            float vb = pw1[(size_t)(D + d) * T + t];
            float s = 1.0f / (1.0f + expf(-vb));
            gated[(size_t)d * T + t] = va * s;
        }
}

/* The same GLU on time-first [T, 2D] -> [T, D] (split along the channel axis). */
void or_glu_time_first(const float *in, float *out, int T, int D)
{
    for (int t = 0; t < T; t++)
        for (int d = 0; d < D; d++) {
            float va = in[(size_t)t * 2 * D + d];
            float vb = in[(size_t)t * 2 * D + D + d];
            float s = 1.0f / (1.0f + expf(-vb));
            out[(size_t)t * D + d] = va * s;
        }
}

/* Conv-module residual (csrc/encoder.c:475-477): x[t,d] += pw2[d,t]. */
void or_transpose_add(float *x, const float *pw2, int T, int D)
{
    for (int t = 0; t < T; t++)
        for (int d = 0; d < D; d++) x[(size_t)t * D + d] += pw2[(size_t)d * T + t];
}

/* Inference BatchNorm on channel-first [C, T]: not present at run time in the
 * reference (folded into the depthwise weights offline, extract_weights.py:
 * 176-196); evaluated as ((y - mean) / sqrtf(var + eps)) * gamma + beta. */
void or_batch_norm(float *y, const float *mean, const float *var, const float *gamma,
                   const float *beta, float eps, int C, int T)
{
    for (int c = 0; c < C; c++) {
        float den = sqrtf(var[c] + eps);
        for (int t = 0; t < T; t++) {
            float v = (y[(size_t)c * T + t] - mean[c]) / den;
            y[(size_t)c * T + t] = v * gamma[c] + beta[c];
        }
    }
}

/* ── One conformer block with stand-in GEMM outputs ──────────────────────── */

enum {
    SI_FF1_H = 0, SI_FF1_OUT, SI_QKV, SI_P, SI_AC, SI_BD, SI_ATTN_H, SI_ATT_OUT,
    SI_PW1, SI_PW2, SI_FF2_H, SI_FF2_OUT
};
enum {
    CAP_LN_FF1 = 0, CAP_H1, CAP_LN_SA, CAP_QU, CAP_K, CAP_QV, CAP_PH, CAP_S, CAP_V,
    CAP_ATTN, CAP_CF, CAP_DW, CAP_LN_FF2, CAP_H2, CAP_N
};

static void save(float *const *outs, int role, const float *src, long long n)
{
    if (outs && outs[role]) memcpy(outs[role], src, (size_t)n * sizeof(float));
}

/* feed_forward (csrc/encoder.c:179-217) with GEMM outputs h_in, out_in. */
static void ff_module(float *x, int T, const float *nw, const float *nb,
                      const float *b1, const float *b2, const float *h_in,
                      const float *out_in, float *const *outs, int cap_ln, int cap_h)
{
    int D = OR_D, FF = OR_FF;
    float *ln = (float *)malloc((size_t)T * D * sizeof(float));
    float *h = (float *)malloc((size_t)T * FF * sizeof(float));
    float *out = (float *)malloc((size_t)T * D * sizeof(float));
    or_layer_norm_rows(x, nw, nb, ln, T, D);
    save(outs, cap_ln, ln, (long long)T * D);
    memcpy(h, h_in, (size_t)T * FF * sizeof(float));
    for (int t = 0; t < T; t++) or_bias_add(h + (size_t)t * FF, b1, FF);
    or_swish(h, (long long)T * FF);
    save(outs, cap_h, h, (long long)T * FF);
    memcpy(out, out_in, (size_t)T * D * sizeof(float));
    for (int t = 0; t < T; t++) or_bias_add(out + (size_t)t * D, b2, D);
    or_residual(x, out, 0.5f, (long long)T * D);
    free(ln); free(h); free(out);
}

/* conformer_block (csrc/encoder.c:482-491): FF1, self-attention
 * (:297-435), conv module (:439-478), FF2, final LN in place. The GEMM
 * outputs come from standins[SI_*]; every GEMM input is written to
 * outs[CAP_*] when that pointer is non-NULL. Parameter order as
 * ref_harness.c's fill_block. */
void or_conformer_block(float *x, int T, const float *const *p,
                        const float *const *si, float *const *outs)
{
    int D = OR_D, H = OR_H, Dh = OR_DH, L = 2 * T - 1;

    ff_module(x, T, p[0], p[1], p[2], p[3], si[SI_FF1_H], si[SI_FF1_OUT], outs,
              CAP_LN_FF1, CAP_H1);

    /* self-attention */
    {
        float *ln = (float *)malloc((size_t)T * D * sizeof(float));
        float *qkv = (float *)malloc((size_t)T * 3 * D * sizeof(float));
        float *Qu = (float *)malloc((size_t)H * T * Dh * sizeof(float));
        float *Qv = (float *)malloc((size_t)H * T * Dh * sizeof(float));
        float *K = (float *)malloc((size_t)H * T * Dh * sizeof(float));
        float *V = (float *)malloc((size_t)H * T * Dh * sizeof(float));
        float *Ph = (float *)malloc((size_t)H * L * Dh * sizeof(float));
        float *ac = (float *)malloc((size_t)H * T * T * sizeof(float));
        float *bds = (float *)malloc((size_t)H * T * T * sizeof(float));
        float *attn = (float *)malloc((size_t)T * D * sizeof(float));
        float *out = (float *)malloc((size_t)T * D * sizeof(float));

        or_layer_norm_rows(x, p[4], p[5], ln, T, D);
        save(outs, CAP_LN_SA, ln, (long long)T * D);
        memcpy(qkv, si[SI_QKV], (size_t)T * 3 * D * sizeof(float));
        for (int t = 0; t < T; t++) or_bias_add(qkv + (size_t)t * 3 * D, p[6], 3 * D);
        or_qkv_split_uv(qkv, p[7], p[8], Qu, Qv, K, V, T);
        save(outs, CAP_QU, Qu, (long long)H * T * Dh);
        save(outs, CAP_QV, Qv, (long long)H * T * Dh);
        save(outs, CAP_K, K, (long long)H * T * Dh);
        save(outs, CAP_V, V, (long long)H * T * Dh);
        or_pos_head_split(si[SI_P], Ph, L);
        save(outs, CAP_PH, Ph, (long long)H * L * Dh);
        memcpy(ac, si[SI_AC], (size_t)H * T * T * sizeof(float));
        or_relative_shift(si[SI_BD], bds, H, T);
        or_relpos_combine(ac, bds, (long long)H * T * T, 1.0f / sqrtf((float)Dh));
        or_softmax_rows(ac, H * T, T);
        save(outs, CAP_S, ac, (long long)H * T * T);
        or_head_concat(si[SI_ATTN_H], attn, T);
        save(outs, CAP_ATTN, attn, (long long)T * D);
        memcpy(out, si[SI_ATT_OUT], (size_t)T * D * sizeof(float));
        for (int t = 0; t < T; t++) or_bias_add(out + (size_t)t * D, p[9], D);
        or_residual(x, out, 1.0f, (long long)T * D);
        free(ln); free(qkv); free(Qu); free(Qv); free(K); free(V); free(Ph);
        free(ac); free(bds); free(attn); free(out);
    }

    /* conv module */
    {
        float *ln = (float *)malloc((size_t)T * D * sizeof(float));
        float *cf = (float *)malloc((size_t)D * T * sizeof(float));
        float *pw1 = (float *)malloc((size_t)2 * D * T * sizeof(float));
        float *gated = (float *)malloc((size_t)D * T * sizeof(float));
        float *dw = (float *)malloc((size_t)D * T * sizeof(float));
        float *pw2 = (float *)malloc((size_t)D * T * sizeof(float));
        or_layer_norm_rows(x, p[10], p[11], ln, T, D);
        or_transpose(ln, cf, T, D);
        save(outs, CAP_CF, cf, (long long)D * T);
        memcpy(pw1, si[SI_PW1], (size_t)2 * D * T * sizeof(float));
        or_pointwise_bias(pw1, p[12], 2 * D, T);
        or_glu_channel_first(pw1, gated, D, T);
        or_depthwise_conv1d(gated, p[13], p[14], dw, D, T, 9);
        or_swish(dw, (long long)D * T);
        save(outs, CAP_DW, dw, (long long)D * T);
        memcpy(pw2, si[SI_PW2], (size_t)D * T * sizeof(float));
        or_pointwise_bias(pw2, p[15], D, T);
        or_transpose_add(x, pw2, T, D);
        free(ln); free(cf); free(pw1); free(gated); free(dw); free(pw2);
    }

    ff_module(x, T, p[16], p[17], p[18], p[19], si[SI_FF2_H], si[SI_FF2_OUT], outs,
              CAP_LN_FF2, CAP_H2);
    or_layer_norm_rows_inplace(x, p[20], p[21], T, D);
}

/* ── csrc/decoder.c ────────────────────────────────────────────────────── */

/* Joint add + activation (csrc/decoder.c:62-67): h = enc + pred, then ReLU
 * (act 0, "if (h < 0) h = 0") or tanhf (act 1, the north-star variant).
 * enc [B, T, J], pred [B, J] broadcast over T. */
void or_joint_add_act(const float *enc, const float *pred, float *out,
                      int B, int T, int J, int act)
{
    for (int b = 0; b < B; b++)
        for (int t = 0; t < T; t++)
            for (int j = 0; j < J; j++) {
                size_t o = ((size_t)b * T + t) * J + j;
                float h = enc[o] + pred[(size_t)b * J + j];
                if (act == 0) { if (h < 0.0f) h = 0.0f; }
                else h = tanhf(h);
                out[o] = h;
            }
}

/* Greedy argmax (csrc/decoder.c:106-114): strict '>' scan from index 0, so
 * the first maximum wins and NaN entries never replace the running best. */
void or_argmax_rows(const float *logits, int32_t *out, long long n_rows, int V)
{
    for (long long r = 0; r < n_rows; r++) {
        const float *l = logits + r * V;
        int best = 0;
        float best_val = l[0];
        for (int v = 1; v < V; v++)
            if (l[v] > best_val) { best_val = l[v]; best = v; }
        out[r] = best;
    }
}
