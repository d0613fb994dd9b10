/* pk_oracle_decode.c -- TEST INFRASTRUCTURE ONLY: plain-C restatement of the
 * reference's greedy RNN-T decode of one utterance, the checker of the batched
 * decode kernels:
 *   pk_greedy_decode   csrc/decoder.c:80-132 (joint, argmax, up to 10 symbols
 *                      per frame, the decoder step after every symbol)
 *   pk_joint           csrc/decoder.c:38-76 (bias adds, add, ReLU)
 *   pk_decoder_step    csrc/decoder.c:12-33 (embedding row, two LSTM layers)
 *   pk_lstm_step       csrc/tensor_ops.c:594-629 (gates, sigmoid / tanh cell)
 *
 * Every matrix-vector product is a stand-in supplied by the caller through
 * `gemm` (the products are outside the path this restatement checks):
 *   OR_DEC_ENC    frame t's encoder projection  [640]   (iter = t, in = NULL)
 *   OR_DEC_PRED   joint.pred applied to h1      [640]
 *   OR_DEC_OUT    joint.out applied to hidden   [1025]
 *   OR_DEC_L{0,1}_W{I,R}  W_i x, W_r h of layer l [2560]
 * `iter` counts the joint evaluations made so far: the k-th joint evaluation
 * and the decoder step just before it (the first one at k = 0, after each
 * emitted symbol at k = the next evaluation) share iteration k.
 *
 * Evaluated in IEEE single precision (built with -ffp-contract=off), libm
 * expf / tanhf for the cell, operations in the order the source states them:
 * gates = W_r h + W_i x, then + (B[i] + B[4H + i]); c = f c + i g; h = o tanh(c). */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "pk_oracle.h"

#define DEC_H 640      /* LSTM hidden = embedding = joint width (csrc/parakeet.h:26-32) */
#define DEC_V 1025     /* vocabulary + blank (:28) */
#define DEC_BLANK 1024 /* (:29) */
#define DEC_MAX_SYMBOLS 10

static float sigmoid1(float x) { return 1.0f / (1.0f + expf(-x)); }

/* One LSTM layer (pk_lstm_step) on input x with the stand-in products. */
static void lstm_layer(or_dec_gemm_fn gemm, void *user, int g_wi, int g_wr, int iter,
                       const float *x, const float *B, float *h, float *c, float *gates,
                       float *tmp)
{
    const int H = DEC_H;
    gemm(user, g_wi, iter, x, H, gates, 4 * H);
    gemm(user, g_wr, iter, h, H, tmp, 4 * H);
    for (int i = 0; i < 4 * H; i++) gates[i] = tmp[i] + gates[i];
    for (int i = 0; i < 4 * H; i++) gates[i] += B[i] + B[4 * H + i];
    for (int j = 0; j < H; j++) {
        const float ig = sigmoid1(gates[j]);
        const float og = sigmoid1(gates[H + j]);
        const float fg = sigmoid1(gates[2 * H + j]);
        const float cg = tanhf(gates[3 * H + j]);
        c[j] = fg * c[j] + ig * cg;
        h[j] = og * tanhf(c[j]);
    }
}

static void decoder_step(or_dec_gemm_fn gemm, void *user, int iter, int token,
                         const float *embed, const float *B0, const float *B1, float *state,
                         float *gates, float *tmp)
{
    float *h0 = state, *h1 = state + DEC_H, *c0 = state + 2 * DEC_H, *c1 = state + 3 * DEC_H;
    lstm_layer(gemm, user, OR_DEC_L0_WI, OR_DEC_L0_WR, iter, embed + (size_t)token * DEC_H, B0,
               h0, c0, gates, tmp);
    lstm_layer(gemm, user, OR_DEC_L1_WI, OR_DEC_L1_WR, iter, h0, B1, h1, c1, gates, tmp);
}

int or_greedy_decode(int T, const float *embed, const float *B0, const float *B1,
                     const float *enc_b, const float *pred_b, const float *out_b,
                     or_dec_gemm_fn gemm, void *user, int *tokens, int max_tokens,
                     float *state, int *n_iters)
{
    float *gates = (float *)malloc(sizeof(float) * 4 * DEC_H);
    float *tmp = (float *)malloc(sizeof(float) * 4 * DEC_H);
    float *e = (float *)malloc(sizeof(float) * DEC_H);
    float *p = (float *)malloc(sizeof(float) * DEC_H);
    float *hid = (float *)malloc(sizeof(float) * DEC_H);
    float *logits = (float *)malloc(sizeof(float) * DEC_V);
    if (!gates || !tmp || !e || !p || !hid || !logits) {
        free(gates); free(tmp); free(e); free(p); free(hid); free(logits);
        return -1;
    }
    memset(state, 0, sizeof(float) * 4 * DEC_H);   /* LSTMState zeroed (:85-86) */
    int n = 0, iter = 0;
    decoder_step(gemm, user, 0, DEC_BLANK, embed, B0, B1, state, gates, tmp);   /* (:96-97) */
    for (int t = 0; t < T; t++) {
        for (int s = 0; s < DEC_MAX_SYMBOLS; s++) {
            /* pk_joint: enc_proj + bias, pred_proj + bias, add, ReLU, out + bias */
            gemm(user, OR_DEC_ENC, t, NULL, 0, e, DEC_H);
            for (int i = 0; i < DEC_H; i++) e[i] += enc_b[i];
            gemm(user, OR_DEC_PRED, iter, state + DEC_H, DEC_H, p, DEC_H);
            for (int i = 0; i < DEC_H; i++) p[i] += pred_b[i];
            for (int i = 0; i < DEC_H; i++) {
                hid[i] = e[i] + p[i];
                if (hid[i] < 0.0f) hid[i] = 0.0f;
            }
            gemm(user, OR_DEC_OUT, iter, hid, DEC_H, logits, DEC_V);
            for (int v = 0; v < DEC_V; v++) logits[v] += out_b[v];
            iter++;
            int best = 0;   /* first maximum, strict > (:106-114) */
            float best_val = logits[0];
            for (int v = 1; v < DEC_V; v++)
                if (logits[v] > best_val) {
                    best_val = logits[v];
                    best = v;
                }
            if (best == DEC_BLANK) break;
            if (n < max_tokens) tokens[n] = best;
            n++;
            decoder_step(gemm, user, iter, best, embed, B0, B1, state, gates, tmp);
        }
    }
    if (n_iters) *n_iters = iter;
    free(gates); free(tmp); free(e); free(p); free(hid); free(logits);
    return n;
}
