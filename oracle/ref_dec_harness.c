/*  ref_dec_harness.c -- TEST INFRASTRUCTURE ONLY (checker, never shipped).
 *
 *  Compiles the reference engine's own csrc/decoder.c into
 *  oracle/_ref/libpkref_dec.so together with its csrc/tensor_ops.c (for
 *  pk_lstm_step and pk_bias_add), blas.c and threadpool.c, straight from the
 *  reference tree (oracle/Makefile; nothing is copied into this repository).
 *  Every cblas_sgemv call of decoder.c and tensor_ops.c is renamed at compile
 *  time to pkh_dec_sgemv below, which stands in for the product: it asks the
 *  caller's callback for the output of that matrix-vector product (the
 *  products are GEMM work, outside the checked path) and applies the call's
 *  beta (y = product, or y = product + y). All other code that runs --
 *  pk_greedy_decode, pk_joint, pk_decoder_step, pk_lstm_step, pk_bias_add --
 *  is the reference's own.
 *
 *  The product is identified by its matrix pointer: the harness builds the
 *  model's decoder weights with a distinct placeholder address for each
 *  matrix. The callback gets the same (gemm, iter) numbering as the
 *  restatement (oracle/pk_oracle_decode.c): iter = frame index for the
 *  encoder projection, else the number of joint evaluations made so far.
 */
#define cblas_sgemv pkh_dec_sgemv
#include "decoder.c"
#undef cblas_sgemv

enum { D_ENC = 0, D_PRED, D_OUT, D_L0_WI, D_L0_WR, D_L1_WI, D_L1_WR, D_N };

typedef void (*pkh_dec_gemm_fn)(void *user, int gemm, int iter, const float *in, int n_in,
                                float *out, int n_out);

static float g_mats[D_N];          /* placeholder matrices: &g_mats[g] identifies product g */
static pkh_dec_gemm_fn g_fn;
static void *g_user;
static const float *g_enc;         /* the enc_out the decode was given */
static int g_iter;                 /* joint evaluations made so far */

void pkh_dec_sgemv(CBLAS_ORDER order, CBLAS_TRANSPOSE trans, int M, int N, float alpha,
                   const float *A, int lda, const float *X, int incX, float beta, float *Y,
                   int incY)
{
    (void)order; (void)alpha; (void)lda; (void)incX; (void)incY;
    const int g = (int)(A - g_mats);
    const int n_out = trans == CblasTrans ? N : M;
    const int n_in = trans == CblasTrans ? M : N;
    float *prod = (float *)malloc(sizeof(float) * (size_t)n_out);
    if (g == D_ENC)
        g_fn(g_user, D_ENC, (int)((X - g_enc) / PK_D_MODEL), NULL, 0, prod, n_out);
    else
        g_fn(g_user, g, g_iter, X, n_in, prod, n_out);
    for (int i = 0; i < n_out; i++) Y[i] = beta == 0.0f ? prod[i] : prod[i] + Y[i];
    free(prod);
    if (g == D_OUT) g_iter++;
}

/* The reference's pk_greedy_decode of one utterance of T frames, products from
 * `fn`. embed [1025, 640], B0 / B1 [5120] (the layers' B), enc_b / pred_b
 * [640], out_b [1025]. Writes up to max_tokens tokens and the number of joint
 * evaluations; returns the number of tokens emitted. The LSTM state is local
 * to pk_greedy_decode: the states it passes through reach the callback as the
 * inputs of the W_r and joint.pred products. */
int pkref_greedy_decode(int T, const float *embed, const float *B0, const float *B1,
                        const float *enc_b, const float *pred_b, const float *out_b,
                        pkh_dec_gemm_fn fn, void *user, int *tokens, int max_tokens,
                        int *n_iters)
{
    PkModel *m = (PkModel *)calloc(1, sizeof(PkModel));
    float *enc = (float *)calloc((size_t)(T > 0 ? T : 1) * PK_D_MODEL, sizeof(float));
    if (!m || !enc) {
        free(m); free(enc);
        return -1;
    }
    DecoderWeights *d = &m->dec;
    d->embed_w = embed;
    d->lstm0_Wi = &g_mats[D_L0_WI]; d->lstm0_Wr = &g_mats[D_L0_WR]; d->lstm0_B = B0;
    d->lstm1_Wi = &g_mats[D_L1_WI]; d->lstm1_Wr = &g_mats[D_L1_WR]; d->lstm1_B = B1;
    d->joint_enc_w = &g_mats[D_ENC]; d->joint_enc_b = enc_b;
    d->joint_pred_w = &g_mats[D_PRED]; d->joint_pred_b = pred_b;
    d->joint_out_w = &g_mats[D_OUT]; d->joint_out_b = out_b;
    g_fn = fn;
    g_user = user;
    g_enc = enc;
    g_iter = 0;
    int *tok = NULL;
    const int n = pk_greedy_decode(m, enc, T, &tok);
    for (int i = 0; i < n && i < max_tokens; i++) tokens[i] = tok[i];
    if (n_iters) *n_iters = g_iter;
    free(tok);
    free(enc);
    free(m);
    return n;
}

/* Products from fixed rows, for timing the reference's non-GEMM decode work
 * alone: enc row t of rows[D_ENC] ([T, 640]), the same row every time for the
 * others (rows[g], g = D_PRED .. D_L1_WR). */
static const float *g_rows[D_N];

static void static_products(void *user, int gemm, int iter, const float *in, int n_in, float *out,
                            int n_out)
{
    (void)user; (void)in; (void)n_in;
    const float *src = gemm == D_ENC ? g_rows[D_ENC] + (size_t)iter * (size_t)n_out : g_rows[gemm];
    memcpy(out, src, sizeof(float) * (size_t)n_out);
}

int pkref_greedy_decode_static(int T, const float *embed, const float *B0, const float *B1,
                               const float *enc_b, const float *pred_b, const float *out_b,
                               const float *const *rows, int *tokens, int max_tokens, int *n_iters)
{
    for (int g = 0; g < D_N; g++) g_rows[g] = rows[g];
    return pkref_greedy_decode(T, embed, B0, B1, enc_b, pred_b, out_b, static_products, NULL,
                               tokens, max_tokens, n_iters);
}
