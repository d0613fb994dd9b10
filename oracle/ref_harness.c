/*  ref_harness.c -- TEST INFRASTRUCTURE ONLY (checker, never shipped).
 *
 *  Compiles the reference engine's own csrc/encoder.c into the reference
 *  library oracle/_ref/libpkref.so (built by oracle/Makefile straight from
 *  the reference tree; nothing from it is copied into this repository).
 *
 *  What it exposes beyond the exported tensor_ops.c / blas.c / threadpool.c
 *  symbols:
 *    - pkref_relative_shift: the static relative_shift() of
 *      csrc/encoder.c:230-254, in place on bd [H, T, 2T-1].
 *    - pkref_conformer_block: the static conformer_block() of
 *      csrc/encoder.c:482-491 run with every GEMM entry point it reaches
 *      (pk_wmatmul csrc/tensor_ops.c:50, cblas_sgemm_st via
 *      batched_head_gemm csrc/encoder.c:267-293, pk_pointwise_conv1d
 *      csrc/tensor_ops.c:579) redirected to a "stand-in" that either copies
 *      a caller-supplied GEMM output (mode PKH_COPY) or leaves the output
 *      buffer untouched (mode PKH_NOOP, used to time the non-GEMM work
 *      alone).  All non-GEMM code that runs is the reference's own.
 *
 *  In PKH_COPY mode every stand-in GEMM also records its input operands (the
 *  LN outputs, Swish outputs, Q+u / Q+v / K / V / P heads, softmax scores,
 *  head concat, channel-first LN and the depthwise-conv output) into the
 *  caller's capture buffers: those are the reference's own intermediates.
 *
 *  Stand-in order inside one conformer_block (csrc/encoder.c:486-490):
 *    wmatmul #0 FF1 linear1 -> h   [T,4096]      #1 FF1 linear2 -> out [T,1024]
 *    wmatmul #2 fused QKV   -> QKV [T,3072]      #3 pos proj    -> P   [2T-1,1024]
 *    wmatmul #4 out proj    -> out [T,1024]
 *    pointwise #0 pw1 -> [2048,T] (+bias)        pointwise #1 pw2 -> [1024,T] (+bias)
 *    wmatmul #5 FF2 linear1, #6 FF2 linear2
 *    head gemm calls 0..7 ac[h], 8..15 bd[h], 16..23 attn_h[h] (one-thread pool)
 */
#include "parakeet.h"
#include "blas.h"
#include "threadpool.h"
#include <stdlib.h>
#include <string.h>

enum { PKH_NOOP = 0, PKH_COPY = 1 };

/* Roles of the stand-in GEMM outputs, in the order the caller passes them. */
enum {
    PKH_FF1_H = 0, PKH_FF1_OUT, PKH_QKV, PKH_P, PKH_AC, PKH_BD, PKH_ATTN_H,
    PKH_ATT_OUT, PKH_PW1, PKH_PW2, PKH_FF2_H, PKH_FF2_OUT, PKH_N_ROLES
};

/* Captured GEMM inputs, in the order the caller passes them. */
enum {
    CAP_LN_FF1 = 0, CAP_H1, CAP_LN_SA, CAP_QU, CAP_K, CAP_QV, CAP_PH, CAP_S, CAP_V,
    CAP_ATTN, CAP_CF, CAP_DW, CAP_LN_FF2, CAP_H2, CAP_N
};

static int g_mode = PKH_NOOP;
static const float *g_standin[PKH_N_ROLES];
static float *g_capture[CAP_N];
static int g_wm_calls, g_pw_calls, g_hg_calls, g_T;

void pkh_wmatmul(const float *A, const Weight *W, float *C,
                 int M, int N, int K, float alpha, float beta);
void pkh_sgemm_st(CBLAS_ORDER order, CBLAS_TRANSPOSE transA, CBLAS_TRANSPOSE transB,
                  int M, int N, int K, float alpha, const float *A, int lda,
                  const float *B, int ldb, float beta, float *C, int ldc);
void pkh_pointwise_conv1d(const float *x, const float *w, const float *b,
                          float *out, int Cin, int Cout, int T);

void pkh_conv2d(const float *x, const float *w, const float *b, float *out, int Cin, int H,
                int W, int Cout, int Kh, int Kw, int sh, int sw, int ph, int pw, int groups);

#define pk_wmatmul          pkh_wmatmul
#define cblas_sgemm_st      pkh_sgemm_st
#define pk_pointwise_conv1d pkh_pointwise_conv1d
#define pk_conv2d           pkh_conv2d
#include "encoder.c"
#undef pk_wmatmul
#undef cblas_sgemm_st
#undef pk_pointwise_conv1d
#undef pk_conv2d

/* Pre-encode stand-ins (pkref_pre_encode): the two 1x1 convolutions and the
 * output projection of csrc/encoder.c:128-164 are the GEMMs of that stage. */
static int g_pre;
static const float *g_pre_y[3];   /* pw1 [256, P2], pw2 [256, P3], proj [T', 1024] */
static float *g_pre_cap[3];       /* their inputs: [256, P2], [256, P3], [T', 4096] */
static int g_pre_pw;

static void copy_rows(float *C, int ldc, const float *src, int M, int N)
{
    for (int i = 0; i < M; i++)
        memcpy(C + (size_t)i * ldc, src + (size_t)i * N, (size_t)N * sizeof(float));
}

static void capture_rows_dense(float *dst, const float *src, int ld, int M, int N)
{
    for (int i = 0; i < M; i++)
        memcpy(dst + (size_t)i * N, src + (size_t)i * ld, (size_t)N * sizeof(float));
}

/* Copies an [M, N] operand with leading dimension ld into a dense buffer. */
static void capture(int role, size_t off, const float *src, int ld, int M, int N)
{
    float *dst = g_capture[role];
    if (!dst) return;
    for (int i = 0; i < M; i++)
        memcpy(dst + off + (size_t)i * N, src + (size_t)i * ld, (size_t)N * sizeof(float));
}

/* pk_conv2d (csrc/tensor_ops.c:439-475) as pre_encode calls it: the reference's
 * own code for the 3x3 convolutions; during pkref_pre_encode the 1x1
 * convolutions become stand-ins, out = GEMM output + bias (the bias the
 * reference's loop starts from), with their input captured. */
void pkh_conv2d(const float *x, const float *w, const float *b, float *out, int Cin, int H,
                int W, int Cout, int Kh, int Kw, int sh, int sw, int ph, int pw, int groups)
{
    if (g_pre && Kh == 1 && Kw == 1 && groups == 1 && g_pre_pw < 2) {
        const int k = g_pre_pw++;
        const size_t P = (size_t)H * W;
        if (g_pre_cap[k]) memcpy(g_pre_cap[k], x, (size_t)Cin * P * sizeof(float));
        for (int oc = 0; oc < Cout; oc++)
            for (size_t p = 0; p < P; p++)
                out[oc * P + p] = g_pre_y[k][oc * P + p] + b[oc];
        return;
    }
    pk_conv2d(x, w, b, out, Cin, H, W, Cout, Kh, Kw, sh, sw, ph, pw, groups);
}

void pkh_wmatmul(const float *A, const Weight *W, float *C,
                 int M, int N, int K, float alpha, float beta)
{
    if (g_pre) {   /* pre_encode's output projection */
        if (g_pre_cap[2]) capture_rows_dense(g_pre_cap[2], A, K, M, K);
        copy_rows(C, N, g_pre_y[2], M, N);
        return;
    }
    static const int role_of_call[7] = {
        PKH_FF1_H, PKH_FF1_OUT, PKH_QKV, PKH_P, PKH_ATT_OUT, PKH_FF2_H, PKH_FF2_OUT
    };
    static const int capture_of_call[7] = {
        CAP_LN_FF1, CAP_H1, CAP_LN_SA, -1, CAP_ATTN, CAP_LN_FF2, CAP_H2
    };
    (void)W; (void)alpha; (void)beta;
    int call = g_wm_calls++;
    if (g_mode == PKH_COPY && call < 7) {
        if (capture_of_call[call] >= 0) capture(capture_of_call[call], 0, A, K, M, K);
        copy_rows(C, N, g_standin[role_of_call[call]], M, N);
    }
}

void pkh_sgemm_st(CBLAS_ORDER order, CBLAS_TRANSPOSE transA, CBLAS_TRANSPOSE transB,
                  int M, int N, int K, float alpha, const float *A, int lda,
                  const float *B, int ldb, float beta, float *C, int ldc)
{
    (void)order; (void)transA; (void)transB; (void)alpha; (void)beta;
    if (g_mode != PKH_COPY) return;
    int call = __atomic_fetch_add(&g_hg_calls, 1, __ATOMIC_RELAXED);
    int role = call / PK_N_HEADS, h = call % PK_N_HEADS;
    int T = g_T, L = 2 * T - 1, Dh = PK_HEAD_DIM;
    const float *src;
    if (role == 0) {            /* ac = Q_u K^T: A [T,Dh], B [T,Dh] (transposed) */
        capture(CAP_QU, (size_t)h * T * Dh, A, lda, M, K);
        capture(CAP_K, (size_t)h * T * Dh, B, ldb, N, K);
        src = g_standin[PKH_AC] + (size_t)h * T * T;
    } else if (role == 1) {     /* bd = Q_v P^T: A [T,Dh], B [2T-1,Dh] (transposed) */
        capture(CAP_QV, (size_t)h * T * Dh, A, lda, M, K);
        capture(CAP_PH, (size_t)h * L * Dh, B, ldb, N, K);
        src = g_standin[PKH_BD] + (size_t)h * T * L;
    } else {                    /* attn_h = S V: A [T,T], B [T,Dh] */
        capture(CAP_S, (size_t)h * T * T, A, lda, M, K);
        capture(CAP_V, (size_t)h * T * Dh, B, ldb, K, N);
        src = g_standin[PKH_ATTN_H] + (size_t)h * T * Dh;
    }
    copy_rows(C, ldc, src, M, N);
}

void pkh_pointwise_conv1d(const float *x, const float *w, const float *b,
                          float *out, int Cin, int Cout, int T)
{
    (void)w;
    int call = g_pw_calls++;
    if (g_mode != PKH_COPY) return;
    capture(call == 0 ? CAP_CF : CAP_DW, 0, x, T, Cin, T);
    memcpy(out, g_standin[call == 0 ? PKH_PW1 : PKH_PW2], (size_t)Cout * T * sizeof(float));
    /* The bias loop that follows the GEMM (csrc/tensor_ops.c:585-589). */
    if (b)
        for (int c = 0; c < Cout; c++)
            for (int t = 0; t < T; t++)
                out[c * T + t] += b[c];
}

/* ── Exports ─────────────────────────────────────────────────────────────── */

size_t pkref_ws_floats(int T) { return conformer_ws_peak(T); }

/* relative_shift (csrc/encoder.c:230-254): bd [H,T,2T-1] -> first H*T*T floats. */
int pkref_relative_shift(float *bd, int H, int T)
{
    size_t n = (size_t)H * T * (2 * T) + (size_t)H * T * T;
    float *ws = (float *)malloc(n * sizeof(float));
    if (!ws) return -1;
    WSA a = {ws, 0};
    relative_shift(bd, H, T, &a);
    free(ws);
    return 0;
}

/* Non-GEMM parameters of one block, in this order (all fp32):
 *   0 norm_ff1_w  1 norm_ff1_b  2 ff1.linear1_b  3 ff1.linear2_b
 *   4 norm_sa_w   5 norm_sa_b   6 linear_qkv_b   7 pos_bias_u  8 pos_bias_v
 *   9 linear_out_b
 *  10 norm_conv_w 11 norm_conv_b 12 pw1_b 13 dw_w 14 dw_b 15 pw2_b
 *  16 norm_ff2_w 17 norm_ff2_b 18 ff2.linear1_b 19 ff2.linear2_b
 *  20 norm_out_w 21 norm_out_b */
#define PKH_N_PARAMS 22

static void fill_block(ConformerBlock *blk, const float *const *p)
{
    memset(blk, 0, sizeof(*blk));
    blk->norm_ff1_w = p[0];  blk->norm_ff1_b = p[1];
    blk->ff1.linear1_b = p[2]; blk->ff1.linear2_b = p[3];
    blk->norm_sa_w = p[4];   blk->norm_sa_b = p[5];
    blk->mha.linear_qkv_b = (float *)p[6];
    blk->mha.pos_bias_u = p[7]; blk->mha.pos_bias_v = p[8];
    blk->mha.linear_out_b = p[9];
    blk->norm_conv_w = p[10]; blk->norm_conv_b = p[11];
    blk->conv.pw1_b = p[12]; blk->conv.dw_w = p[13]; blk->conv.dw_b = p[14];
    blk->conv.pw2_b = p[15];
    blk->norm_ff2_w = p[16]; blk->norm_ff2_b = p[17];
    blk->ff2.linear1_b = p[18]; blk->ff2.linear2_b = p[19];
    blk->norm_out_w = p[20]; blk->norm_out_b = p[21];
}

static ThreadPool *g_one_pool;

/* Runs n_blocks reference conformer blocks on x [T,1024] in place.
 *   params   : n_blocks * 22 pointers (block-major), see fill_block
 *   standins : 12 pointers (PKH_* roles), used when mode == PKH_COPY
 *   captures : 14 pointers (CAP_* roles, NULL entries skipped) or NULL
 *   ws       : conformer_ws_peak(T) floats, or NULL to allocate
 * In PKH_COPY mode the call runs on a private one-thread pool so the head
 * GEMM stand-ins are consumed in order. Not re-entrant. */
int pkref_conformer_blocks(float *x, int T, int n_blocks,
                           const float *const *params,
                           const float *const *standins,
                           float *const *captures, int mode, float *ws)
{
    CfmWS w;
    w.cap = conformer_ws_peak(T);
    w.buf = ws ? ws : (float *)calloc(w.cap, sizeof(float));
    if (!w.buf) return -1;
    g_mode = mode;
    g_T = T;
    for (int r = 0; r < PKH_N_ROLES; r++) g_standin[r] = standins ? standins[r] : NULL;
    for (int r = 0; r < CAP_N; r++) g_capture[r] = captures ? captures[r] : NULL;
    if (mode == PKH_COPY) {
        if (!g_one_pool) g_one_pool = pk_pool_create(1);
        pk_set_pool(g_one_pool);
    }
    for (int i = 0; i < n_blocks; i++) {
        ConformerBlock blk;
        fill_block(&blk, params + (size_t)i * PKH_N_PARAMS);
        g_wm_calls = g_pw_calls = g_hg_calls = 0;
        conformer_block(&blk, x /* pe_slice: only read by the stand-in GEMM */, x, T, &w);
    }
    if (mode == PKH_COPY) pk_set_pool(NULL);
    if (!ws) free(w.buf);
    return 0;
}

/* Loads weights through the reference loader pk_load_weights
 * (csrc/weights.c:268-549) and returns block 0's fused QKV weight
 * [1024, 3072]: int8 after the common-scale requantisation (bits 8) or fp32
 * (bits 32). scales_out[0..3] = sq, sk, sv as parsed, and the fused scale. */
int pkref_load_fused_qkv(const char *bin_path, const char *json_path, void *out,
                         size_t out_bytes, float *scales_out, int *bits_out)
{
    PkModel *m = (PkModel *)calloc(1, sizeof(PkModel));
    if (!m) return -1;
    if (pk_load_weights(m, bin_path, json_path) != 0) { free(m); return -1; }
    const MHAWeights *mha = &m->enc.blocks[0].mha;
    const Weight *w = &mha->linear_qkv_w;
    size_t n = (size_t)PK_D_MODEL * 3 * PK_D_MODEL, need = w->bits == 8 ? n : n * sizeof(float);
    int rc = 0;
    if (!w->data || out_bytes < need) rc = -2;
    else {
        memcpy(out, w->data, need);
        scales_out[0] = mha->linear_q_w.scale;
        scales_out[1] = mha->linear_k_w.scale;
        scales_out[2] = mha->linear_v_w.scale;
        scales_out[3] = w->scale;
        *bits_out = w->bits;
    }
    pk_free_weights(m);
    free(m);
    return rc;
}

/* The reference's pre-encode and scaling (csrc/encoder.c:103-175, 578-593) for
 * one utterance of T mel frames (mel [128, T]): pre_encode_and_scale with the
 * two 1x1 convolutions and the output projection as stand-ins (y2 [256, P2],
 * y3 [256, P3], proj [T', 1024], P = rows x width after each stride-2 stage)
 * whose inputs are captured (s2d, s3d, flat; any may be NULL). params: conv0_w,
 * conv0_b, conv2_w, conv2_b, conv3_b, conv5_w, conv5_b, conv6_b, out_b.
 * x_out [T', 1024]. Returns T', or -1. */
int pkref_pre_encode(const float *mel, int T, const float *const *params, const float *y2,
                     const float *y3, const float *proj, float *s2d, float *s3d, float *flat,
                     float *x_out)
{
    PkModel *m = (PkModel *)calloc(1, sizeof(PkModel));
    if (!m) return -1;
    PreEncodeWeights *w = &m->enc.pre_encode;
    w->conv0_w = params[0]; w->conv0_b = params[1];
    w->conv2_w = params[2]; w->conv2_b = params[3];
    w->conv3_b = params[4];
    w->conv5_w = params[5]; w->conv5_b = params[6];
    w->conv6_b = params[7];
    w->out_b = params[8];
    g_pre = 1;
    g_pre_pw = 0;
    g_pre_y[0] = y2; g_pre_y[1] = y3; g_pre_y[2] = proj;
    g_pre_cap[0] = s2d; g_pre_cap[1] = s3d; g_pre_cap[2] = flat;
    float *x = NULL;
    const int Tp = pre_encode_and_scale(m, mel, T, &x);
    g_pre = 0;
    if (x) {
        memcpy(x_out, x, (size_t)Tp * PK_D_MODEL * sizeof(float));
        free(x);
    }
    free(m);
    return x ? Tp : -1;
}

/* Number of threads the process-wide reference pool runs with (PK_THREADS). */
int pkref_pool_threads(void) { return pk_pool_nthreads(pk_pool()); }
