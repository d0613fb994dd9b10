/* pk_encoder_model.c -- the whole encoder stack on the GPU: the fused non-GEMM
 * block sequence (pkcu_encoder_nongemm) with its twelve GEMM points served by
 * the library itself, on the weights of an uploaded checkpoint.
 *
 * Every GEMM weight of every block is made an fp32 device copy once
 * (pkcu_weights_dequant: int8 (float)q * scale, int4 (float)nibble * group
 * scale, fp32 copied; the fused QKV as the reference's loader builds it), so a
 * forward pass is fp32 throughout like the reference's (csrc/encoder.c). The
 * row-major projections of the block (FF, QKV, output, and the positional
 * projection of the sinusoidal table's slice, csrc/encoder.c:220-227, once per
 * distinct utterance length) run on the library's tcgen05 GEMM (k_tcgemm.cu)
 * with fp32 accuracy: an int8 weight used as stored (q exact in bf16, its
 * scale applied to the sum), any other as the three bf16 parts of its fp32
 * values, the activation as three bf16 parts; the pointwise convolutions on it
 * too (the first one's GLU and the second one's residual in its epilogues),
 * and the per-head score, positional-score and context products as batched
 * launches over heads (and over utterances when the batch is uniform) with
 * both operands split. cuBLAS single-precision GEMMs remain only for a model
 * that could not hold the GEMM's operands. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <stdint.h>

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include "pkcuda_internal.h"

#define PE_CENTER 4999   /* row of relative position 0 (csrc/parakeet.h:127-128) */
#define PE_ROWS 9999

enum { W_FF1_1, W_FF1_2, W_QKV, W_POS, W_OUT, W_PW1, W_PW2, W_FF2_1, W_FF2_2, W_N };

static const char *const W_NAME[W_N] = {
    "feed_forward1.linear1.weight", "feed_forward1.linear2.weight", NULL,
    "self_attn.linear_pos.weight", "self_attn.linear_out.weight",
    "conv.pointwise_conv1.weight", "conv.pointwise_conv2.weight",
    "feed_forward2.linear1.weight", "feed_forward2.linear2.weight"};
static const long long W_ELEMS[W_N] = {
    (long long)PK_D * PK_FF, (long long)PK_FF * PK_D, (long long)PK_D * 3 * PK_D,
    (long long)PK_D * PK_D, (long long)PK_D * PK_D, 2LL * PK_D * PK_D, (long long)PK_D * PK_D,
    (long long)PK_D * PK_FF, (long long)PK_FF * PK_D};

/* [K, N] of each weight as the product x W reads it (row-major, [in, out]). */
static const int W_K[W_N] = {PK_D, PK_FF, PK_D, PK_D, PK_D, PK_D, PK_D, PK_D, PK_FF};
static const int W_COLS[W_N] = {PK_FF, PK_D, 3 * PK_D, PK_D, PK_D, 2 * PK_D, PK_D, PK_FF, PK_D};
/* Every block weight runs on the tcgen05 GEMM (k_tcgemm.cu) as K-major bf16
 * planes: 1 = a row-major projection's [K, N] weight, transposed to [N, K]
 * (int8: q; else three parts); 2 = a pointwise convolution's [out, in] weight,
 * three parts as it is (the first one's rows interleaved value / gate). */
static const int W_SPLIT[W_N] = {1, 1, 1, 1, 1, 2, 2, 1, 1};

struct pkcu_encoder_model {
    int device, n_blocks;
    cublasHandle_t blas;
    float *arena;                      /* fp32 GEMM weights, block after block */
    const float *w[64][W_N];
    pkcu_block_params params[64];
    const float *pe;                   /* pos_encoding.pe_table [9999, 1024] */
    void *stacks;                      /* bf16 operands of the W_SPLIT weights */
    const void *stack[64][W_N];        /* K-major planes [N, K] (int8 q) or [N, 3K] (three parts);
                                          NULL: the fp32 path */
    float qscale[64][W_N];             /* > 0: the int8 weight's scale, w = q x this */
    void *split_ws;                    /* activation parts [rows, 3K] bf16, grown per forward */
    size_t split_cap;                  /* its bytes */
    void *hsplit_ws;                   /* the FF hidden layer's parts [rows, 3 x 4096], written by
                                          the first FF product's epilogue (fused forward) */
    size_t hsplit_cap;
};

void pkcu_encoder_model_destroy(pkcu_encoder_model *m)
{
    if (!m) return;
    if (m->blas) cublasDestroy(m->blas);
    if (m->arena) cudaFree(m->arena);
    if (m->stacks) cudaFree(m->stacks);
    if (m->split_ws) cudaFree(m->split_ws);
    if (m->hsplit_ws) cudaFree(m->hsplit_ws);
    free(m);
}

static long long block_elems(void)
{
    long long n = 0;
    for (int k = 0; k < W_N; k++) n += W_ELEMS[k];
    return n;
}

/* Block b's weight k as stored when it is int8 with one per-tensor scale (the
 * reference's int8 projections; the fused QKV at its common scale): the device
 * int8 [K, N] and the scale, else NULL. */
static const int8_t *int8_source(const pkcu_weights *w, int b, int k, float *scale)
{
    if (k == W_QKV) {
        const void *qw;
        int bits;
        const float *qb;
        if (pkcu_weights_fused_qkv(w, b, &qw, &bits, scale, &qb) == PKCU_OK && bits == 8)
            return (const int8_t *)qw;
        return NULL;
    }
    char name[128];
    pkcu_tensor t;
    snprintf(name, sizeof(name), "layers.%d.%s", b, W_NAME[k]);
    if (pkcu_weights_find(w, name, &t) == PKCU_OK && t.dtype == PKCU_DTYPE_I8 && t.dev &&
        t.numel == W_ELEMS[k] && t.scale > 0.f) {
        *scale = t.scale;
        return (const int8_t *)t.dev;
    }
    return NULL;
}

/* The bf16 operands of the split-operand GEMMs: an int8 projection weight as
 * its q (exact in bf16, 2 bytes per element; the scale goes into the GEMM's
 * alpha), any other W_SPLIT weight as its three parts (6 bytes per element).
 * Without the memory for them the model keeps the fp32 path. */
static int build_stacks(pkcu_encoder_model *m, const pkcu_weights *w, long long per, pkcu_stream_t stream)
{
    long long bytes = 0;
    for (int b = 0; b < m->n_blocks; b++)
        for (int k = 0; k < W_N; k++) {
            float sc;
            if (W_SPLIT[k]) bytes += (W_SPLIT[k] == 1 && int8_source(w, b, k, &sc) ? 2 : 6) * W_ELEMS[k];
        }
    if (cudaMalloc(&m->stacks, (size_t)bytes) != cudaSuccess) {
        cudaGetLastError();
        m->stacks = NULL;
        return PKCU_OK;
    }
    char *p = (char *)m->stacks;
    for (int b = 0; b < m->n_blocks; b++) {
        const float *src = m->arena + per * b;
        for (int k = 0; k < W_N; k++) {
            if (W_SPLIT[k]) {
                float sc = 0.f;
                const int8_t *q = W_SPLIT[k] == 1 ? int8_source(w, b, k, &sc) : NULL;
                int st;
                if (W_SPLIT[k] == 1) {
                    /* K-major planes for the library's tcgen05 GEMM: q of an
                     * int8 weight (its scale as the GEMM's alpha), else the
                     * three parts of the fp32 values */
                    float alpha = 1.0f;
                    st = q ? pk_tc_prepare(q, 8, sc, W_K[k], W_COLS[k], p, &alpha, stream)
                           : pk_tc_prepare(src, 32, 0.0f, W_K[k], W_COLS[k], p, &alpha, stream);
                    m->qscale[b][k] = q ? alpha : 0.0f;
                } else {
                    /* a pointwise weight is [out channels, 1024] (W_COLS x W_K),
                     * already K-major: three-part planes, the first conv's rows
                     * interleaved value / gate for its GLU epilogue */
                    st = pk_tc_prepare_rows(src, W_COLS[k], W_K[k], k == W_PW1, p, stream);
                }
                if (st) return st;
                m->stack[b][k] = p;
                p += (q ? 2 : 6) * W_ELEMS[k];
            }
            src += W_ELEMS[k];
        }
    }
    return PKCU_OK;
}

int pkcu_encoder_model_create(const pkcu_weights *w, pkcu_stream_t stream, pkcu_encoder_model **out)
{
    if (!out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_model_create: NULL out");
    *out = NULL;
    if (!w) return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_model_create: NULL weights");
    const int nb = pkcu_weights_blocks(w);
    if (nb <= 0 || nb > 64)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_model_create: %d blocks (1 .. 64)", nb);
    pkcu_tensor pe;
    int st = pkcu_weights_find(w, "pos_encoding.pe_table", &pe);
    if (st) return st;
    if (pe.dtype != PKCU_DTYPE_F32 || pe.numel != (long long)PE_ROWS * PK_D || !pe.dev)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_model_create: pos_encoding.pe_table is not "
                                       "a float32 [9999, 1024] table on the device");
    pkcu_encoder_model *m = (pkcu_encoder_model *)calloc(1, sizeof(*m));
    if (!m) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_encoder_model_create: host allocation");
    cudaGetDevice(&m->device);
    m->n_blocks = nb;
    m->pe = (const float *)pe.dev;
    if (cublasCreate(&m->blas) != CUBLAS_STATUS_SUCCESS) {
        m->blas = NULL;
        pkcu_encoder_model_destroy(m);
        return pkcu_fail(PKCU_ERR_CUDA, "pkcu_encoder_model_create: cublasCreate failed");
    }
    const long long per = block_elems();
    if (cudaMalloc((void **)&m->arena, sizeof(float) * (size_t)(per * nb)) != cudaSuccess) {
        cudaGetLastError();
        m->arena = NULL;
        pkcu_encoder_model_destroy(m);
        return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_encoder_model_create: %lld bytes of fp32 weights",
                         (long long)sizeof(float) * per * nb);
    }
    char name[128];
    for (int b = 0; b < nb; b++) {
        float *p = m->arena + per * b;
        for (int k = 0; k < W_N; k++) {
            m->w[b][k] = p;
            if (k == W_QKV) {
                const void *qw;
                int bits;
                float scale;
                const float *qb;
                st = pkcu_weights_fused_qkv(w, b, &qw, &bits, &scale, &qb);
                if (!st && bits == 8)
                    st = pkcu_dequant_i8((const int8_t *)qw, scale, p, W_ELEMS[k], stream);
                else if (!st)
                    st = cudaMemcpyAsync(p, qw, sizeof(float) * (size_t)W_ELEMS[k],
                                         cudaMemcpyDeviceToDevice, (cudaStream_t)stream) == cudaSuccess
                             ? PKCU_OK : pkcu_launch_status("pkcu_encoder_model_create: fused QKV");
            } else {
                pkcu_tensor t;
                snprintf(name, sizeof(name), "layers.%d.%s", b, W_NAME[k]);
                st = pkcu_weights_find(w, name, &t);
                if (!st && t.numel != W_ELEMS[k])
                    st = pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_model_create: '%s' has %lld elements, "
                                                 "expected %lld", name, t.numel, W_ELEMS[k]);
                if (!st) st = pkcu_weights_dequant(w, name, p, stream);
            }
            if (st) {
                pkcu_encoder_model_destroy(m);
                return st;
            }
            p += W_ELEMS[k];
        }
        st = pkcu_weights_block_params(w, b, &m->params[b]);
        if (st) {
            pkcu_encoder_model_destroy(m);
            return st;
        }
    }
    st = build_stacks(m, w, per, stream);
    if (st) {
        pkcu_encoder_model_destroy(m);
        return st;
    }
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) {
        pkcu_encoder_model_destroy(m);
        return pkcu_launch_status("pkcu_encoder_model_create");
    }
    *out = m;
    return PKCU_OK;
}

int pkcu_encoder_model_blocks(const pkcu_encoder_model *m) { return m ? m->n_blocks : 0; }

/* ── the GEMM hook ─────────────────────────────────────────────────────────── */

typedef struct {
    pkcu_encoder_model *m;
    const pkcu_gemm_outputs *go;
    const pkcu_gemm_inputs *gi;
    const pkcu_seq *seq;
    long long *off;   /* per item: frame, pos row, score, bd element offsets (4 x n_items) */
    unsigned fused;   /* PKCU_FUSED_* epilogues the hook's GEMMs apply */
    float *x;         /* the residual stream (the fused PW2 epilogue adds to it) */
    void *hsplit;     /* fused: the FF hidden layer as bf16 parts (gemm_in h1 / h2 not written) */
} Fwd;

static const float ONE = 1.0f, ZERO = 0.0f;

/* The GEMM output buffers are const in pkcu_gemm_outputs (the non-GEMM
 * kernels only read them); the GEMM hook is what writes them. */
static float *gemm_dst(const float *p) { return (float *)p; }

/* Row-major C[M, N] = A[M, K] B[K, N] (leading dimensions lda, ldb, ldc),
 * as the column-major product C^T = B^T A^T; tb: B is stored [N, K] (C = A B^T). */
static int rm_gemm(cublasHandle_t h, int M, int N, int K, const float *A, int lda, long long sA,
                   const float *B, int ldb, long long sB, int tb, float *C, int ldc, long long sC,
                   int batch)
{
    const cublasStatus_t s = cublasSgemmStridedBatched(
        h, tb ? CUBLAS_OP_T : CUBLAS_OP_N, CUBLAS_OP_N, N, M, K, &ONE, B, ldb, sB, A, lda, sA, &ZERO,
        C, ldc, sC, batch);
    return s == CUBLAS_STATUS_SUCCESS ? PKCU_OK
                                      : pkcu_fail(PKCU_ERR_CUDA, "cuBLAS SGEMM failed (%d)", (int)s);
}

/* Row-major projection of the whole batch: the fp32-accurate tensor-core GEMM
 * when the shape suits it, cuBLAS SGEMM otherwise. */
static int proj(cublasHandle_t h, int M, int N, int K, const float *A, const float *B, float *C,
                pkcu_stream_t stream)
{
    if (pk_gemm_f32_rm(A, B, C, M, N, K, stream) == PKCU_OK) return PKCU_OK;
    return rm_gemm(h, M, N, K, A, K, 0, B, N, 0, 0, C, N, 0, 1);
}

/* The block's row-major projection on the library's tcgen05 GEMM: the
 * activation's three parts into the model's workspace, then the product with
 * the weight's K-major planes (an int8 weight's q with its scale as alpha, or
 * the three parts of fp32 values); the fp32 tensor-core GEMM when the model
 * could not hold the planes. */
static int proj_tc(pkcu_encoder_model *m, int b, int k, int M, const float *A, pk_tc_epi *e,
                   pkcu_stream_t stream)
{
    if ((size_t)M * 3 * W_K[k] * 2 > m->split_cap)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_forward: split workspace too small");
    int st = pk_split_rows_bf16x3(A, m->split_ws, M, W_K[k], stream);
    if (st) return st;
    e->alpha = m->qscale[b][k] > 0.f ? m->qscale[b][k] : 1.0f;
    return pk_tc_gemm(m->split_ws, m->stack[b][k], m->qscale[b][k] > 0.f ? 1 : 3, M, W_COLS[k], W_K[k], e,
                      stream);
}

static int proj_w(pkcu_encoder_model *m, cublasHandle_t h, int b, int k, int M, const float *A, float *C,
                  pkcu_stream_t stream)
{
    if (!m->stack[b][k]) return proj(h, M, W_COLS[k], W_K[k], A, m->w[b][k], C, stream);
    pk_tc_epi e;
    memset(&e, 0, sizeof(e));
    e.mode = PK_TC_STORE;
    e.C = C;
    return proj_tc(m, b, k, M, A, &e, stream);
}

/* FF linear1 with its bias and Swish in the GEMM's epilogue, h = Swish(A W + b1),
 * written only as the three bf16 parts that FF linear2 reads (hparts [M, 3 x 4096]):
 * the hidden layer never exists in fp32 and needs no split pass. */
static int proj_swish(pkcu_encoder_model *m, int b, int k, int M, const float *A, const float *b1, void *hparts,
                      pkcu_stream_t stream)
{
    pk_tc_epi e;
    memset(&e, 0, sizeof(e));
    e.mode = PK_TC_SWISH_SPLIT;
    e.bias = b1;
    e.Cb = hparts;
    return proj_tc(m, b, k, M, A, &e, stream);
}

/* Workspace bytes of the per-head products of `per` items of T frames on the
 * tcgen05 GEMM: the larger of the score products' two operands (K / P heads
 * and Q heads, 128 wide) and the context product's (the score rows padded to
 * Kp = T rounded up to 32, and the value heads transposed). */
static size_t heads_need(int T, int per)
{
    const long long Z = (long long)PK_H * per, L = 2LL * T - 1, Kp = (T + 31) & ~31;
    const long long sc = (Z * L + Z * T) * 3 * PK_DH * 2;
    const long long av = (Z * T + Z * PK_DH) * 3 * Kp * 2;
    return (size_t)(sc > av ? sc : av);
}

/* The per-head products of `per` consecutive items of T frames (Z = 8 per
 * entries of one shape, one launch) on the tcgen05 GEMM, both operands split
 * into the model's workspace:
 *   ac[z][i][j] = K[z][j] . Qu[z][i]  (A = K heads, B = Q+u heads, stored transposed)
 *   bd[z][i][j] = P[z][j] . Qv[z][i]  (A = P heads, B = Q+v heads, stored transposed)
 *   attn[z] = S[z] V[z]                (A = score rows padded, B = V heads transposed)
 * The transposed stores put the lanes of a warp on consecutive j. */
static int heads_tc(pkcu_encoder_model *m, int gemm, int T, int per, const pkcu_gemm_inputs *gi,
                    const pkcu_gemm_outputs *go, long long fo, long long po, long long so, long long bo,
                    pkcu_stream_t stream)
{
    const int Z = PK_H * per, L = 2 * T - 1, Kp = (T + 31) & ~31;
    uint16_t *ws = (uint16_t *)m->split_ws;
    pk_tc_epi e;
    memset(&e, 0, sizeof(e));
    e.alpha = 1.0f;
    int st;
    if (gemm == PKCU_GEMM_AC || gemm == PKCU_GEMM_BD) {
        const int ac = gemm == PKCU_GEMM_AC;
        const long long arows = (long long)Z * (ac ? T : L), brows = (long long)Z * T;
        uint16_t *pa = ws, *pb = ws + arows * 3 * PK_DH;
        st = pk_split_rows_bf16x3(ac ? gi->K + fo * PK_D : gi->P_h + po * PK_D, pa, arows, PK_DH, stream);
        if (!st) st = pk_split_rows_bf16x3(ac ? gi->Qu + fo * PK_D : gi->Qv + fo * PK_D, pb, brows, PK_DH, stream);
        if (st) return st;
        e.mode = PK_TC_STORE_T;
        e.C = ac ? gemm_dst(go->ac) + so : gemm_dst(go->bd) + bo;
        e.ldc = ac ? T : L;
        return pk_tc_gemm_batched(pa, arows, pb, brows, ac ? T : L, T, PK_DH, &e, Z, ac ? T : L, T,
                                  (long long)T * (ac ? T : L), stream);
    }
    const long long arows = (long long)Z * T, brows = (long long)Z * PK_DH;
    uint16_t *pa = ws, *pb = ws + arows * 3 * Kp;
    st = pk_split_rows_pad(gi->S + so, pa, arows, T, Kp, stream);
    if (!st) st = pk_split_t_pad(gi->V + fo * PK_D, pb, Z, T, PK_DH, Kp, stream);
    if (st) return st;
    e.mode = PK_TC_STORE;
    e.C = gemm_dst(go->attn_h) + fo * PK_D;
    e.ldc = PK_DH;
    return pk_tc_gemm_batched(pa, arows, pb, brows, T, PK_DH, Kp, &e, Z, T, PK_DH, (long long)T * PK_DH, stream);
}

static int fwd_hook(void *user, int b, int gemm, pkcu_stream_t stream)
{
    Fwd *f = (Fwd *)user;
    cublasHandle_t h = f->m->blas;
    if (cublasSetStream(h, (cudaStream_t)stream) != CUBLAS_STATUS_SUCCESS)
        return pkcu_fail(PKCU_ERR_CUDA, "cublasSetStream failed");
    const float *const *W = f->m->w[b];
    const pkcu_gemm_outputs *go = f->go;
    const pkcu_gemm_inputs *gi = f->gi;
    const int n = f->seq->dev.n_items, uni = f->seq->dev.uniform_T;
    const long long F = f->seq->frames;
    const pkcu_block_params *p = &f->m->params[b];
    if (f->fused) {   /* the projections whose epilogues the sequence leaves to the GEMM */
        switch (gemm) {
        case PKCU_GEMM_FF1_1: return proj_swish(f->m, b, W_FF1_1, (int)F, gi->ln_ff1, p->ff1_b1, f->hsplit, stream);
        case PKCU_GEMM_FF2_1: return proj_swish(f->m, b, W_FF2_1, (int)F, gi->ln_ff2, p->ff2_b1, f->hsplit, stream);
        case PKCU_GEMM_FF1_2:   /* the hidden layer's parts are already in hsplit */
        case PKCU_GEMM_FF2_2: {
            const int k = gemm == PKCU_GEMM_FF1_2 ? W_FF1_2 : W_FF2_2;
            pk_tc_epi e;
            memset(&e, 0, sizeof(e));
            e.mode = PK_TC_STORE;
            e.C = gemm_dst(gemm == PKCU_GEMM_FF1_2 ? go->ff1_out : go->ff2_out);
            e.alpha = f->m->qscale[b][k] > 0.f ? f->m->qscale[b][k] : 1.0f;
            return pk_tc_gemm(f->hsplit, f->m->stack[b][k], f->m->qscale[b][k] > 0.f ? 1 : 3, (int)F,
                              W_COLS[k], W_K[k], &e, stream);
        }
        case PKCU_GEMM_PW1: {   /* gated [1024, T] = GLU(W_pw1 LN_conv + b) from time-first LN rows */
            pk_tc_epi e;
            memset(&e, 0, sizeof(e));
            e.mode = PK_TC_GLU;
            e.bias = p->pw1_b;
            e.C = gi->gated;
            e.seq = f->seq;
            return proj_tc(f->m, b, W_PW1, (int)F, gi->cf, &e, stream);
        }
        case PKCU_GEMM_PW2: {   /* x[t, d] += (W_pw2 dw + b)[d, t], dw channel-first per item */
            Fwd *ff = f;
            if ((size_t)F * 3 * PK_D * 2 > ff->m->split_cap)
                return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_forward: split workspace too small");
            int st = pk_split_cf_t(gi->dw, ff->m->split_ws, PK_D, ff->seq, stream);
            if (st) return st;
            pk_tc_epi e;
            memset(&e, 0, sizeof(e));
            e.mode = PK_TC_RESID;
            e.alpha = 1.0f;
            e.rscale = 1.0f;
            e.bias = p->pw2_b;
            e.C = ff->x;
            return pk_tc_gemm(ff->m->split_ws, ff->m->stack[b][W_PW2], 3, (int)F, PK_D, PK_D, &e, stream);
        }
        case PKCU_GEMM_QKV: {
            pk_tc_epi e;
            memset(&e, 0, sizeof(e));
            e.mode = PK_TC_QKV;
            e.bias = p->qkv_b;
            e.u = p->pos_u;
            e.v = p->pos_v;
            e.Qu = gi->Qu;
            e.Qv = gi->Qv;
            e.K = gi->K;
            e.V = gi->V;
            e.seq = f->seq;
            return proj_tc(f->m, b, W_QKV, (int)F, gi->ln_sa, &e, stream);
        }
        default: break;
        }
    }
    switch (gemm) {   /* the row-major projections of the whole batch */
    case PKCU_GEMM_FF1_1: return proj_w(f->m, h, b, W_FF1_1, (int)F, gi->ln_ff1, gemm_dst(go->ff1_h), stream);
    case PKCU_GEMM_FF1_2: return proj_w(f->m, h, b, W_FF1_2, (int)F, gi->h1, gemm_dst(go->ff1_out), stream);
    case PKCU_GEMM_QKV:   return proj_w(f->m, h, b, W_QKV, (int)F, gi->ln_sa, gemm_dst(go->qkv), stream);
    case PKCU_GEMM_OUT:   return proj_w(f->m, h, b, W_OUT, (int)F, gi->attn, gemm_dst(go->att_out), stream);
    case PKCU_GEMM_FF2_1: return proj_w(f->m, h, b, W_FF2_1, (int)F, gi->ln_ff2, gemm_dst(go->ff2_h), stream);
    case PKCU_GEMM_FF2_2: return proj_w(f->m, h, b, W_FF2_2, (int)F, gi->h2, gemm_dst(go->ff2_out), stream);
    default: break;
    }
    if (gemm == PKCU_GEMM_POS) {
        /* P = pe slice [2T-1, 1024] x W_pos depends on T only: one projection
         * per distinct length, copied to the other items of that length */
        for (int i = 0; i < n; i++) {
            const int T = f->seq->lengths[i], L = 2 * T - 1;
            float *dst = gemm_dst(go->P) + f->off[4 * i + 1] * PK_D;
            int j = 0;
            while (j < i && f->seq->lengths[j] != T) j++;
            int st;
            if (j < i) {
                st = cudaMemcpyAsync(dst, go->P + f->off[4 * j + 1] * PK_D, sizeof(float) * (size_t)L * PK_D,
                                     cudaMemcpyDeviceToDevice, (cudaStream_t)stream) == cudaSuccess
                         ? PKCU_OK : pkcu_fail(PKCU_ERR_CUDA, "pkcu_encoder_forward: positional copy");
            } else {
                const float *pe = f->m->pe + (long long)(PE_CENTER - T + 1) * PK_D;
                st = proj_w(f->m, h, b, W_POS, L, pe, dst, stream);
            }
            if (st) return st;
        }
        return PKCU_OK;
    }
    /* per utterance (all utterances in one batch when the lengths agree) */
    const int groups = uni ? 1 : n, per = uni ? n : 1;
    for (int i = 0; i < groups; i++) {
        const int T = uni ? uni : f->seq->lengths[i], L = 2 * T - 1, Hb = PK_H * per;
        const long long fo = f->off[4 * i], po = f->off[4 * i + 1], so = f->off[4 * i + 2],
                        bo = f->off[4 * i + 3];
        int st = PKCU_OK;
        if ((gemm == PKCU_GEMM_AC || gemm == PKCU_GEMM_BD || gemm == PKCU_GEMM_AV) && f->m->stacks &&
            heads_need(T, per) <= f->m->split_cap) {
            st = heads_tc(f->m, gemm, T, per, gi, go, fo, po, so, bo, stream);
            if (st) return st;
            continue;
        }
        switch (gemm) {
        case PKCU_GEMM_AC:    /* ac[h] = (Q + u)[h] K[h]^T */
            st = rm_gemm(h, T, T, PK_DH, gi->Qu + fo * PK_D, PK_DH, (long long)T * PK_DH,
                         gi->K + fo * PK_D, PK_DH, (long long)T * PK_DH, 1, gemm_dst(go->ac) + so, T,
                         (long long)T * T, Hb);
            break;
        case PKCU_GEMM_BD:    /* bd[h] = (Q + v)[h] P[h]^T (P heads [8, 2T-1, 128] per utterance) */
            st = rm_gemm(h, T, L, PK_DH, gi->Qv + fo * PK_D, PK_DH, (long long)T * PK_DH,
                         gi->P_h + po * PK_D, PK_DH, (long long)L * PK_DH, 1, gemm_dst(go->bd) + bo, L,
                         (long long)T * L, Hb);
            break;
        case PKCU_GEMM_AV:    /* attn[h] = S[h] V[h] */
            st = rm_gemm(h, T, PK_DH, T, gi->S + so, T, (long long)T * T, gi->V + fo * PK_D, PK_DH,
                         (long long)T * PK_DH, 0, gemm_dst(go->attn_h) + fo * PK_D, PK_DH, (long long)T * PK_DH, Hb);
            break;
        case PKCU_GEMM_PW1:   /* [2048, T] = W_pw1 [2048, 1024] x cf [1024, T] (fp32 path) */
            st = rm_gemm(h, 2 * PK_D, T, PK_D, W[W_PW1], PK_D, 0, gi->cf + fo * PK_D, T,
                         (long long)PK_D * T, 0, gemm_dst(go->pw1) + fo * 2 * PK_D, T, 2LL * PK_D * T, per);
            break;
        case PKCU_GEMM_PW2:   /* [1024, T] = W_pw2 x dw [1024, T] (fp32 path) */
            st = rm_gemm(h, PK_D, T, PK_D, W[W_PW2], PK_D, 0, gi->dw + fo * PK_D, T,
                         (long long)PK_D * T, 0, gemm_dst(go->pw2) + fo * PK_D, T, (long long)PK_D * T, per);
            break;
        default:
            return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_forward: unknown GEMM %d", gemm);
        }
        if (st) return st;
    }
    return PKCU_OK;
}

int pkcu_encoder_forward(pkcu_encoder_model *m, float *x, const pkcu_gemm_outputs *gemm_out,
                         const pkcu_gemm_inputs *gemm_in, const pkcu_seq *seq, pkcu_stream_t stream)
{
    if (!m || !x || !gemm_out || !gemm_in || !seq)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_forward: NULL argument");
    const int n = seq->dev.n_items;
    for (int i = 0; i < n; i++)
        if (seq->lengths[i] > PE_CENTER + 1)
            return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_forward: item %d has %d frames (the "
                                           "positional table covers %d)", i, seq->lengths[i],
                             PE_CENTER + 1);
    long long *off = (long long *)malloc(sizeof(long long) * 4 * (size_t)n);
    if (!off) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_encoder_forward: host allocation");
    long long acc[4] = {0, 0, 0, 0};
    for (int i = 0; i < n; i++) {
        const long long T = seq->lengths[i];
        memcpy(off + 4 * i, acc, sizeof(acc));
        acc[0] += T;
        acc[1] += 2 * T - 1;
        acc[2] += (long long)PK_H * T * T;
        acc[3] += (long long)PK_H * T * (2 * T - 1);
    }
    /* the activation parts of the largest projection: F rows of K = 4096, or
     * 2T - 1 positional rows of K = 1024 */
    long long rows_ff = 0, rows_pos = 0;
    for (int i = 0; i < n; i++) {
        rows_ff += seq->lengths[i];
        if (2LL * seq->lengths[i] - 1 > rows_pos) rows_pos = 2LL * seq->lengths[i] - 1;
    }
    size_t need = (size_t)rows_ff * 3 * PK_FF * 2;
    if ((size_t)rows_pos * 3 * PK_D * 2 > need) need = (size_t)rows_pos * 3 * PK_D * 2;
    /* the per-head products: all items at once when the lengths agree, else one item at a time */
    const int uni = seq->dev.uniform_T;
    for (int i = 0; i < (uni ? 1 : n); i++) {
        const size_t hn = heads_need(uni ? uni : seq->lengths[i], uni ? n : 1);
        if (hn > need) need = hn;
    }
    if (m->stacks && need > m->split_cap) {
        if (m->split_ws) cudaFree(m->split_ws);
        m->split_ws = NULL;
        m->split_cap = 0;
        if (cudaMalloc(&m->split_ws, need) != cudaSuccess) {
            cudaGetLastError();
            m->split_ws = NULL;
            free(off);
            return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_encoder_forward: %zu bytes of split workspace", need);
        }
        m->split_cap = need;
    }
    /* with every projection on the tcgen05 GEMM, bias+Swish and the QKV split
     * run in its epilogues */
    int all_tc = m->stacks != NULL && gemm_in->gated != NULL;
    for (int b = 0; b < m->n_blocks && all_tc; b++)
        all_tc = m->stack[b][W_FF1_1] && m->stack[b][W_FF1_2] && m->stack[b][W_FF2_1] &&
                 m->stack[b][W_FF2_2] && m->stack[b][W_QKV] && m->stack[b][W_PW1] && m->stack[b][W_PW2];
    if (all_tc) {   /* the FF hidden layer's parts */
        const size_t hneed = (size_t)rows_ff * 3 * PK_FF * 2;
        if (hneed > m->hsplit_cap) {
            if (m->hsplit_ws) cudaFree(m->hsplit_ws);
            m->hsplit_ws = NULL;
            m->hsplit_cap = 0;
            if (cudaMalloc(&m->hsplit_ws, hneed) != cudaSuccess) {
                cudaGetLastError();
                m->hsplit_ws = NULL;
                free(off);
                return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_encoder_forward: %zu bytes of hidden-layer parts", hneed);
            }
            m->hsplit_cap = hneed;
        }
    }
    Fwd f = {m, gemm_out, gemm_in, seq, off,
             all_tc ? (PKCU_FUSED_FF_SWISH | PKCU_FUSED_QKV | PKCU_FUSED_CONV) : 0u, x,
             all_tc ? m->hsplit_ws : NULL};
    const int st = pkcu_encoder_nongemm_fused(x, m->params, m->n_blocks, gemm_out, gemm_in, seq, fwd_hook,
                                              &f, f.fused, stream);
    free(off);
    return st;
}

/* ── mel spectrograms to tokens: pre-encode, the encoder stack, greedy decode ──
 * pre_encode_and_scale + encode_blocks + pk_greedy_decode (csrc/encoder.c:
 * 578-593, 495-512; csrc/decoder.c:80-132) for a batch of utterances, every
 * GEMM done by the library: the pre-encode's 1x1 convolutions and projection
 * and joint.enc on the fp32-accurate tensor-core GEMM (cuBLAS SGEMM when a
 * shape does not suit it), the decoder's per-iteration products (B rows) on
 * cuBLAS SGEMM. */

typedef struct {
    pkcu_asr *m;
    pkcu_pre_gemm_outputs go;
    pkcu_pre_gemm_inputs gi;
    long long P2, P3, F;
} PreCtx;

typedef struct {
    pkcu_asr *m;
    pkcu_dec_gemm_outputs go;
    pkcu_dec_gemm_inputs gi;
    const float *x;
    long long F;
    int B;
} DecCtx;

struct pkcu_asr {
    pkcu_encoder_model *enc;
    cublasHandle_t blas;
    float *owned;                      /* fp32 copies of int8 / int4 weights */
    const float *w3, *w6, *w_out;      /* pre-encode 1x1 convs [256, 256], projection [4096, 1024] */
    pkcu_pre_params pre;
    const float *wi[2], *wr[2];        /* LSTM W_i, W_r [2560, 640] */
    const float *j_enc, *j_pred, *j_out;   /* [1024, 640], [640, 640], [640, 1025] */
    pkcu_dec_params dec;
    int decode_mode;                   /* PKCU_ASR_DECODE_* */
    void *tc_planes;                   /* the decoder's products as tcgen05 GEMM operands */
    const void *tc_w[5];               /* joint.enc, [W_i | W_r] of both layers, joint.pred, joint.out:
                                          K-major three-part planes */
    void *dec_ws;                      /* the products' activation parts */
    size_t dec_ws_cap;
    /* the last call's working buffers, kept while the same lengths come again */
    int t_n, *t_frames;                /* mel frames the transcribe buffers were made for */
    pkcu_pre_plan *t_plan;
    float *t_pre;
    pkcu_encoder_ws *t_ws;             /* the blocks' batch: utterances, or their chunks */
    int *t_chunked;                    /* per utterance: chunked (the decisions t_ws was made for) */
    pkcu_chunk_plan *t_chunk;          /* NULL when no utterance is chunked */
    float *t_x;                        /* utterance-layout x of a chunked batch (in t_pre) */
    int chunk_mode;                    /* PKCU_CHUNK_* */
    PreCtx t_pc;
    int d_n, *d_frames;                /* encoder frames the decoder was made for */
    pkcu_decoder *d_dec;
    int d_weights;                     /* pkcu_decoder_set_weights done on d_dec */
    DecCtx d_dc;                       /* the decode hook's context (a stable address) */
};

static void asr_release_transcribe(pkcu_asr *m)
{
    pkcu_encoder_ws_destroy(m->t_ws);
    pkcu_pre_plan_destroy(m->t_plan);
    pkcu_chunk_plan_destroy(m->t_chunk);
    if (m->t_pre) cudaFree(m->t_pre);
    free(m->t_frames);
    free(m->t_chunked);
    m->t_chunk = NULL;
    m->t_chunked = NULL;
    m->t_x = NULL;
    m->t_ws = NULL;
    m->t_plan = NULL;
    m->t_pre = NULL;
    m->t_frames = NULL;
    m->t_n = 0;
}

static void asr_release_decoder(pkcu_asr *m)
{
    pkcu_decoder_destroy(m->d_dec);
    free(m->d_frames);
    m->d_dec = NULL;
    m->d_frames = NULL;
    m->d_n = 0;
    m->d_weights = 0;
}

/* 1 when frames[0..n) equals the kept key (kn, kf). */
static int same_lengths(int kn, const int *kf, int n, const int *frames)
{
    if (!kf || kn != n) return 0;
    for (int i = 0; i < n; i++)
        if (kf[i] != frames[i]) return 0;
    return 1;
}

static int *copy_lengths(const int *frames, int n)
{
    int *c = (int *)malloc(sizeof(int) * (size_t)n);
    if (c) memcpy(c, frames, sizeof(int) * (size_t)n);
    return c;
}

int pkcu_asr_set_decode_mode(pkcu_asr *m, int mode)
{
    if (!m) return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_set_decode_mode: NULL model");
    if (mode != PKCU_ASR_DECODE_FUSED && mode != PKCU_ASR_DECODE_GRAPH && mode != PKCU_ASR_DECODE_EAGER &&
        mode != PKCU_ASR_DECODE_TC)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_set_decode_mode: unknown mode %d", mode);
    m->decode_mode = mode;
    return PKCU_OK;
}

void pkcu_asr_destroy(pkcu_asr *m)
{
    if (!m) return;
    asr_release_transcribe(m);
    asr_release_decoder(m);
    pkcu_encoder_model_destroy(m->enc);
    if (m->blas) cublasDestroy(m->blas);
    if (m->owned) cudaFree(m->owned);
    if (m->tc_planes) cudaFree(m->tc_planes);
    if (m->dec_ws) cudaFree(m->dec_ws);
    free(m);
}

int pkcu_asr_encoder_frames(int mel_frames)
{
    int h = mel_frames;
    for (int s = 0; s < 3; s++) h = (h + 1) / 2;
    return h;
}

/* Device fp32 view of a checkpoint tensor of numel elements: the stored copy
 * for float32, else dequantised into *dst (advanced past it). */
static int fp32_tensor(const pkcu_weights *w, const char *name, long long numel, float **dst,
                       const float **out, pkcu_stream_t stream)
{
    pkcu_tensor t;
    int st = pkcu_weights_find(w, name, &t);
    if (st) return st;
    if (t.numel != numel)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_create: '%s' has %lld elements, expected %lld", name,
                         t.numel, numel);
    if (t.dtype == PKCU_DTYPE_F32) {
        *out = (const float *)t.dev;
        return PKCU_OK;
    }
    st = pkcu_weights_dequant(w, name, *dst, stream);
    if (st) return st;
    *out = *dst;
    *dst += (numel + 63) & ~63LL;
    return PKCU_OK;
}

int pkcu_asr_create(const pkcu_weights *w, pkcu_stream_t stream, pkcu_asr **out)
{
    if (!out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_create: NULL out");
    *out = NULL;
    pkcu_asr *m = (pkcu_asr *)calloc(1, sizeof(*m));
    if (!m) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_asr_create: host allocation");
    int st = pkcu_encoder_model_create(w, stream, &m->enc);
    if (!st && cublasCreate(&m->blas) != CUBLAS_STATUS_SUCCESS) {
        m->blas = NULL;
        st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_asr_create: cublasCreate failed");
    }
    /* room for every weight below should the checkpoint quantise it */
    const long long room = 2 * 65536 + 4096LL * PK_D + 4 * 2560LL * 640 + PK_D * 640LL +
                           640LL * 640 + 640LL * 1025 + 16 * 64;
    if (!st && cudaMalloc((void **)&m->owned, sizeof(float) * (size_t)room) != cudaSuccess) {
        cudaGetLastError();
        m->owned = NULL;
        st = pkcu_fail(PKCU_ERR_NOMEM, "pkcu_asr_create: weight copies");
    }
    float *dst = m->owned;
    if (!st) st = fp32_tensor(w, "pre_encode.conv.3.weight", 65536, &dst, &m->w3, stream);
    if (!st) st = fp32_tensor(w, "pre_encode.conv.6.weight", 65536, &dst, &m->w6, stream);
    if (!st) st = fp32_tensor(w, "pre_encode.out.weight", 4096LL * PK_D, &dst, &m->w_out, stream);
    if (!st) st = pkcu_weights_pre_params(w, &m->pre);
    char name[64];
    for (int l = 0; l < 2 && !st; l++) {
        snprintf(name, sizeof(name), "decoder.lstm.%d.W_i", l);
        st = fp32_tensor(w, name, 2560LL * 640, &dst, &m->wi[l], stream);
        snprintf(name, sizeof(name), "decoder.lstm.%d.W_r", l);
        if (!st) st = fp32_tensor(w, name, 2560LL * 640, &dst, &m->wr[l], stream);
    }
    if (!st) st = fp32_tensor(w, "joint.enc.weight", PK_D * 640LL, &dst, &m->j_enc, stream);
    if (!st) st = fp32_tensor(w, "joint.pred.weight", 640LL * 640, &dst, &m->j_pred, stream);
    if (!st) st = fp32_tensor(w, "joint.out.weight", 640LL * 1025, &dst, &m->j_out, stream);
    static const char *const dn[6] = {"decoder.prediction.embed.weight", "decoder.lstm.0.B",
                                      "decoder.lstm.1.B", "joint.enc.bias", "joint.pred.bias",
                                      "joint.joint_net.2.bias"};
    static const long long dnum[6] = {1025LL * 640, 5120, 5120, 640, 640, 1025};
    const float *dp[6] = {0};
    for (int i = 0; i < 6 && !st; i++) st = fp32_tensor(w, dn[i], dnum[i], &dst, &dp[i], stream);
    if (!st) {
        m->dec.embed = dp[0]; m->dec.lstm0_b = dp[1]; m->dec.lstm1_b = dp[2];
        m->dec.joint_enc_b = dp[3]; m->dec.joint_pred_b = dp[4]; m->dec.joint_out_b = dp[5];
    }
    /* the decoder's products as tcgen05 GEMM operands (three bf16 parts,
     * K-major): joint.enc [1024, 640], the LSTM W_i / W_r [2560, 640] (already
     * [N, K]), joint.pred [640, 640], joint.out [640, 1025]; without the memory
     * the cuBLAS / CUDA-core paths remain */
    if (!st) {
        /* 0 joint.enc [K 1024, N 640]; 1, 2 the layers' [W_i | W_r] as rows [2560, 1280]
         * (one product of [x | h] per layer); 3 joint.pred [640, 640]; 4 joint.out [640, 1025] */
        static const long long tk[5] = {PK_D, 1280, 1280, 640, 640};
        static const long long tn[5] = {640, 2560, 2560, 640, 1025};
        long long off[6] = {0};
        for (int i = 0; i < 5; i++) off[i + 1] = off[i] + ((3 * tk[i] * tn[i] + 127) & ~127LL);
        if (cudaMalloc(&m->tc_planes, sizeof(uint16_t) * (size_t)off[5]) != cudaSuccess) {
            cudaGetLastError();
            m->tc_planes = NULL;
        } else {
            float alpha;
            for (int i = 0; i < 5; i++) m->tc_w[i] = (uint16_t *)m->tc_planes + off[i];
            st = pk_tc_prepare(m->j_enc, 32, 0.0f, PK_D, 640, (void *)m->tc_w[0], &alpha, stream);
            for (int l = 0; l < 2 && !st; l++)
                st = pk_split_rows_cat(m->wi[l], m->wr[l], (void *)m->tc_w[1 + l], 2560, 640, 640, stream);
            if (!st) st = pk_tc_prepare(m->j_pred, 32, 0.0f, 640, 640, (void *)m->tc_w[3], &alpha, stream);
            if (!st) st = pk_tc_prepare(m->j_out, 32, 0.0f, 640, 1025, (void *)m->tc_w[4], &alpha, stream);
            if (!st) pk_tc_warm();
        }
    }
    if (!st && cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess)
        st = pkcu_launch_status("pkcu_asr_create");
    if (st) {
        pkcu_asr_destroy(m);
        return st;
    }
    *out = m;
    return PKCU_OK;
}


static int pre_hook(void *user, int block, int gemm, pkcu_stream_t stream)
{
    (void)block;
    PreCtx *c = (PreCtx *)user;
    cublasHandle_t h = c->m->blas;
    if (cublasSetStream(h, (cudaStream_t)stream) != CUBLAS_STATUS_SUCCESS)
        return pkcu_fail(PKCU_ERR_CUDA, "cublasSetStream failed");
    switch (gemm) {
    case PKCU_GEMM_PRE_PW1: return proj(h, 256, (int)c->P2, 256, c->m->w3, c->gi.s2d, c->go.pw1, stream);
    case PKCU_GEMM_PRE_PW2: return proj(h, 256, (int)c->P3, 256, c->m->w6, c->gi.s3d, c->go.pw2, stream);
    case PKCU_GEMM_PRE_OUT: return proj(h, (int)c->F, PK_D, 4096, c->gi.flat, c->m->w_out, c->go.proj, stream);
    }
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_transcribe: unknown pre-encode GEMM %d", gemm);
}


static int dec_hook(void *user, int block, int gemm, pkcu_stream_t stream)
{
    (void)block;
    DecCtx *c = (DecCtx *)user;
    cublasHandle_t h = c->m->blas;
    if (cublasSetStream(h, (cudaStream_t)stream) != CUBLAS_STATUS_SUCCESS)
        return pkcu_fail(PKCU_ERR_CUDA, "cublasSetStream failed");
    const int B = c->B, Hd = 640;
    switch (gemm) {
    case PKCU_GEMM_DEC_ENC:   return proj(h, (int)c->F, Hd, PK_D, c->x, c->m->j_enc, c->go.enc, stream);
    case PKCU_GEMM_DEC_L0_WI: return rm_gemm(h, B, 4 * Hd, Hd, c->gi.x0, Hd, 0, c->m->wi[0], Hd, 0, 1, c->go.g0i, 4 * Hd, 0, 1);
    case PKCU_GEMM_DEC_L0_WR: return rm_gemm(h, B, 4 * Hd, Hd, c->gi.h0, Hd, 0, c->m->wr[0], Hd, 0, 1, c->go.g0r, 4 * Hd, 0, 1);
    case PKCU_GEMM_DEC_L1_WI: return rm_gemm(h, B, 4 * Hd, Hd, c->gi.h0, Hd, 0, c->m->wi[1], Hd, 0, 1, c->go.g1i, 4 * Hd, 0, 1);
    case PKCU_GEMM_DEC_L1_WR: return rm_gemm(h, B, 4 * Hd, Hd, c->gi.h1, Hd, 0, c->m->wr[1], Hd, 0, 1, c->go.g1r, 4 * Hd, 0, 1);
    case PKCU_GEMM_DEC_PRED:  return rm_gemm(h, B, Hd, Hd, c->gi.h1, Hd, 0, c->m->j_pred, Hd, 0, 0, c->go.pred, Hd, 0, 1);
    case PKCU_GEMM_DEC_OUT:   return rm_gemm(h, B, 1025, Hd, c->gi.hidden, Hd, 0, c->m->j_out, 1025, 0, 0, c->go.out, 1025, 0, 1);
    }
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_transcribe: unknown decoder GEMM %d", gemm);
}

/* The decoder's products on the library's tcgen05 GEMM: the activation rows'
 * three bf16 parts into the decode workspace, then the product with the
 * weight's planes (prepared at pkcu_asr_create). Capture-safe: no allocation,
 * no synchronisation (the workspace is sized before the decode starts). */
static int dec_tc(DecCtx *c, int which, int M, int N, int K, const float *A, const float *A2, float *C,
                  pkcu_stream_t stream)
{
    pkcu_asr *m = c->m;
    if ((size_t)M * 3 * K * 2 > m->dec_ws_cap)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr: decode workspace too small");
    int st = A2 ? pk_split_rows_cat(A, A2, m->dec_ws, M, K / 2, K / 2, stream)
                : pk_split_rows_bf16x3(A, m->dec_ws, M, K, stream);
    if (st) return st;
    pk_tc_epi e;
    memset(&e, 0, sizeof(e));
    e.mode = PK_TC_STORE;
    e.alpha = 1.0f;
    e.C = C;
    return pk_tc_gemm(m->dec_ws, m->tc_w[which], 3, M, N, K, &e, stream);
}

static int dec_hook_tc(void *user, int block, int gemm, pkcu_stream_t stream)
{
    (void)block;
    DecCtx *c = (DecCtx *)user;
    const int B = c->B, Hd = 640;
    /* each layer's two gate products as one, [x | h] [W_i | W_r]^T, into g*i; the
     * W_r outputs g*r stay zero (cleared before the decode), so the cell's
     * g_r + g_i is that one product exactly */
    switch (gemm) {
    case PKCU_GEMM_DEC_ENC:   return dec_tc(c, 0, (int)c->F, Hd, PK_D, c->x, NULL, c->go.enc, stream);
    case PKCU_GEMM_DEC_L0_WI: return dec_tc(c, 1, B, 4 * Hd, 2 * Hd, c->gi.x0, c->gi.h0, c->go.g0i, stream);
    case PKCU_GEMM_DEC_L0_WR: return PKCU_OK;
    case PKCU_GEMM_DEC_L1_WI: return dec_tc(c, 2, B, 4 * Hd, 2 * Hd, c->gi.h0, c->gi.h1, c->go.g1i, stream);
    case PKCU_GEMM_DEC_L1_WR: return PKCU_OK;
    case PKCU_GEMM_DEC_PRED:  return dec_tc(c, 3, B, Hd, Hd, c->gi.h1, NULL, c->go.pred, stream);
    case PKCU_GEMM_DEC_OUT:   return dec_tc(c, 4, B, 1025, Hd, c->gi.hidden, NULL, c->go.out, stream);
    }
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr: unknown decoder GEMM %d", gemm);
}

/* Greedy decode of encoder outputs x [sum enc_frames, 1024] with the model's
 * decoder, in the model's decode mode; host results. The decoder (with its
 * captured graph) is kept for the next call with the same lengths. */
static int asr_decode(pkcu_asr *m, const float *x, const int *enc_frames, int n_utts, int *tokens,
                      int *n_tokens, pkcu_stream_t stream)
{
    int st = PKCU_OK;
    if (!same_lengths(m->d_n, m->d_frames, n_utts, enc_frames)) {
        asr_release_decoder(m);
        st = pkcu_decoder_create(enc_frames, n_utts, &m->d_dec);
        if (!st && !(m->d_frames = copy_lengths(enc_frames, n_utts)))
            st = pkcu_fail(PKCU_ERR_NOMEM, "pkcu_asr_decode: host allocation");
        if (!st) st = pkcu_decoder_buffers(m->d_dec, &m->d_dc.go, &m->d_dc.gi);
        if (st) {
            asr_release_decoder(m);
            return st;
        }
        m->d_n = n_utts;
    }
    long long F = 0;
    for (int i = 0; i < n_utts; i++) F += enc_frames[i];
    DecCtx *dc = &m->d_dc;
    dc->m = m;
    dc->x = x;
    dc->F = F;
    dc->B = n_utts;
    pkcu_decoder *dec = m->d_dec;
    /* the tcgen05 products' activation parts: the encoder projection's F rows
     * of 1024, the per-iteration products' B rows of 640 */
    const size_t need = (size_t)(F * 3 * PK_D * 2 > (long long)n_utts * 3 * 1280 * 2 ? F * 3 * PK_D * 2
                                                                                    : (long long)n_utts * 3 * 1280 * 2);
    if (m->tc_planes && need > m->dec_ws_cap) {
        if (m->dec_ws) cudaFree(m->dec_ws);
        m->dec_ws_cap = 0;
        if (cudaMalloc(&m->dec_ws, need) != cudaSuccess) {
            cudaGetLastError();
            m->dec_ws = NULL;
            return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_asr: %zu bytes of decode workspace", need);
        }
        m->dec_ws_cap = need;
    }
    pkcu_gemm_hook enc_hook = m->tc_planes ? dec_hook_tc : dec_hook;
    if (m->decode_mode == PKCU_ASR_DECODE_FUSED) {
        if (!m->d_weights) {
            const pkcu_dec_weights dw = {m->wi[0], m->wr[0], m->wi[1], m->wr[1], m->j_pred, m->j_out};
            st = pkcu_decoder_set_weights(dec, &dw, stream);
            m->d_weights = !st;
        }
        if (!st) st = enc_hook(dc, -1, PKCU_GEMM_DEC_ENC, stream);
        if (!st) st = pkcu_greedy_decode_fused(dec, &m->dec, stream);
    } else if (m->decode_mode == PKCU_ASR_DECODE_TC) {
        if (!m->tc_planes) return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr: the tensor-core decode needs its operands");
        const size_t gb = sizeof(float) * (size_t)n_utts * 2560;
        if (cudaMemsetAsync(dc->go.g0r, 0, gb, (cudaStream_t)stream) != cudaSuccess ||
            cudaMemsetAsync(dc->go.g1r, 0, gb, (cudaStream_t)stream) != cudaSuccess)
            return pkcu_fail(PKCU_ERR_CUDA, "pkcu_asr: clearing the W_r products");
        st = pkcu_greedy_decode_graph(dec, &m->dec, dec_hook_tc, dc, stream);
    } else {
        st = m->decode_mode == PKCU_ASR_DECODE_EAGER
                 ? pkcu_greedy_decode(dec, &m->dec, dec_hook, dc, stream)
                 : pkcu_greedy_decode_graph(dec, &m->dec, dec_hook, dc, stream);
    }
    if (!st) st = pkcu_decoder_results(dec, n_tokens, NULL, tokens, stream);
    if (!st) st = pk_check_wait_timeouts("pkcu_asr");
    return st;
}

int pkcu_asr_decode(pkcu_asr *m, const float *enc, const int *enc_frames, int n_utts, int *tokens,
                    int *n_tokens, pkcu_stream_t stream)
{
    if (!m || !enc || !enc_frames || n_utts <= 0 || !tokens || !n_tokens)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_decode: bad argument");
    if (!PK_ALIGNED16(enc)) return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_decode: enc must be 16-byte aligned");
    return asr_decode(m, enc, enc_frames, n_utts, tokens, n_tokens, stream);
}

/* Chunking decision of each utterance of this call (PK_CHUNK is read per
 * call, as the reference's should_chunk does); *any: one or more chunked. */
static int *chunk_decisions(const pkcu_asr *m, const int *mel_frames, int n_utts, int *any)
{
    int *d = (int *)malloc(sizeof(int) * (size_t)n_utts);
    *any = 0;
    if (!d) return NULL;
    for (int i = 0; i < n_utts; i++) {
        d[i] = pkcu_should_chunk(pkcu_asr_encoder_frames(mel_frames[i]), m->chunk_mode);
        *any |= d[i];
    }
    return d;
}

/* pre_encode_and_scale + the 24 blocks, chunked as pk_encoder chunks
 * (csrc/encoder.c:612-633): on success *x_out is the encoder output
 * [sum encoder frames, 1024], utterance after utterance, in a kept buffer. */
static int asr_encode(pkcu_asr *m, const float *mel, const int *mel_frames, int n_utts,
                      float **x_out, pkcu_stream_t stream)
{
    int st = PKCU_OK, any = 0;
    PreCtx *pc = &m->t_pc;
    int *dec = chunk_decisions(m, mel_frames, n_utts, &any);
    if (!dec) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_asr: host allocation");
    if (!same_lengths(m->t_n, m->t_frames, n_utts, mel_frames) ||
        !same_lengths(m->t_n, m->t_chunked, n_utts, dec)) {
        asr_release_transcribe(m);
        st = pkcu_pre_plan_create(mel_frames, n_utts, &m->t_plan);
        if (!st && !(m->t_frames = copy_lengths(mel_frames, n_utts)))
            st = pkcu_fail(PKCU_ERR_NOMEM, "pkcu_asr: host allocation");
        if (!st) {
            m->t_chunked = dec;
            dec = NULL;
        }
        if (!st) {
            memset(pc, 0, sizeof(*pc));
            pc->m = m;
            pc->P2 = pkcu_pre_plan_p2(m->t_plan);
            pc->P3 = pkcu_pre_plan_p3(m->t_plan);
            pc->F = pkcu_pre_plan_frames(m->t_plan);
            const long long n2 = 256 * pc->P2, n3 = 256 * pc->P3;
            /* + the utterance-layout x of a chunked batch */
            const long long total = 2 * n2 + 2 * n3 + pc->F * 4096 + pc->F * PK_D + (any ? pc->F * PK_D : 0);
            if (cudaMalloc((void **)&m->t_pre, sizeof(float) * (size_t)total) != cudaSuccess) {
                cudaGetLastError();
                m->t_pre = NULL;
                st = pkcu_fail(PKCU_ERR_NOMEM, "pkcu_asr: pre-encode buffers");
            } else {
                float *pre = m->t_pre;
                pc->gi.s2d = pre;
                pc->go.pw1 = pre + n2;
                pc->gi.s3d = pre + 2 * n2;
                pc->go.pw2 = pre + 2 * n2 + n3;
                pc->gi.flat = pre + 2 * n2 + 2 * n3;
                pc->go.proj = pc->gi.flat + pc->F * 4096;
                m->t_x = any ? pc->go.proj + pc->F * PK_D : NULL;
            }
        }
        if (!st && any) {
            int *ef = (int *)malloc(sizeof(int) * (size_t)n_utts);
            if (!ef) st = pkcu_fail(PKCU_ERR_NOMEM, "pkcu_asr: host allocation");
            for (int i = 0; i < n_utts && !st; i++) ef[i] = pkcu_asr_encoder_frames(mel_frames[i]);
            if (!st) st = pkcu_chunk_plan_create(ef, n_utts, m->chunk_mode, &m->t_chunk);
            free(ef);
        }
        if (!st)
            st = pkcu_encoder_ws_create(m->t_chunk ? pkcu_chunk_plan_seq(m->t_chunk)
                                                   : pkcu_pre_plan_out_seq(m->t_plan), 1, &m->t_ws);
        if (st) {
            free(dec);
            asr_release_transcribe(m);
            return st;
        }
        m->t_n = n_utts;
    }
    free(dec);
    const pkcu_seq *seq = m->t_chunk ? pkcu_chunk_plan_seq(m->t_chunk) : pkcu_pre_plan_out_seq(m->t_plan);
    float *xb = NULL;
    pkcu_gemm_outputs go;
    pkcu_gemm_inputs gi;
    st = pkcu_encoder_ws_device(m->t_ws, &xb, &go, &gi);
    float *xu = m->t_chunk ? m->t_x : xb;   /* utterance layout */
    if (!st) st = pkcu_pre_encode(mel, &m->pre, &pc->go, &pc->gi, xu, m->t_plan, pre_hook, pc, stream);
    if (!st && m->t_chunk) st = pkcu_chunk_split(m->t_chunk, xu, xb, stream);
    if (!st) st = pkcu_encoder_forward(m->enc, xb, &go, &gi, seq, stream);
    if (!st && m->t_chunk) st = pkcu_chunk_stitch(m->t_chunk, xb, xu, stream);
    if (!st) *x_out = xu;
    return st;
}

int pkcu_asr_set_chunk_mode(pkcu_asr *m, int mode)
{
    if (!m) return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_set_chunk_mode: NULL model");
    if (mode != PKCU_CHUNK_AUTO && mode != PKCU_CHUNK_OFF && mode != PKCU_CHUNK_ON)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_set_chunk_mode: unknown mode %d", mode);
    m->chunk_mode = mode;
    return PKCU_OK;
}

int pkcu_asr_encode(pkcu_asr *m, const float *mel, const int *mel_frames, int n_utts, float *enc,
                    pkcu_stream_t stream)
{
    if (!m || !mel || !mel_frames || n_utts <= 0 || !enc)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_encode: bad argument");
    float *x = NULL;
    int st = asr_encode(m, mel, mel_frames, n_utts, &x, stream);
    if (st) return st;
    long long F = 0;
    for (int i = 0; i < n_utts; i++) F += pkcu_asr_encoder_frames(mel_frames[i]);
    if (cudaMemcpyAsync(enc, x, sizeof(float) * (size_t)(F * PK_D), cudaMemcpyDeviceToDevice,
                        (cudaStream_t)stream) != cudaSuccess ||
        cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess)
        return pkcu_fail(PKCU_ERR_CUDA, "pkcu_asr_encode: %s", cudaGetErrorString(cudaGetLastError()));
    return pk_check_wait_timeouts("pkcu_asr_encode");
}

int pkcu_asr_transcribe(pkcu_asr *m, const float *mel, const int *mel_frames, int n_utts,
                        int *tokens, int *n_tokens, pkcu_stream_t stream)
{
    if (!m || !mel || !mel_frames || n_utts <= 0 || !tokens || !n_tokens)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_asr_transcribe: bad argument");
    float *x = NULL;
    int st = asr_encode(m, mel, mel_frames, n_utts, &x, stream);
    int *enc_frames = NULL;
    if (!st) {
        enc_frames = (int *)malloc(sizeof(int) * (size_t)n_utts);
        if (!enc_frames) st = pkcu_fail(PKCU_ERR_NOMEM, "pkcu_asr_transcribe: host allocation");
        for (int i = 0; i < n_utts && !st; i++) enc_frames[i] = pkcu_asr_encoder_frames(mel_frames[i]);
    }
    if (!st) st = asr_decode(m, x, enc_frames, n_utts, tokens, n_tokens, stream);
    free(enc_frames);
    return st;
}
