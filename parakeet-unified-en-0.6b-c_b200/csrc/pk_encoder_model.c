/* pk_encoder_model.c -- the whole encoder stack on the GPU: the fused non-GEMM
 * block sequence (pkcu_encoder_nongemm) with its twelve GEMM points served by
 * the library itself, on the weights of an uploaded checkpoint.
 *
 * Every GEMM weight of every block is made an fp32 device copy once
 * (pkcu_weights_dequant: int8 (float)q * scale, int4 (float)nibble * group
 * scale, fp32 copied; the fused QKV as the reference's loader builds it), so a
 * forward pass is fp32 throughout like the reference's (csrc/encoder.c). The
 * row-major projections of the block (FF, QKV, output) run on the tensor cores
 * with fp32 accuracy (k_gemm.cu: three bf16 parts per operand, nine MMAs per
 * product); the other products are cuBLAS single-precision GEMMs (no TF32):
 * per utterance the
 * positional projection of its slice of the sinusoidal table
 * (csrc/encoder.c:220-227), the per-head score, positional-score and context
 * products and the two pointwise convolutions, as strided batches over heads
 * (and over utterances when the batch is uniform). */
#include <stdlib.h>
#include <string.h>

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

struct pkcu_encoder_model {
    int device, n_blocks;
    cublasHandle_t blas;
    float *arena;                      /* fp32 GEMM weights, block after block */
    const float *w[64][W_N];
    pkcu_block_params params[64];
    const float *pe;                   /* pos_encoding.pe_table [9999, 1024] */
};

void pkcu_encoder_model_destroy(pkcu_encoder_model *m)
{
    if (!m) return;
    if (m->blas) cublasDestroy(m->blas);
    if (m->arena) cudaFree(m->arena);
    free(m);
}

static long long block_elems(void)
{
    long long n = 0;
    for (int k = 0; k < W_N; k++) n += W_ELEMS[k];
    return n;
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
} Fwd;

static const float ONE = 1.0f, ZERO = 0.0f;

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
    switch (gemm) {   /* the row-major projections of the whole batch */
    case PKCU_GEMM_FF1_1: return proj(h, (int)F, PK_FF, PK_D, gi->ln_ff1, W[W_FF1_1], go->ff1_h, stream);
    case PKCU_GEMM_FF1_2: return proj(h, (int)F, PK_D, PK_FF, gi->h1, W[W_FF1_2], go->ff1_out, stream);
    case PKCU_GEMM_QKV:   return proj(h, (int)F, 3 * PK_D, PK_D, gi->ln_sa, W[W_QKV], go->qkv, stream);
    case PKCU_GEMM_OUT:   return proj(h, (int)F, PK_D, PK_D, gi->attn, W[W_OUT], go->att_out, stream);
    case PKCU_GEMM_FF2_1: return proj(h, (int)F, PK_FF, PK_D, gi->ln_ff2, W[W_FF2_1], go->ff2_h, stream);
    case PKCU_GEMM_FF2_2: return proj(h, (int)F, PK_D, PK_FF, gi->h2, W[W_FF2_2], go->ff2_out, stream);
    default: break;
    }
    /* per utterance (all utterances in one batch when the lengths agree) */
    const int groups = uni ? 1 : n, per = uni ? n : 1;
    for (int i = 0; i < groups; i++) {
        const int T = uni ? uni : f->seq->lengths[i], L = 2 * T - 1, Hb = PK_H * per;
        const long long fo = f->off[4 * i], po = f->off[4 * i + 1], so = f->off[4 * i + 2],
                        bo = f->off[4 * i + 3];
        const float *pe = f->m->pe + (long long)(PE_CENTER - T + 1) * PK_D;
        int st = PKCU_OK;
        switch (gemm) {
        case PKCU_GEMM_POS:   /* P = pe slice [2T-1, 1024] x W_pos */
            st = rm_gemm(h, L, PK_D, PK_D, pe, PK_D, 0, W[W_POS], PK_D, 0, 0, go->P + po * PK_D, PK_D,
                         (long long)L * PK_D, per);
            break;
        case PKCU_GEMM_AC:    /* ac[h] = (Q + u)[h] K[h]^T */
            st = rm_gemm(h, T, T, PK_DH, gi->Qu + fo * PK_D, PK_DH, (long long)T * PK_DH,
                         gi->K + fo * PK_D, PK_DH, (long long)T * PK_DH, 1, go->ac + so, T,
                         (long long)T * T, Hb);
            break;
        case PKCU_GEMM_BD:    /* bd[h] = (Q + v)[h] P[h]^T (P heads [8, 2T-1, 128] per utterance) */
            st = rm_gemm(h, T, L, PK_DH, gi->Qv + fo * PK_D, PK_DH, (long long)T * PK_DH,
                         gi->P_h + po * PK_D, PK_DH, (long long)L * PK_DH, 1, go->bd + bo, L,
                         (long long)T * L, Hb);
            break;
        case PKCU_GEMM_AV:    /* attn[h] = S[h] V[h] */
            st = rm_gemm(h, T, PK_DH, T, gi->S + so, T, (long long)T * T, gi->V + fo * PK_D, PK_DH,
                         (long long)T * PK_DH, 0, go->attn_h + fo * PK_D, PK_DH, (long long)T * PK_DH, Hb);
            break;
        case PKCU_GEMM_PW1:   /* [2048, T] = W_pw1 [2048, 1024] x cf [1024, T] */
            st = rm_gemm(h, 2 * PK_D, T, PK_D, W[W_PW1], PK_D, 0, gi->cf + fo * PK_D, T,
                         (long long)PK_D * T, 0, go->pw1 + fo * 2 * PK_D, T, 2LL * PK_D * T, per);
            break;
        case PKCU_GEMM_PW2:   /* [1024, T] = W_pw2 x dw [1024, T] */
            st = rm_gemm(h, PK_D, T, PK_D, W[W_PW2], PK_D, 0, gi->dw + fo * PK_D, T,
                         (long long)PK_D * T, 0, go->pw2 + fo * PK_D, T, (long long)PK_D * T, per);
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
    Fwd f = {m, gemm_out, gemm_in, seq, off};
    const int st = pkcu_encoder_nongemm(x, m->params, m->n_blocks, gemm_out, gemm_in, seq, fwd_hook,
                                        &f, stream);
    free(off);
    return st;
}
