/* pkcuda_internal.h -- definitions shared by the C host code and the CUDA
 * kernels of libpk_tensor_ops_cuda.so. Not installed; the public interface is
 * include/pkcuda.h. */
#ifndef PKCUDA_INTERNAL_H
#define PKCUDA_INTERNAL_H

#include <stddef.h>
#include <stdint.h>
#include "pkcuda.h"

#define PK_D   1024   /* model width (csrc/parakeet.h:15) */
#define PK_H   8      /* attention heads (:16) */
#define PK_DH  128    /* head width (:17) */
#define PK_FF  4096   /* feed-forward width (:18) */
#define PK_DW_MAX_K 129  /* widest depthwise kernel the conv kernels stage */

#ifdef __cplusplus
extern "C" {
#endif

/* Device view of a batch of items (utterances or chunks) of T_b frames each,
 * concatenated item after item. uniform_T > 0: all items share that length and
 * the array pointers are NULL. */
typedef struct {
    int n_items;
    int uniform_T;
    int max_T;
    const int *T;
    const long long *frame_off;
    const long long *score_off;
    const long long *bd_off;
    const long long *pos_off;
} pkcu_seq_dev;

struct pkcu_seq {
    pkcu_seq_dev dev;
    int *lengths;            /* host copy [n_items] */
    long long frames, score_elems, bd_elems, pos_rows;
    void *dev_block;         /* one cudaMalloc holding the device arrays (ragged only) */
    int device;
};

/* Records a failure message for pkcu_last_error() and returns status. */
int pkcu_fail(int status, const char *fmt, ...);
/* Maps the last launch error (cudaGetLastError) to a status. */
int pkcu_launch_status(const char *what);
/* Streaming multiprocessor count of the current device (cached). */
int pkcu_sm_count(void);
/* Current device index, or 0. */
int pkcu_device(void);
/* Per-translation-unit counters of device waits that ran out (k_softmax.cu,
 * k_conv.cu); read and optionally reset on the current device. */
int pk_softmax_wait_timeouts(unsigned *count, int reset);
int pk_conv_wait_timeouts(unsigned *count, int reset);
int pk_tc_wait_timeouts(unsigned *count, int reset);   /* k_tcgemm.cu */

/* The library's tcgen05 GEMM (k_tcgemm.cu): C = epilogue(alpha * A W) with A
 * given as its three bf16 parts [M, 3K] (pk_split_rows_bf16x3) and W as
 * npb K-major bf16 planes [N, npb K] (pk_tc_prepare); K % 32 == 0, N % 32 == 0. */
#define PK_TC_STORE 0   /* C = alpha A W (+ bias) (+ beta C)            */
#define PK_TC_SWISH 1   /* C = Swish(alpha A W + bias)                  */
#define PK_TC_RESID 2   /* C += rscale (alpha A W + bias), one FMA      */
#define PK_TC_QKV   3   /* the QKV head split with pos_bias_u / v       */
#define PK_TC_CF    4   /* rows = frames of seq: C per item [N, T] (+ bias[n]) */
#define PK_TC_GLU   5   /* as CF, columns interleaved value / gate by 32: GLU -> [N/2, T] */
#define PK_TC_STORE_T 6 /* C[n * ldc + m] = alpha (A W)[m, n]: the product written transposed */
#define PK_TC_SWISH_SPLIT 7 /* Swish(alpha A W + bias) written only as its three bf16 parts,
                               Cb [M, 3N] = [h0 | h1 | h2]: the next product's operand */
typedef struct {
    int mode;
    float alpha, beta, rscale;
    const float *bias;
    float *C;
    long long ldc;                       /* 0: N */
    const float *u, *v;                  /* QKV: pos_bias_u / v [8, 128] */
    float *Qu, *Qv, *K, *V;              /* QKV: per-item [8, T, 128] outputs */
    const pkcu_seq *seq;                 /* QKV: the batch (M = its frames) */
    void *Cb;                            /* SWISH_SPLIT: bf16 parts [M, 3N], 16-byte aligned */
} pk_tc_epi;
/* W [K, N] (bits 32: fp32, 8: int8 with per-tensor scale) -> planes: one
 * [N, K] plane of q for int8 (alpha = scale), else three [N, 3K] parts. */
int pk_tc_prepare(const void *data, int bits, float scale, int K, int N, void *planes, float *alpha,
                  pkcu_stream_t stream);
int pk_tc_gemm(const void *a_parts, const void *planes, int npb, int M, int N, int K,
               const pk_tc_epi *ep, pkcu_stream_t stream);
/* Z products of one shape in one launch, both operands three-part planes:
 * A [a_rows, 3K] with entry z's M rows from row z * a_z, B [b_rows, 3K] with
 * its N rows from z * b_z (rows past an entry's own belong to the next one and
 * only produce discarded outputs), output from ep->C + z * c_z. */
int pk_tc_gemm_batched(const void *a_parts, long long a_rows, const void *b_parts, long long b_rows,
                       int M, int N, int K, const pk_tc_epi *ep, int Z, long long a_z, long long b_z,
                       long long c_z, pkcu_stream_t stream);
/* Raises the GEMM kernels' shared-memory limit now, so that a first launch
 * inside a stream capture makes no attribute call. */
void pk_tc_warm(void);
/* A pointwise weight W [N, K] (already K-major) -> three-part planes [N, 3K];
 * glu: rows interleaved value / gate in groups of 32 for PK_TC_GLU. */
int pk_tc_prepare_rows(const float *W, int N, int K, int glu, void *planes, pkcu_stream_t stream);
/* Rows A [M, K] -> parts [M, 3 Kp] zero-padded from K; Z matrices X [R, Cc]
 * -> the parts of their transposes, rows z Cc + c of 3 Kp, zero from R. */
int pk_split_rows_pad(const float *A, void *parts, long long M, int K, int Kp, pkcu_stream_t stream);
int pk_split_t_pad(const float *X, void *parts, int Z, int R, int Cc, int Kp, pkcu_stream_t stream);
/* Rows [X1[m] | X2[m]] (K1 + K2 wide) -> parts [M, 3 (K1 + K2)]. */
int pk_split_rows_cat(const float *X1, const float *X2, void *parts, long long M, int K1, int K2,
                      pkcu_stream_t stream);
/* Channel-first items X [C, T_b] -> time-first three-part rows [frames, 3C]. */
int pk_split_cf_t(const float *X, void *parts, int C, const pkcu_seq *seq, pkcu_stream_t stream);

/* For synchronous entry points, after their final synchronisation: reads and
 * resets both counters and returns PKCU_ERR_CUDA (with a message naming what)
 * when any wait ran out since the last reset, anywhere in the process on this
 * device. */
int pk_check_wait_timeouts(const char *what);

#define PK_ALIGNED16(p) ((((uintptr_t)(p)) & 15u) == 0)

/* fp32-accurate tensor-core GEMM (k_gemm.cu): C[M, N] = A[M, K] B[K, N],
 * row-major, packed rows; PKCU_ERR_ARG (without a message) when N or K is not
 * a multiple of 4 or a pointer is not 16-byte aligned. */
int pk_gemm_f32_rm(const float *A, const float *B, float *C, int M, int N, int K,
                   pkcu_stream_t stream);

/* fp32 activations as three bf16 parts (k_split.cu): rows of A [M, K] to
 * out [M, 3K] = [a0 | a1 | a2] (K a multiple of 4, 16-byte aligned). */
int pk_split_rows_bf16x3(const float *A, void *out, long long M, int K, pkcu_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif
