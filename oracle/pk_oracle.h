/*  pk_oracle.h -- CPU restatement of the reference's non-GEMM encoder ops.
 *
 *  TEST INFRASTRUCTURE ONLY: the checker for the B200 kernels. Only tests/,
 *  __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it.
 *
 *  Every function restates one piece of the reference
 *  (eschmidbauer/parakeet-unified-en-0.6b-c, files under csrc/) in plain
 *  scalar C evaluated in IEEE single precision (no -ffast-math): the same
 *  operations in the same order, with an explicit fmaf() wherever the
 *  reference's AVX2 path fuses a multiply-add. It is pinned against the
 *  reference's own compiled code (oracle/_ref) and the committed golden
 *  vectors (tests/golden/) by the CPU test suite.
 */
#ifndef PK_ORACLE_H
#define PK_ORACLE_H
#include <stdint.h>

#define OR_D   1024
#define OR_H   8
#define OR_DH  128
#define OR_FF  4096

/* ── csrc/tensor_ops.c ─────────────────────────────────────────────────── */
float or_exp_poly(float x);
void or_layer_norm(const float *x, const float *g, const float *b, float *out, int len);
void or_layer_norm_rows(const float *x, const float *g, const float *b, float *out,
                        int n_rows, int D);
void or_layer_norm_rows_inplace(float *x, const float *g, const float *b, int n_rows, int D);
void or_softmax(float *x, int len);
void or_softmax_rows(float *x, int n_rows, int len);
void or_swish(float *x, long long n);
void or_relu(float *x, long long n);
void or_bias_add(float *x, const float *b, int len);
void or_depthwise_conv1d(const float *x, const float *w, const float *b, float *out,
                         int C, int T, int K);

/* ── csrc/encoder.c inline ops ─────────────────────────────────────────── */
void or_relative_shift(const float *bd, float *out, int H, int T);
void or_relpos_combine(float *ac, const float *bd_shifted, long long n, float scale);
void or_qkv_split_uv(const float *qkv, const float *u, const float *v,
                     float *Qu, float *Qv, float *K, float *V, int T);
void or_pos_head_split(const float *P, float *P_h, int L);
void or_head_concat(const float *attn_h, float *attn, int T);
void or_residual(float *x, const float *y, float alpha, long long n);
void or_transpose(const float *src, float *dst, int rows, int cols);
void or_pointwise_bias(float *out, const float *b, int C, int T);
void or_glu_channel_first(const float *pw1, float *gated, int D, int T);
void or_glu_time_first(const float *in, float *out, int T, int D);
void or_transpose_add(float *x, const float *pw2, int T, int D);
void or_batch_norm(float *y, const float *mean, const float *var, const float *gamma,
                   const float *beta, float eps, int C, int T);

/* One conformer block (csrc/encoder.c:482-491) with its GEMM outputs taken
 * from 12 stand-ins; the 14 GEMM inputs it produces are written to outs[]
 * (NULL array or NULL entries skip). params/standins/outs use the role order
 * of ref_harness.c. */
void or_conformer_block(float *x, int T, const float *const *params,
                        const float *const *standins, float *const *outs);

/* ── csrc/decoder.c ────────────────────────────────────────────────────── */
void or_joint_add_act(const float *enc, const float *pred, float *out,
                      int B, int T, int J, int act);
void or_argmax_rows(const float *logits, int32_t *out, long long n_rows, int V);

/* ── csrc/blas.c, csrc/weights.c (built without -ffast-math) ───────────── */
void or_dequant_i8(const int8_t *q, float scale, float *out, long long n);
float or_requant_qkv_i8(const int8_t *q, const int8_t *k, const int8_t *v,
                        float sq, float sk, float sv, int8_t *fused, int K, int D);
void or_dequant_i4(const uint8_t *packed, const float *scales, float *out,
                   int K, int N, int group, int axis);
void or_dequant_i4_qkv(const uint8_t *pq, const uint8_t *pk, const uint8_t *pv,
                       const float *sq, const float *sk, const float *sv,
                       float *fused, int K, int D, int group);


/* Pre-encode subsampling + input scaling (pk_oracle_preencode.c). */
int or_pre_out_frames(int T);
int or_pre_encode(const float *mel, int T, const float *const *params, const float *y2,
                  const float *y3, const float *proj, float *s2d_cap, float *s3d_cap,
                  float *flat_cap, float *x_out);

/* Greedy RNN-T decode of one utterance (pk_oracle_decode.c), GEMM products as
 * caller stand-ins. */
enum { OR_DEC_ENC = 0, OR_DEC_PRED, OR_DEC_OUT, OR_DEC_L0_WI, OR_DEC_L0_WR, OR_DEC_L1_WI,
       OR_DEC_L1_WR };
typedef void (*or_dec_gemm_fn)(void *user, int gemm, int iter, const float *in, int n_in,
                               float *out, int n_out);
int or_greedy_decode(int T, const float *embed, const float *B0, const float *B1,
                     const float *enc_b, const float *pred_b, const float *out_b,
                     or_dec_gemm_fn gemm, void *user, int *tokens, int max_tokens,
                     float *state, int *n_iters);

#endif
