/* pkcuda.h -- C ABI of libpk_tensor_ops_cuda.so: B200 (sm_100a) kernels for the
 * non-GEMM work of the Parakeet FastConformer encoder and RNN-T joint.
 *
 * Reference: eschmidbauer/parakeet-unified-en-0.6b-c, a pure-C CPU engine.
 * Citations below are file:line within that project.
 *
 * Three layers, all plain C:
 *
 *  1. Drop-in host API -- the exact prototypes of csrc/parakeet.h:231-262
 *     (pk_layer_norm ... pk_depthwise_conv1d). Host pointers in and out,
 *     synchronous, no return value, like the functions they replace. Each call
 *     copies its operands to the GPU, runs the kernel and copies the result
 *     back. pk_cuda_status() reports the outcome of the calling thread's last
 *     drop-in call (the reference itself reports no errors).
 *
 *  2. Device API -- pkcu_*: device pointers, asynchronous on the given stream,
 *     int status (PKCU_OK or an error code). Covers the reference's tensor_ops
 *     (csrc/tensor_ops.c), the inline loops of csrc/encoder.c and
 *     csrc/decoder.c, and the dequantisation of csrc/blas.c / csrc/weights.c,
 *     plus producer/consumer fusions of adjacent ops. Unless stated otherwise
 *     every float pointer must be 16-byte aligned (cudaMalloc memory is) and
 *     in/out buffers of one call must not overlap.
 *
 *  3. Sequence driver -- pkcu_encoder_nongemm: the whole per-block non-GEMM op
 *     sequence of csrc/encoder.c:482-491 for a batch of utterances or chunks,
 *     with a hook at every GEMM.
 *
 * Model constants follow csrc/parakeet.h:15-30: D = 1024, 8 heads of 128,
 * FF = 4096, conv kernel 9, joint width 640, 1025 logits.
 */
#ifndef PKCUDA_H
#define PKCUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same underlying type as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st *pkcu_stream_t;

/* ── status ──────────────────────────────────────────────────────────────── */

#define PKCU_OK          0
#define PKCU_ERR_ARG     1   /* NULL pointer, size out of range, misaligned pointer */
#define PKCU_ERR_CUDA    2   /* a CUDA runtime call or kernel launch failed */
#define PKCU_ERR_NOMEM   3   /* device or host allocation failed */

const char *pkcu_status_string(int status);
/* Detail of the calling thread's most recent failure ("" if none). */
const char *pkcu_last_error(void);
/* Library version, e.g. "0.1.0". */
const char *pkcu_version(void);
/* Device self-test (no counterpart in the reference): checks, for every float
 * d in [1, 2^126), that the fast reciprocal the Swish kernels use equals the
 * correctly rounded IEEE reciprocal on the current device. *mismatches
 * receives the number of differing inputs (0 expected). Synchronous, ~1 ms. */
int pkcu_selftest(unsigned long long *mismatches);
/* Device-side wait check (no counterpart in the reference): kernels that stage
 * rows with bulk asynchronous copies wait for them at most 1 s; a wait that
 * runs out makes the kernel abandon that part of its output and is counted.
 * *count receives the number of such waits on the current device since the
 * last reset (0 in correct operation); reset != 0 clears it. Synchronous.
 * The asynchronous pkcu_* calls report such timeouts only through this
 * counter; the synchronous host-buffer calls (the drop-ins,
 * pkcu_encoder_nongemm_host, pkcu_asr_transcribe / pkcu_asr_decode) read and
 * reset it after their final synchronisation and return PKCU_ERR_CUDA when
 * it is not 0. */
int pkcu_wait_timeouts(unsigned *count, int reset);
/* Self-test of that bound: one warp waits 20 ms on a barrier whose copy never
 * comes; *timed_out receives 1 when the wait gave up as designed. */
int pkcu_selftest_wait(int *timed_out);

/* ── batches of items (utterances / chunks) ─────────────────────────────────
 * Ops that know about sequence structure take a pkcu_seq: n_items items of
 * T_b frames each, concatenated. Per-item tensor layouts, item after item:
 *   frames [T_b, D] (time-first rows)         -> offset Σ T       * D
 *   heads  [H, T_b, 128]                       -> offset Σ T       * D
 *   channel-first [C, T_b]                     -> offset Σ T       * C
 *   scores [H, T_b, T_b]                       -> offset Σ H T^2
 *   bd     [H, T_b, 2T_b-1]                    -> offset Σ H T(2T-1)
 *   pos    [2T_b-1, D]                         -> offset Σ (2T-1)  * D
 * The edge chunks of the reference's chunked encoder have fewer frames than
 * the interior ones (csrc/encoder.c:531-543); a ragged batch keeps them
 * unpadded. pkcu_seq_create allocates on the current device (ragged batches
 * only) and synchronises; a pkcu_seq is read-only afterwards and may be shared
 * by concurrent calls. */
typedef struct pkcu_seq pkcu_seq;

int  pkcu_seq_create(const int *lengths, int n_items, pkcu_seq **out);
void pkcu_seq_destroy(pkcu_seq *seq);
int       pkcu_seq_n_items(const pkcu_seq *seq);
long long pkcu_seq_frames(const pkcu_seq *seq);       /* Σ T_b            */
long long pkcu_seq_score_elems(const pkcu_seq *seq);  /* Σ H T_b^2        */
long long pkcu_seq_bd_elems(const pkcu_seq *seq);     /* Σ H T_b(2T_b-1)  */
long long pkcu_seq_pos_rows(const pkcu_seq *seq);     /* Σ (2T_b-1)       */

/* ── 1. drop-in host API (csrc/parakeet.h:231-262) ────────────────────────── */

/* csrc/tensor_ops.c:151 */
void pk_layer_norm(const float *x, const float *gamma, const float *beta_, float *out, int len);
/* csrc/tensor_ops.c:249 */
void pk_layer_norm_rows(const float *x, const float *gamma, const float *beta_, float *out,
                        int n_rows, int D);
/* csrc/tensor_ops.c:275 */
void pk_layer_norm_rows_inplace(float *x, const float *gamma, const float *beta_, int n_rows,
                                int D);
/* csrc/tensor_ops.c:367 */
void pk_swish(float *x, int len);
/* csrc/tensor_ops.c:401 */
void pk_relu(float *x, int len);
/* csrc/tensor_ops.c:284 */
void pk_softmax(float *x, int len);
/* csrc/tensor_ops.c:359 */
void pk_softmax_rows(float *x, int n_rows, int len);
/* csrc/tensor_ops.c:420 */
void pk_bias_add(float *x, const float *b, int len);
/* csrc/tensor_ops.c:570; b may be NULL (:561) */
void pk_depthwise_conv1d(const float *x, const float *w, const float *b, float *out, int C,
                         int T, int K);
/* No counterpart in the reference. pk_softmax_rows for callers that cannot let
 * the library allocate device memory (a real-time callback that must not wait
 * on cudaMalloc, which can synchronise the device; a process that pre-assigns
 * all device memory to its own pool): the rows are staged in a fixed 16 MiB
 * array that every device loading the library holds until exit, so
 * n_rows * len may be at most 4,194,304 (larger sizes return PKCU_ERR_ARG).
 * The first call on a device looks up the array's address -- make it before
 * any stream capture; the looked-up address does not survive cudaDeviceReset.
 * Calls share the array; calls whose GPU work overlaps race on it. An empty
 * call (n_rows or len 0) does nothing and accepts a NULL x. Returns PKCU_OK or
 * an error code. */
int pk_softmax_rows_noalloc(float *x, int n_rows, int len);
/* Status of the calling thread's last drop-in call: PKCU_OK or an error code
 * (the message is in pkcu_last_error()). A failing drop-in also prints one
 * line to stderr. */
int pk_cuda_status(void);

/* ── 2. device API ──────────────────────────────────────────────────────────
 * The reference's tensor_ops. Any alignment is accepted here; the 16-byte
 * aligned, D % 4 == 0 case takes the vectorised kernels. */

/* pk_layer_norm_rows (csrc/tensor_ops.c:151-254): out = (x-mean)/sqrt(var+1e-5)
 * * gamma + beta per row of D. out may equal x (pk_layer_norm_rows_inplace,
 * :256-280). */
int pkcu_layer_norm_rows(const float *x, const float *gamma, const float *beta, float *out,
                         int n_rows, int D, pkcu_stream_t stream);
/* pk_softmax_rows (csrc/tensor_ops.c:284-363), in place, rows of len. */
int pkcu_softmax_rows(float *x, int n_rows, int len, pkcu_stream_t stream);
/* pk_swish (csrc/tensor_ops.c:367-397) over a flat array, in place. */
int pkcu_swish(float *x, long long n, pkcu_stream_t stream);
/* pk_relu (csrc/tensor_ops.c:401-416), in place. */
int pkcu_relu(float *x, long long n, pkcu_stream_t stream);
/* pk_bias_add (csrc/tensor_ops.c:420-435) applied to each of n_rows rows. */
int pkcu_bias_add_rows(float *x, const float *b, int n_rows, int len, pkcu_stream_t stream);
/* pk_depthwise_conv1d (csrc/tensor_ops.c:477-575): x, out [C, T]; w [C, K];
 * b [C] or NULL; symmetric zero padding (K-1)/2. */
int pkcu_depthwise_conv1d(const float *x, const float *w, const float *b, float *out, int C,
                          int T, int K, pkcu_stream_t stream);

/* Feed-forward bias + Swish (csrc/encoder.c:193-196): out = swish(in + b)
 * row-wise over [n_rows, len]; out may equal in. */
int pkcu_bias_swish_rows(const float *in, const float *b, float *out, int n_rows, int len,
                         pkcu_stream_t stream);
/* Residual (csrc/encoder.c:199-216 macaron alpha=0.5, :420-434 attention
 * alpha=1): x += alpha * (y + bias) over [n_rows, D]; bias may be NULL. */
int pkcu_residual_add(float *x, const float *y, const float *bias, float alpha, int n_rows,
                      int D, pkcu_stream_t stream);
/* Residual then the next module's LayerNorm in one pass (D = 1024):
 * x += alpha*(y + bias); ln = LN(x; gamma, beta). */
int pkcu_residual_layer_norm(float *x, const float *y, const float *bias, float alpha,
                             const float *gamma, const float *beta, float *ln, int n_rows,
                             pkcu_stream_t stream);
/* End of a block and start of the next (csrc/encoder.c:489-490 then :191):
 * x = LN_out(x + alpha*(y + bias)) in place; when g_next != NULL also
 * ln_next = LN_next(x). D = 1024. */
int pkcu_residual_layer_norm2(float *x, const float *y, const float *bias, float alpha,
                              const float *g_out, const float *b_out, const float *g_next,
                              const float *b_next, float *ln_next, int n_rows,
                              pkcu_stream_t stream);

/* Attention head gather (csrc/encoder.c:313-356): qkv [frames, 3D] (+ bqkv
 * [3D]) -> Qu = Q + u[h], Qv = Q + v[h], K, V, each per item [H, T_b, 128];
 * u, v [H, 128]. */
int pkcu_qkv_split_uv(const float *qkv, const float *bqkv, const float *u, const float *v,
                      float *Qu, float *Qv, float *K, float *V, const pkcu_seq *seq,
                      pkcu_stream_t stream);
/* Positional head split (csrc/encoder.c:362-368): P per item [2T_b-1, D] ->
 * P_h per item [H, 2T_b-1, 128]. */
int pkcu_pos_head_split(const float *P, float *P_h, const pkcu_seq *seq, pkcu_stream_t stream);
/* relative_shift (csrc/encoder.c:230-254): out[h,i,j] = bd[h,i,T-1-i+j]
 * (bd per item [H,T,2T-1], out per item [H,T,T]). */
int pkcu_relative_shift(const float *bd, float *out, const pkcu_seq *seq, pkcu_stream_t stream);
/* Score combine (csrc/encoder.c:380-400): S = (ac + rel_shift(bd)) * scale. */
int pkcu_relpos_combine(const float *ac, const float *bd, float *S, float scale,
                        const pkcu_seq *seq, pkcu_stream_t stream);
/* Score combine fused with the row softmax of csrc/encoder.c:403. S may equal ac. */
int pkcu_relpos_combine_softmax(const float *ac, const float *bd, float *S, float scale,
                                const pkcu_seq *seq, pkcu_stream_t stream);
/* Head concat (csrc/encoder.c:410-415): per item [H, T_b, 128] -> [T_b, D]. */
int pkcu_head_concat(const float *attn_h, float *attn, const pkcu_seq *seq,
                     pkcu_stream_t stream);
/* Conv-module LayerNorm + channel-first copy (csrc/encoder.c:446-452):
 * x [frames, D] -> cf per item [D, T_b]. */
int pkcu_layer_norm_transpose(const float *x, const float *gamma, const float *beta, float *cf,
                              const pkcu_seq *seq, pkcu_stream_t stream);
/* Attention residual (csrc/encoder.c:420-434) fused with the above:
 * x += alpha*(y + bias); cf = channel-first LN(x). */
int pkcu_residual_layer_norm_transpose(float *x, const float *y, const float *bias,
                                       float alpha, const float *gamma, const float *beta,
                                       float *cf, const pkcu_seq *seq, pkcu_stream_t stream);

#define PKCU_CHANNEL_FIRST 0   /* per item [2C, T_b] -> [C, T_b] (csrc/encoder.c:457-465) */
#define PKCU_TIME_FIRST    1   /* [frames, 2C] -> [frames, C] */
/* GLU with the pointwise-conv bias (csrc/tensor_ops.c:585-589) folded in:
 * a = in[c] + bias[c], g = in[C+c] + bias[C+c], out = a / (1 + exp(-g)).
 * bias may be NULL. */
int pkcu_glu(const float *in, const float *bias, float *out, int C, int layout,
             const pkcu_seq *seq, pkcu_stream_t stream);
/* Depthwise conv (csrc/tensor_ops.c:477-575) + bias, optional inference
 * BatchNorm (bn = [mean C | var C | gamma C | beta C], or NULL: the reference
 * folds BN into w/b offline), optional Swish (csrc/encoder.c:470), on
 * channel-first per item [C, T_b]; w [C, K], b [C] or NULL. */
int pkcu_dwconv_bn_swish(const float *x, const float *w, const float *b, const float *bn,
                         float bn_eps, int apply_swish, float *out, int C, int K,
                         const pkcu_seq *seq, pkcu_stream_t stream);
/* The GLU (csrc/encoder.c:457-465, as pkcu_glu with PKCU_CHANNEL_FIRST) fused
 * into the depthwise conv's input: reads the pointwise-conv output pw1 per
 * item [2C, T_b] (+ pw1_bias [2C], may be NULL) and never materialises the
 * GLU output. Bit-identical to pkcu_glu followed by pkcu_dwconv_bn_swish. */
int pkcu_glu_dwconv_bn_swish(const float *pw1, const float *pw1_bias, const float *w,
                             const float *b, const float *bn, float bn_eps, int apply_swish,
                             float *out, int C, int K, const pkcu_seq *seq,
                             pkcu_stream_t stream);
/* Conv residual (csrc/encoder.c:475-477): x[t,d] += y[d,t] + bias[d], y per
 * item [D, T_b] (bias: the pw2 bias, csrc/tensor_ops.c:585-589; may be NULL). */
int pkcu_transpose_add(float *x, const float *y, const float *bias, const pkcu_seq *seq,
                       pkcu_stream_t stream);
/* The same fused with the FF2 LayerNorm (csrc/encoder.c:489 -> :191):
 * x[t,d] += y[d,t] + bias[d]; ln = LN(x). */
int pkcu_transpose_add_layer_norm(float *x, const float *y, const float *bias,
                                  const float *gamma, const float *beta, float *ln,
                                  const pkcu_seq *seq, pkcu_stream_t stream);

/* int8 per-tensor dequant (csrc/blas.c:526-558): out = (float)q * scale. */
int pkcu_dequant_i8(const int8_t *q, float scale, float *out, long long n, pkcu_stream_t stream);
/* Fused-QKV int8 build (csrc/weights.c:437-487): ms = max(sq, sk, sv); each of
 * q, k, v [K, D] requantised to ms (clamp(roundf(x * s/ms), +-127), copied
 * when s == ms) into fused [K, 3D]. *ms_out (host) receives ms. */
int pkcu_requant_qkv_i8(const int8_t *q, const int8_t *k, const int8_t *v, float sq, float sk,
                        float sv, int8_t *fused, float *ms_out, int K, int D,
                        pkcu_stream_t stream);
#define PKCU_GROUP_ALONG_K 0   /* scales [K/G, N] */
#define PKCU_GROUP_ALONG_N 1   /* scales [K, N/G]: the reference layout, G = 32 */
/* int4 group dequant (csrc/blas.c:780-843, csrc/weights.c:505-515, format
 * extract_weights.py:589-594): packed [K, N/2] bytes, low nibble = even
 * column, signed 4-bit; out [K, N] = (float)q * scale. */
int pkcu_dequant_i4(const uint8_t *packed, const float *scales, float *out, int K, int N,
                    int group, int axis, pkcu_stream_t stream);
/* Fused-QKV int4 path (csrc/weights.c:488-544): three int4 [K, D] with
 * [K, D/G] scales -> fp32 fused [K, 3D]. */
int pkcu_dequant_i4_qkv(const uint8_t *pq, const uint8_t *pk, const uint8_t *pv,
                        const float *sq, const float *sk, const float *sv, float *fused, int K,
                        int D, int group, pkcu_stream_t stream);

#define PKCU_ACT_RELU 0   /* csrc/decoder.c:62-67 */
#define PKCU_ACT_TANH 1
/* Joint add + activation: out[b,t,j] = act(enc[b,t,j] + pred[b,j]). */
int pkcu_joint_add_act(const float *enc, const float *pred, float *out, int B, int T, int J,
                       int act, pkcu_stream_t stream);
/* Greedy argmax (csrc/decoder.c:106-114): first maximum of each row of V
 * logits, NaN never selected after index 0. out int32 [n_rows]. */
int pkcu_argmax_rows(const float *logits, int32_t *out, long long n_rows, int V,
                     pkcu_stream_t stream);

/* ── 3. sequence driver ──────────────────────────────────────────────────── */

/* Non-GEMM parameters of one conformer block (csrc/parakeet.h:78-125). */
typedef struct {
    const float *norm_ff1_w, *norm_ff1_b, *ff1_b1, *ff1_b2;
    const float *norm_sa_w, *norm_sa_b, *qkv_b, *pos_u, *pos_v, *out_b;
    const float *norm_conv_w, *norm_conv_b, *pw1_b, *dw_w, *dw_b, *pw2_b;
    const float *norm_ff2_w, *norm_ff2_b, *ff2_b1, *ff2_b2;
    const float *norm_out_w, *norm_out_b;
} pkcu_block_params;

/* GEMM outputs the non-GEMM ops consume (bias not yet added). */
typedef struct {
    const float *ff1_h;    /* [frames, 4096]     */
    const float *ff1_out;  /* [frames, 1024]     */
    const float *qkv;      /* [frames, 3072]     */
    const float *P;        /* pos [2T-1, 1024]   */
    const float *ac;       /* scores [H, T, T]   */
    const float *bd;       /* bd [H, T, 2T-1]    */
    const float *attn_h;   /* heads [H, T, 128]  */
    const float *att_out;  /* [frames, 1024]     */
    const float *pw1;      /* channel-first [2048, T] */
    const float *pw2;      /* channel-first [1024, T] */
    const float *ff2_h;    /* [frames, 4096]     */
    const float *ff2_out;  /* [frames, 1024]     */
} pkcu_gemm_outputs;

/* GEMM inputs the non-GEMM ops produce (per-item layouts as above). Buffers
 * whose consumers run one after another may alias (e.g. the four LN outputs). */
typedef struct {
    float *ln_ff1, *h1, *ln_sa, *Qu, *K, *Qv, *P_h, *S, *V, *attn, *cf, *dw, *ln_ff2, *h2;
    float *gated;   /* GLU output [D, T] per item: not written by the fused sequence (may be NULL) */
} pkcu_gemm_inputs;

/* GEMM points, in the order they occur in one block. */
enum {
    PKCU_GEMM_FF1_1 = 0, PKCU_GEMM_FF1_2, PKCU_GEMM_QKV, PKCU_GEMM_POS, PKCU_GEMM_AC,
    PKCU_GEMM_BD, PKCU_GEMM_AV, PKCU_GEMM_OUT, PKCU_GEMM_PW1, PKCU_GEMM_PW2,
    PKCU_GEMM_FF2_1, PKCU_GEMM_FF2_2
};
/* Called (on the host, in stream order) where a GEMM runs: it must enqueue on
 * `stream` the product that fills the matching pkcu_gemm_outputs buffer from
 * the pkcu_gemm_inputs buffers of block `block`. Return PKCU_OK to continue.
 * With no hook the pkcu_gemm_outputs buffers are consumed as they are. */
typedef int (*pkcu_gemm_hook)(void *user, int block, int gemm, pkcu_stream_t stream);

/* Runs n_blocks conformer blocks' non-GEMM ops (csrc/encoder.c:482-491) on x
 * [frames, D] in place, fused at producer/consumer boundaries:
 *   LN_ff1 | bias+Swish | res+LN_sa | QKV split | pos split | combine+softmax |
 *   head concat | res+LN_conv+transpose | GLU+dwconv+bias+Swish |
 *   transpose-add+LN_ff2 | bias+Swish | res+LN_out(+LN_ff1 of the next block)
 * All pointers are device pointers; blocks[] is a host array. */
int pkcu_encoder_nongemm(float *x, const pkcu_block_params *blocks, int n_blocks,
                         const pkcu_gemm_outputs *gemm_out, const pkcu_gemm_inputs *gemm_in,
                         const pkcu_seq *seq, pkcu_gemm_hook hook, void *hook_user,
                         pkcu_stream_t stream);

/* The same sequence with some GEMM epilogues done by the hook's GEMMs
 * (pkcu_encoder_forward uses this with its tcgen05 GEMMs):
 *   PKCU_FUSED_FF_SWISH -- the FF1_1 / FF2_1 hooks write Swish(x W + b1) into
 *     gemm_in->h1 / h2 themselves; the sequence's bias+Swish steps are skipped;
 *   PKCU_FUSED_QKV -- the QKV hook writes Qu, Qv, K, V (bias, head split and
 *     pos_bias_u / v, as pkcu_qkv_split_uv) itself; that step is skipped;
 *   PKCU_FUSED_CONV -- the conv module's GEMMs carry its epilogues: the
 *     sequence writes LN_conv time-first ([frames, 1024]) into gemm_in->cf,
 *     the PW1 hook writes the GLU output (bias included) into gemm_in->gated
 *     (per item [1024, T]), the depthwise conv reads it, and the PW2 hook adds
 *     pw2 + bias to x itself (the residual of csrc/encoder.c:475-477); the
 *     sequence then takes LN_ff2 of x.
 * The skipped GEMM outputs (ff1_h, ff2_h, qkv, pw1, pw2) are then not read. */
#define PKCU_FUSED_FF_SWISH 1u
#define PKCU_FUSED_QKV      2u
#define PKCU_FUSED_CONV     4u
int pkcu_encoder_nongemm_fused(float *x, const pkcu_block_params *blocks, int n_blocks,
                               const pkcu_gemm_outputs *gemm_out, const pkcu_gemm_inputs *gemm_in,
                               const pkcu_seq *seq, pkcu_gemm_hook hook, void *hook_user,
                               unsigned fused, pkcu_stream_t stream);

/* Number of kernel launches pkcu_encoder_nongemm makes for n_blocks blocks. */
int pkcu_encoder_nongemm_launches(int n_blocks);

/* Host-buffer form (the reference's pk_encoder takes and returns host
 * buffers, csrc/encoder.c:612-633). A workspace owns the device copies of x,
 * the GEMM outputs and the GEMM inputs for one batch shape, split into
 * n_groups groups of consecutive items. pkcu_encoder_nongemm_host copies x
 * and the GEMM outputs (host arrays in the batch layouts above) to the device,
 * runs the sequence and copies x back, pipelining the copies of one group
 * against the compute of the next; it returns when x_host holds the result.
 * Host arrays should be page-locked for the copies to overlap. */
typedef struct pkcu_encoder_ws pkcu_encoder_ws;
int  pkcu_encoder_ws_create(const pkcu_seq *seq, int n_groups, pkcu_encoder_ws **out);
void pkcu_encoder_ws_destroy(pkcu_encoder_ws *ws);
/* Device views of the workspace's whole-batch buffers. */
int  pkcu_encoder_ws_device(pkcu_encoder_ws *ws, float **x, pkcu_gemm_outputs *gemm_out,
                            pkcu_gemm_inputs *gemm_in);
long long pkcu_encoder_ws_device_bytes(const pkcu_encoder_ws *ws);
long long pkcu_encoder_ws_h2d_bytes(const pkcu_encoder_ws *ws);   /* per host call */
long long pkcu_encoder_ws_d2h_bytes(const pkcu_encoder_ws *ws);   /* per host call */
int  pkcu_encoder_nongemm_host(pkcu_encoder_ws *ws, float *x_host,
                               const pkcu_gemm_outputs *gemm_out_host,
                               const pkcu_block_params *blocks, int n_blocks,
                               pkcu_stream_t stream);

/* ── pre-encode: subsampling and input scaling (csrc/encoder.c:103-175, 578-593) ──
 * For a batch of utterances of T_b mel frames (mel per utterance [128, T_b],
 * utterance after utterance): conv0 (1 -> 256, 3x3 stride 2) + ReLU and the
 * depthwise 3x3 stride-2 conv fused in one kernel, the first 1x1 conv (GEMM),
 * its bias + ReLU folded into the second depthwise conv, the second 1x1 conv
 * (GEMM), its bias + ReLU folded into the flatten, the output projection
 * (GEMM), then x = (proj + bias) * sqrt(1024), the blocks' input [F', 1024].
 * Output frames per utterance T'_b = ceil(ceil(ceil(T_b/2)/2)/2). The
 * [256, *] tensors are channel-major across the batch: row c holds every
 * utterance's plane in turn, so each 1x1 conv is one GEMM
 * [256 x 256] x [256 x P] (P = pkcu_pre_plan_p2 / _p3). */
typedef struct pkcu_pre_plan pkcu_pre_plan;
int pkcu_pre_plan_create(const int *mel_lengths, int n_items, pkcu_pre_plan **out);
void pkcu_pre_plan_destroy(pkcu_pre_plan *p);
long long pkcu_pre_plan_p2(const pkcu_pre_plan *p);      /* columns of pw1's [256, P2] */
long long pkcu_pre_plan_p3(const pkcu_pre_plan *p);      /* columns of pw2's [256, P3] */
long long pkcu_pre_plan_frames(const pkcu_pre_plan *p);  /* F' = sum of T'_b */
/* The T'_b batch descriptor for pkcu_encoder_nongemm (owned by the plan). */
const pkcu_seq *pkcu_pre_plan_out_seq(const pkcu_pre_plan *p);

typedef struct {   /* [256, 1, 3, 3] weights, [256] / [1024] biases (csrc/parakeet.h:59-76) */
    const float *conv0_w, *conv0_b, *conv2_w, *conv2_b, *conv3_b;
    const float *conv5_w, *conv5_b, *conv6_b, *out_b;
} pkcu_pre_params;
typedef struct {   /* GEMM products, bias not added */
    float *pw1;    /* [256, P2] = W3 [256, 256] x s2d */
    float *pw2;    /* [256, P3] = W6 x s3d */
    float *proj;   /* [F', 1024] = flat x W_out [4096, 1024] */
} pkcu_pre_gemm_outputs;
typedef struct {
    float *s2d;    /* [256, P2] */
    float *s3d;    /* [256, P3] */
    float *flat;   /* [F', 4096] */
} pkcu_pre_gemm_inputs;
enum { PKCU_GEMM_PRE_PW1 = 16, PKCU_GEMM_PRE_PW2, PKCU_GEMM_PRE_OUT };
/* Runs the stage; hook (block -1) at each GEMM as in pkcu_encoder_nongemm. */
int pkcu_pre_encode(const float *mel, const pkcu_pre_params *params,
                    const pkcu_pre_gemm_outputs *gemm_out, const pkcu_pre_gemm_inputs *gemm_in,
                    float *x, const pkcu_pre_plan *plan, pkcu_gemm_hook hook, void *hook_user,
                    pkcu_stream_t stream);

/* ── GEMMs with the non-GEMM epilogue fused (tcgen05 tensor cores) ─────────
 * A [M, K] x W [K, N] (row-major fp32, the reference's pk_wmatmul layout,
 * csrc/tensor_ops.c:50-61) computed on the B200's tensor cores with fp32-level
 * accuracy (each fp32 operand split into three bf16 parts, nine bf16 MMAs per
 * product, fp32 accumulation), the bias / activation / residual applied to the
 * accumulator tile before the single store. N, K multiples of 4; A, W, bias and
 * the output 16-byte aligned. */
/* D = Swish(A W + bias): FF linear1 + bias + Swish (csrc/encoder.c:193-196). */
int pkcu_gemm_bias_swish(const float *A, const float *W, const float *bias, float *D,
                         int M, int N, int K, pkcu_stream_t stream);
/* X = X + scale * (A W + bias), in place: FF linear2 + the 0.5-scaled macaron
 * residual (csrc/encoder.c:198-216, scale 0.5), attention output projection +
 * residual (:418-434, scale 1). */
int pkcu_gemm_bias_residual(const float *A, const float *W, const float *bias, float *X,
                            float scale, int M, int N, int K, pkcu_stream_t stream);

/* ── weight products on the library's own tcgen05 GEMM ───────────────────────
 * pk_wmatmul (csrc/tensor_ops.c:50-61) and the epilogues that follow it in a
 * block, for the reference's three weight storages (Weight, csrc/parakeet.h:
 * 52-57): float32 (cblas_sgemm_st), int8 with one per-tensor scale
 * (cblas_sgemm_qb, csrc/blas.c:759, dequantised while packing :526-558) and
 * GPTQ int4 with group scales (cblas_sgemm_q4b, :950, :780-843). fp32
 * accurate on the bf16 tensor cores: the activation as three bf16 parts, an
 * int8 weight as its q (exact in bf16, the scale applied to the sum), a float32
 * or int4 weight as the three bf16 parts of its fp32 values (int4: (float)q *
 * scale first, bit for bit); tcgen05.mma with TMEM accumulators drained to
 * fp32 every 24 MMAs.
 * A weight is prepared once (synchronous): data is device memory, [K, N]
 * row-major for bits 32 / 8, packed [K, N/2] bytes + scales for bits 4 (group /
 * axis as pkcu_dequant_i4; the reference's layout is 32, PKCU_GROUP_ALONG_N);
 * K and N multiples of 32. Every call needs a work buffer of
 * pkcu_wmatmul_work_bytes(M, K) bytes (the activation's parts), 16-byte
 * aligned; calls sharing one run one at a time. All arrays are device
 * memory, 16-byte aligned, rows packed. */
typedef struct pkcu_weight pkcu_weight;
int  pkcu_weight_create(const void *data, int bits, float scale, const float *scales, int group,
                        int axis, int K, int N, pkcu_stream_t stream, pkcu_weight **out);
void pkcu_weight_destroy(pkcu_weight *w);
long long pkcu_wmatmul_work_bytes(int M, int K);
/* C[M, N] = alpha A[M, K] W + beta C (pk_wmatmul). */
int pkcu_wmatmul(const float *A, const pkcu_weight *W, float *C, int M, float alpha, float beta,
                 void *work, pkcu_stream_t stream);
/* D = Swish(A W + bias): feed_forward's linear1 + pk_bias_add + pk_swish
 * (csrc/encoder.c:193-196), Swish the reference's polynomial form. */
int pkcu_wmatmul_bias_swish(const float *A, const pkcu_weight *W, const float *bias, float *D,
                            int M, void *work, pkcu_stream_t stream);
/* X += scale (A W + bias), one fused multiply-add per entry: linear2 + the
 * 0.5 macaron residual (csrc/encoder.c:198-216), the output projection + the
 * attention residual (scale 1, :418-434). */
int pkcu_wmatmul_bias_residual(const float *A, const pkcu_weight *W, const float *bias, float *X,
                               float scale, int M, void *work, pkcu_stream_t stream);
/* The fused QKV projection with its bias, head split and pos_bias_u / v
 * (csrc/encoder.c:313-356) in the epilogue: A = the batch's LN_sa rows
 * [frames, 1024], W the fused [1024, 3072] weight, outputs as
 * pkcu_qkv_split_uv writes them (per item [8, T, 128]). */
int pkcu_wmatmul_qkv(const float *A, const pkcu_weight *W, const float *bqkv, const float *u,
                     const float *v, float *Qu, float *Qv, float *K, float *V, const pkcu_seq *seq,
                     void *work, pkcu_stream_t stream);

/* pk_pointwise_conv1d (csrc/tensor_ops.c:579-590) on the same GEMM: x [Cin, T]
 * channel-first, W [Cout, Cin] (float32, as the reference stores it; prepared
 * once, synchronous; glu != 0 prepares it for pkcu_pointwise_conv1d_glu),
 * out [Cout, T] = W x + b[c]; b may be NULL. Work: pkcu_wmatmul_work_bytes(T,
 * Cin) bytes. Cin a multiple of 32, Cout of 32 (64 with glu). */
int pkcu_conv_weight_create(const float *w, int Cout, int Cin, int glu, pkcu_stream_t stream,
                            pkcu_weight **out);
int pkcu_pointwise_conv1d(const float *x, const pkcu_weight *W, const float *b, float *out, int T,
                          void *work, pkcu_stream_t stream);
/* The first pointwise convolution and the GLU after it (csrc/encoder.c:454-465)
 * in one pass: gated [Cout/2, T] = a * 1/(1 + expf(-g)), a = rows [0, Cout/2)
 * of W x + b, g = rows [Cout/2, Cout). */
int pkcu_pointwise_conv1d_glu(const float *x, const pkcu_weight *W, const float *b, float *gated, int T,
                              void *work, pkcu_stream_t stream);

/* ── the encoder stack on the GPU, GEMMs included ──────────────────────────
 * Replaces encode_blocks (csrc/encoder.c:495-512) for a batch: fp32 device
 * copies of every block's GEMM weights from an uploaded checkpoint (int8 /
 * int4 dequantised once, the fused QKV as the reference's loader builds it),
 * then pkcu_encoder_nongemm with its twelve GEMM points done by the library,
 * fp32-accurate: the projections (the positional one on each distinct
 * utterance length's slice of pos_encoding.pe_table, csrc/encoder.c:220-227)
 * and the pointwise convolutions as bf16 tensor-core GEMMs on operands split
 * into three bf16 parts (the weights' parts made once here; an int8 weight
 * with a per-tensor scale is used as stored, q exact in bf16), the per-head
 * products as cuBLAS single-precision GEMMs (no TF32). A model keeps a working
 * buffer for the split operands (grown by the largest forward so far), so one
 * model serves one forward at a time. */
typedef struct pkcu_weights pkcu_weights;   /* a loaded checkpoint (section 4 below) */
typedef struct pkcu_encoder_model pkcu_encoder_model;
int  pkcu_encoder_model_create(const pkcu_weights *w, pkcu_stream_t stream, pkcu_encoder_model **out);
void pkcu_encoder_model_destroy(pkcu_encoder_model *m);
int  pkcu_encoder_model_blocks(const pkcu_encoder_model *m);
/* All blocks on x [frames, 1024] in place; gemm_out / gemm_in: device buffers
 * for the batch (those of a 1-group pkcu_encoder_ws fit), used as scratch.
 * With every projection on the tensor-core GEMM the FF hidden layers stay in
 * the model's own buffer as the second product's bf16 operand parts, so
 * gemm_in->h1 / h2 are not written. */
int  pkcu_encoder_forward(pkcu_encoder_model *m, float *x, const pkcu_gemm_outputs *gemm_out,
                          const pkcu_gemm_inputs *gemm_in, const pkcu_seq *seq,
                          pkcu_stream_t stream);

/* ── long audio: the chunked encoder (csrc/encoder.c:514-575, 597-633) ──────
 * The reference encodes an utterance of more than PK_CHUNK_THRESHOLD encoder
 * frames in chunks: chunk c owns frames [400c, min(400c + 400, T)) and runs the
 * blocks over them plus up to 8 frames of overlap each side (clipped to the
 * utterance), with the positional encoding of its own input length; only the
 * owned frames are kept. A chunk plan lays the chunks of a batch of
 * utterances out as one ragged batch (pkcu_chunk_plan_seq; an utterance that
 * is not chunked is one item of its full length), so one pkcu_encoder_forward
 * or pkcu_encoder_nongemm call encodes them all:
 *   pkcu_chunk_split (x [sum T, 1024] -> xc [chunk frames, 1024]),
 *   the blocks on xc with the plan's seq, pkcu_chunk_stitch (xc -> x).
 * pkcu_encoder_forward itself never chunks (it is encode_blocks);
 * pkcu_asr_transcribe chunks as pk_encoder does. */
#define PKCU_CHUNK_SIZE      400   /* csrc/parakeet.h:132 */
#define PKCU_CHUNK_OVERLAP   8     /* csrc/parakeet.h:133 */
#define PKCU_CHUNK_THRESHOLD 500   /* csrc/parakeet.h:134 */
/* AUTO: should_chunk (csrc/encoder.c:602-610) -- the PK_CHUNK environment
 * variable ("0"/"off": never, "1"/"on": always), else T > 500; OFF / ON: never
 * / always, whatever the environment says. */
#define PKCU_CHUNK_AUTO 0
#define PKCU_CHUNK_OFF  1
#define PKCU_CHUNK_ON   2
int  pkcu_should_chunk(int frames, int mode);
/* Chunk bounds of one utterance (host only, no CUDA call): chunk c reads
 * in_len[c] frames from in_start[c] and owns out_len[c] frames from
 * out_start[c]; an utterance that is not chunked is one chunk of all its
 * frames. Returns the number of chunks; with every array NULL it only counts,
 * else -1 when that exceeds cap (or frames <= 0). */
int  pkcu_chunk_bounds(int frames, int mode, int cap, int *in_start, int *in_len, int *out_start,
                       int *out_len);
typedef struct pkcu_chunk_plan pkcu_chunk_plan;
int  pkcu_chunk_plan_create(const int *frames, int n_utts, int mode, pkcu_chunk_plan **out);
void pkcu_chunk_plan_destroy(pkcu_chunk_plan *p);
const pkcu_seq *pkcu_chunk_plan_seq(const pkcu_chunk_plan *p);   /* the chunk batch */
int  pkcu_chunk_plan_chunked(const pkcu_chunk_plan *p);          /* utterances split */
int  pkcu_chunk_plan_items(const pkcu_chunk_plan *p);            /* items of the chunk batch */
/* Item `item` of the chunk batch: its utterance, its first input frame in that
 * utterance and its frame count (any pointer may be NULL). */
int  pkcu_chunk_plan_item(const pkcu_chunk_plan *p, int item, int *utt, int *first_frame,
                          int *frames);
/* Device arrays, 16-byte aligned; asynchronous on stream. */
int  pkcu_chunk_split(const pkcu_chunk_plan *p, const float *x, float *xc, pkcu_stream_t stream);
int  pkcu_chunk_stitch(const pkcu_chunk_plan *p, const float *xc, float *x, pkcu_stream_t stream);

/* ── mel spectrograms to tokens on the GPU ─────────────────────────────────
 * pre_encode_and_scale + encode_blocks + pk_greedy_decode (csrc/encoder.c:
 * 578-593, 495-512; csrc/decoder.c:80-132) for a batch of utterances, every
 * GEMM done by the library (fp32-accurate tensor-core GEMMs where the shape
 * suits them, cuBLAS single precision elsewhere). One pkcu_asr serves one call
 * at a time: its calls share the kept working buffers and decoder. */
typedef struct pkcu_asr pkcu_asr;
int  pkcu_asr_create(const pkcu_weights *w, pkcu_stream_t stream, pkcu_asr **out);
void pkcu_asr_destroy(pkcu_asr *m);
/* Encoder frames of an utterance of mel_frames frames: ceil(ceil(ceil(T/2)/2)/2). */
int  pkcu_asr_encoder_frames(int mel_frames);
/* mel: device, n_utts spectrograms [128, mel_frames[b]] one after another.
 * tokens (host, capacity 10 x the sum of encoder frames) receives utterance
 * b's tokens from 10 x the number of encoder frames before it; n_tokens (host)
 * their counts. Synchronous. The working buffers (and the decoder, with its
 * captured graph) of the last call are kept while the same lengths come again
 * (a call with other lengths replaces them; pkcu_asr_destroy frees them). */
int  pkcu_asr_transcribe(pkcu_asr *m, const float *mel, const int *mel_frames, int n_utts,
                         int *tokens, int *n_tokens, pkcu_stream_t stream);
/* pk_encoder (csrc/encoder.c:612-633) for a batch: pre-encode and the blocks,
 * utterances above the chunk threshold encoded in chunks (the model's chunk
 * mode, PKCU_CHUNK_AUTO by default: the reference's should_chunk, PK_CHUNK
 * included). enc (device) receives [sum encoder frames, 1024], utterance
 * after utterance. Synchronous; pkcu_asr_transcribe encodes the same way. */
int  pkcu_asr_encode(pkcu_asr *m, const float *mel, const int *mel_frames, int n_utts,
                     float *enc, pkcu_stream_t stream);
int  pkcu_asr_set_chunk_mode(pkcu_asr *m, int mode);   /* PKCU_CHUNK_AUTO / _OFF / _ON */
/* The decode alone, a batched pk_greedy_decode (csrc/decoder.c:80-132) with
 * the model's decoder: enc (device, 16-byte aligned) holds the encoder
 * outputs [enc_frames[b], 1024] of n_utts utterances one after another;
 * tokens / n_tokens as for pkcu_asr_transcribe. */
int  pkcu_asr_decode(pkcu_asr *m, const float *enc, const int *enc_frames, int n_utts,
                     int *tokens, int *n_tokens, pkcu_stream_t stream);
/* How pkcu_asr_transcribe and pkcu_asr_decode decode: FUSED (the default) -- the decoder's own
 * CUDA-core product kernels (pkcu_greedy_decode_fused); TC -- the products on
 * the library's tcgen05 GEMM at the decoder's hooks inside its CUDA graph;
 * GRAPH -- cuBLAS products at those hooks (pkcu_greedy_decode_graph);
 * EAGER -- the cuBLAS products launched one at a time (pkcu_greedy_decode).
 * The encoder projection (joint.enc) runs on the tcgen05 GEMM in every mode. */
#define PKCU_ASR_DECODE_FUSED 0
#define PKCU_ASR_DECODE_GRAPH 1
#define PKCU_ASR_DECODE_EAGER 2
#define PKCU_ASR_DECODE_TC    3
int  pkcu_asr_set_decode_mode(pkcu_asr *m, int mode);

/* ── batched greedy RNN-T decode (csrc/decoder.c:80-132) ──────────────────
 * Replaces pk_greedy_decode for a batch of utterances (the encoder outputs of
 * n_utts utterances of T_b frames, frames of every utterance in turn). Every
 * utterance goes through the reference's own sequence -- a decoder step on
 * blank, then per frame up to 10 x { joint, first-maximum argmax; blank ->
 * next frame; else emit the token and run a decoder step } -- one joint
 * evaluation per utterance per iteration. The non-GEMM work (embedding rows,
 * LSTM cells csrc/tensor_ops.c:594-629, joint bias adds + add + ReLU
 * csrc/decoder.c:38-76, bias + argmax, the state machine) runs as kernels;
 * each matrix-vector product of the reference is a batched GEMM that the
 * hook enqueues (block = -1, gemm = PKCU_GEMM_DEC_*), computed for every
 * utterance's row: rows that do not need it ignore it. */
typedef struct pkcu_decoder pkcu_decoder;
typedef struct {
    const float *embed;        /* [1025, 640] decoder.prediction.embed.weight (16-byte aligned) */
    const float *lstm0_b;      /* [5120] decoder.lstm.0.B */
    const float *lstm1_b;      /* [5120] decoder.lstm.1.B */
    const float *joint_enc_b;  /* [640] (16-byte aligned) */
    const float *joint_pred_b; /* [640] (16-byte aligned) */
    const float *joint_out_b;  /* [1025] joint.joint_net.2.bias */
} pkcu_dec_params;
typedef struct {   /* products the hook writes, bias not added (device, owned by the decoder) */
    float *enc;    /* [F, 640]   = encoder output [F, 1024] x joint.enc.weight   (DEC_ENC, once) */
    float *pred;   /* [B, 640]   = h1 x joint.pred.weight                         (DEC_PRED) */
    float *out;    /* [B, 1025]  = hidden x joint.out.weight                      (DEC_OUT) */
    float *g0i, *g0r, *g1i, *g1r;   /* [B, 2560] = x0 W_i0^T, h0 W_r0^T, h0 W_i1^T, h1 W_r1^T */
} pkcu_dec_gemm_outputs;
typedef struct {   /* the products' inputs, written by the decode (device, owned by the decoder) */
    float *x0;     /* [B, 640] embedding rows of the tokens whose decoder step is pending */
    float *h0;     /* [B, 640] layer-0 hidden state: input of W_r0 (before its cell), of W_i1 (after) */
    float *h1;     /* [B, 640] layer-1 hidden state: input of W_r1 (before), of joint.pred (after) */
    float *hidden; /* [B, 640] joint hidden (zeros for finished utterances) */
} pkcu_dec_gemm_inputs;
enum { PKCU_GEMM_DEC_ENC = 32, PKCU_GEMM_DEC_L0_WI, PKCU_GEMM_DEC_L0_WR, PKCU_GEMM_DEC_L1_WI,
       PKCU_GEMM_DEC_L1_WR, PKCU_GEMM_DEC_PRED, PKCU_GEMM_DEC_OUT };
/* Device state and buffers for a batch of utterances of frames[b] >= 1 frames
 * (B = n_utts, F = sum of frames). */
int  pkcu_decoder_create(const int *frames, int n_utts, pkcu_decoder **out);
void pkcu_decoder_destroy(pkcu_decoder *dec);
int  pkcu_decoder_buffers(const pkcu_decoder *dec, pkcu_dec_gemm_outputs *gemm_out,
                          pkcu_dec_gemm_inputs *gemm_in);
/* Runs the decode to the end (the host polls the device every 8 iterations).
 * Order per iteration: L0_WI, L0_WR, L1_WI, L1_WR, PRED, OUT hooks, with the
 * kernels between them; DEC_ENC once before the first. */
int  pkcu_greedy_decode(pkcu_decoder *dec, const pkcu_dec_params *params, pkcu_gemm_hook hook,
                        void *hook_user, pkcu_stream_t stream);
/* The same decode with the hook's per-iteration GEMMs inside the decoder's
 * CUDA graph of 8 iterations: the hook must be capture-safe (only stream-
 * ordered work on the stream it is given, e.g. cuBLAS calls, no synchronisation
 * or allocation) and its work must not depend on the iteration. It is called
 * 8 times per product for each of the decoder's two graphs while they are
 * captured (the host launches one while it reads the other's live count), and
 * again only when the hook, its user pointer or the parameter pointers change;
 * DEC_ENC is called once per decode outside the graphs. */
int  pkcu_greedy_decode_graph(pkcu_decoder *dec, const pkcu_dec_params *params,
                              pkcu_gemm_hook hook, void *hook_user, pkcu_stream_t stream);
/* The decode with its own products: the decoder's weights in the reference's
 * layouts -- LSTM W_i / W_r [2560, 640] (csrc/decoder.c:20-27), joint.pred
 * [640, 640] and joint.out [640, 1025] as (in, out) (csrc/decoder.c:53-72),
 * device, 16-byte aligned; the LSTM matrices must outlive the decodes, the
 * joint matrices are copied (transposed) by pkcu_decoder_set_weights. */
typedef struct {
    const float *lstm0_wi, *lstm0_wr, *lstm1_wi, *lstm1_wr;
    const float *joint_pred, *joint_out;
} pkcu_dec_weights;
int  pkcu_decoder_set_weights(pkcu_decoder *dec, const pkcu_dec_weights *w, pkcu_stream_t stream);
/* Runs the decode with every product but DEC_ENC done by the decoder's own
 * kernels (fp32; per iteration: LSTM layer 0 and 1 with their cells, pred +
 * joint hidden, out, argmax + state), replayed as a CUDA graph of 8
 * iterations. The encoder projection (the DEC_ENC product) must be in
 * gemm_out.enc before the call. */
int  pkcu_greedy_decode_fused(pkcu_decoder *dec, const pkcu_dec_params *params, pkcu_stream_t stream);
int  pkcu_decoder_iterations(const pkcu_decoder *dec);   /* of the last decode */
/* Host copies (any may be NULL): n_tokens[B], evals[B] (joint evaluations per
 * utterance), tokens[10 F] (utterance b's tokens start at 10 x its first frame). */
int  pkcu_decoder_results(const pkcu_decoder *dec, int *n_tokens, int *evals, int *tokens,
                          pkcu_stream_t stream);

/* ── 4. weights: the reference checkpoint format on the device ─────────────
 * Replaces pk_load_weights / lookup_weight / pk_free_weights
 * (csrc/weights.c:240-402, 551-564) for a GPU engine: weights.bin +
 * weights.json as written by extract_weights.py:894-945. Open parses the
 * manifest and reads the file on the host (no CUDA call); upload puts every
 * tensor in its own 256-byte aligned slot of one device allocation on the
 * current device and builds each block's fused QKV weight and bias as the
 * reference does after loading (csrc/weights.c:403-544). Device pointers
 * stay valid until pkcu_weights_destroy. */
#define PKCU_DTYPE_F32 0
#define PKCU_DTYPE_I8  1   /* per-tensor scale */
#define PKCU_DTYPE_I4  2   /* packed [K, N/2], fp32 group scales [K, N/32] */

typedef struct pkcu_weights pkcu_weights;

typedef struct {
    int dtype;                  /* PKCU_DTYPE_*, as stored */
    int ndim;
    long long shape[4];         /* manifest shape (int4: the packed [K, N/2]) */
    long long numel;            /* elements (float32, int8) or packed bytes (int4) */
    float scale;                /* int8 per-tensor scale, else 0 */
    long long n_scales;         /* int4 group scales, else 0 */
    const void *host;           /* the bytes in the host copy of weights.bin */
    const float *host_scales;   /* int4 */
    const void *dev;            /* device copy; NULL before upload */
    const float *dev_scales;    /* int4, device */
} pkcu_tensor;

int pkcu_weights_open(const char *bin_path, const char *json_path, pkcu_weights **out);
int pkcu_weights_upload(pkcu_weights *w, pkcu_stream_t stream);   /* synchronous */
void pkcu_weights_destroy(pkcu_weights *w);
int pkcu_weights_count(const pkcu_weights *w);
const char *pkcu_weights_name(const pkcu_weights *w, int index);   /* manifest order */
/* Conformer blocks present (layers.0 .. with a linear_q weight). */
int pkcu_weights_blocks(const pkcu_weights *w);
/* lookup_weight (csrc/weights.c:240-266): PKCU_ERR_ARG if the name is absent. */
int pkcu_weights_find(const pkcu_weights *w, const char *name, pkcu_tensor *t);
/* Any tensor as fp32 on the device: float32 copied, int8 (float)q * scale,
 * int4 (float)nibble * scale[k, col/32], the reference's dequant formulas. */
int pkcu_weights_dequant(const pkcu_weights *w, const char *name, float *out,
                         pkcu_stream_t stream);
/* Block b's fused QKV (csrc/weights.c:403-544): int8 [D, 3D] at the common
 * scale (*bits = 8, *scale = max(sq, sk, sv)) when q, k, v are int8; fp32
 * [D, 3D] (*bits = 32) when they are float32 or int4; bias = [Bq | Bk | Bv]. */
int pkcu_weights_fused_qkv(const pkcu_weights *w, int block, const void **weight, int *bits,
                           float *scale, const float **bias);
/* The non-GEMM parameters of block b for pkcu_encoder_nongemm (qkv_b is the
 * fused bias above). */
int pkcu_weights_block_params(const pkcu_weights *w, int block, pkcu_block_params *p);
/* The pre-encode parameters (pre_encode.conv.{0,2,3,5,6}.*, pre_encode.out.bias). */
int pkcu_weights_pre_params(const pkcu_weights *w, pkcu_pre_params *p);

#ifdef __cplusplus
}
#endif

#endif /* PKCUDA_H */
