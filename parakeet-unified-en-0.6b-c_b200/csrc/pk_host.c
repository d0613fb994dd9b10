/* pk_host.c -- host side of libpk_tensor_ops_cuda.so (plain C over the CUDA
 * runtime): status and error reporting, batch descriptors, the drop-in
 * host-pointer API with the prototypes of csrc/parakeet.h:231-262, and the
 * per-block non-GEMM sequence driver.
 *
 * Replaces the reference's thread-pool dispatch (pk_parallel,
 * csrc/threadpool.c:183-212): where the reference forks rows across pthreads
 * and joins, a call here is one kernel launch on a CUDA stream. */
#include <cuda_runtime_api.h>
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pkcuda_internal.h"

/* ── status ──────────────────────────────────────────────────────────────── */

static __thread char tls_err[512];

const char *pkcu_version(void) { return "0.1.0"; }

const char *pkcu_status_string(int status)
{
    switch (status) {
    case PKCU_OK: return "ok";
    case PKCU_ERR_ARG: return "invalid argument";
    case PKCU_ERR_CUDA: return "CUDA error";
    case PKCU_ERR_NOMEM: return "out of memory";
    default: return "unknown status";
    }
}

const char *pkcu_last_error(void) { return tls_err; }

int pkcu_fail(int status, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(tls_err, sizeof(tls_err), fmt, ap);
    va_end(ap);
    return status;
}

int pkcu_launch_status(const char *what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return pkcu_fail(PKCU_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return PKCU_OK;
}

#define PK_MAX_DEVICES 64
static int g_sm_count[PK_MAX_DEVICES];

int pkcu_device(void)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= PK_MAX_DEVICES) return 0;
    return dev;
}

int pkcu_wait_timeouts(unsigned *count, int reset)
{
    if (!count) return pkcu_fail(PKCU_ERR_ARG, "pkcu_wait_timeouts: NULL count");
    unsigned a = 0, b = 0, c = 0;
    if (pk_softmax_wait_timeouts(&a, reset) != PKCU_OK || pk_conv_wait_timeouts(&b, reset) != PKCU_OK ||
        pk_tc_wait_timeouts(&c, reset) != PKCU_OK)
        return pkcu_fail(PKCU_ERR_CUDA, "pkcu_wait_timeouts: reading the device counters failed");
    *count = a + b + c;
    return PKCU_OK;
}

int pk_check_wait_timeouts(const char *what)
{
    unsigned a = 0, b = 0, c = 0;
    if (pk_softmax_wait_timeouts(&a, 1) != PKCU_OK || pk_conv_wait_timeouts(&b, 1) != PKCU_OK ||
        pk_tc_wait_timeouts(&c, 1) != PKCU_OK) {
        cudaGetLastError();
        return pkcu_fail(PKCU_ERR_CUDA, "%s: reading the device wait counters failed", what);
    }
    if (a + b + c)
        return pkcu_fail(PKCU_ERR_CUDA, "%s: %u bounded device wait(s) ran out; outputs are incomplete",
                         what, a + b + c);
    return PKCU_OK;
}

int pkcu_sm_count(void)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= PK_MAX_DEVICES) return 148;
    if (!g_sm_count[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        g_sm_count[dev] = n;
    }
    return g_sm_count[dev];
}

/* ── batches ─────────────────────────────────────────────────────────────── */

int pkcu_seq_create(const int *lengths, int n_items, pkcu_seq **out)
{
    if (!out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_seq_create: NULL out");
    *out = NULL;
    if (!lengths || n_items <= 0) return pkcu_fail(PKCU_ERR_ARG, "pkcu_seq_create: no items");
    int uniform = 1, max_T = 0;
    for (int i = 0; i < n_items; i++) {
        if (lengths[i] <= 0 || lengths[i] > (1 << 20))
            return pkcu_fail(PKCU_ERR_ARG, "pkcu_seq_create: item %d has length %d", i, lengths[i]);
        if (lengths[i] != lengths[0]) uniform = 0;
        if (lengths[i] > max_T) max_T = lengths[i];
    }
    pkcu_seq *s = (pkcu_seq *)calloc(1, sizeof(*s));
    if (!s) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_seq_create: host allocation");
    s->lengths = (int *)malloc((size_t)n_items * sizeof(int));
    if (!s->lengths) { free(s); return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_seq_create: host allocation"); }
    memcpy(s->lengths, lengths, (size_t)n_items * sizeof(int));
    cudaGetDevice(&s->device);

    /* Host prefix sums (also the device arrays of a ragged batch). */
    size_t n1 = (size_t)n_items + 1;
    long long *pre = (long long *)calloc(4 * n1, sizeof(long long));
    if (!pre) { free(s->lengths); free(s); return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_seq_create"); }
    long long *fo = pre, *so = pre + n1, *bo = pre + 2 * n1, *po = pre + 3 * n1;
    for (int i = 0; i < n_items; i++) {
        long long T = lengths[i];
        fo[i + 1] = fo[i] + T;
        so[i + 1] = so[i] + (long long)PK_H * T * T;
        bo[i + 1] = bo[i] + (long long)PK_H * T * (2 * T - 1);
        po[i + 1] = po[i] + 2 * T - 1;
    }
    s->frames = fo[n_items];
    s->score_elems = so[n_items];
    s->bd_elems = bo[n_items];
    s->pos_rows = po[n_items];
    s->dev.n_items = n_items;
    s->dev.max_T = max_T;
    s->dev.uniform_T = uniform ? lengths[0] : 0;
    if (!uniform) {
        size_t bytes = 4 * n1 * sizeof(long long) + (size_t)n_items * sizeof(int);
        if (cudaMalloc(&s->dev_block, bytes) != cudaSuccess) {
            free(pre); free(s->lengths); free(s);
            cudaGetLastError();
            return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_seq_create: device allocation");
        }
        char *d = (char *)s->dev_block;
        if (cudaMemcpy(d, pre, 4 * n1 * sizeof(long long), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(d + 4 * n1 * sizeof(long long), lengths, (size_t)n_items * sizeof(int),
                       cudaMemcpyHostToDevice) != cudaSuccess) {
            cudaFree(s->dev_block); free(pre); free(s->lengths); free(s);
            return pkcu_fail(PKCU_ERR_CUDA, "pkcu_seq_create: upload failed");
        }
        const long long *dl = (const long long *)d;
        s->dev.frame_off = dl;
        s->dev.score_off = dl + n1;
        s->dev.bd_off = dl + 2 * n1;
        s->dev.pos_off = dl + 3 * n1;
        s->dev.T = (const int *)(d + 4 * n1 * sizeof(long long));
    }
    free(pre);
    *out = s;
    return PKCU_OK;
}

void pkcu_seq_destroy(pkcu_seq *s)
{
    if (!s) return;
    if (s->dev_block) {
        int cur = 0;
        cudaGetDevice(&cur);
        if (cur != s->device) cudaSetDevice(s->device);
        cudaFree(s->dev_block);
        if (cur != s->device) cudaSetDevice(cur);
    }
    free(s->lengths);
    free(s);
}

int pkcu_seq_n_items(const pkcu_seq *s) { return s ? s->dev.n_items : 0; }
long long pkcu_seq_frames(const pkcu_seq *s) { return s ? s->frames : 0; }
long long pkcu_seq_score_elems(const pkcu_seq *s) { return s ? s->score_elems : 0; }
long long pkcu_seq_bd_elems(const pkcu_seq *s) { return s ? s->bd_elems : 0; }
long long pkcu_seq_pos_rows(const pkcu_seq *s) { return s ? s->pos_rows : 0; }

/* ── drop-in host API ────────────────────────────────────────────────────────
 * One device workspace and one non-blocking stream per host thread and
 * device, grown on demand and released when the thread exits. */

typedef struct {
    int device;
    void *buf;
    size_t cap;
    cudaStream_t stream;
} DropinCtx;

static pthread_key_t g_ctx_key;
static pthread_once_t g_ctx_once = PTHREAD_ONCE_INIT;
static __thread int tls_status;

static void ctx_free(void *p)
{
    DropinCtx *c = (DropinCtx *)p;
    if (!c) return;
    if (c->buf) cudaFree(c->buf);
    if (c->stream) cudaStreamDestroy(c->stream);
    free(c);
}

static void ctx_key_init(void) { pthread_key_create(&g_ctx_key, ctx_free); }

int pk_cuda_status(void) { return tls_status; }

static void dropin_report(const char *what, int st)
{
    tls_status = st;
    if (st != PKCU_OK)
        fprintf(stderr, "[pk_tensor_ops_cuda] %s failed: %s (%s)\n", what, pkcu_status_string(st),
                pkcu_last_error());
}

/* Returns a device workspace of at least `bytes` on the current device. */
static DropinCtx *dropin_ctx(size_t bytes, int *st)
{
    pthread_once(&g_ctx_once, ctx_key_init);
    DropinCtx *c = (DropinCtx *)pthread_getspecific(g_ctx_key);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        *st = pkcu_fail(PKCU_ERR_CUDA, "no CUDA device");
        return NULL;
    }
    if (c && c->device != dev) {
        int cur = dev;
        cudaSetDevice(c->device);
        ctx_free(c);
        cudaSetDevice(cur);
        c = NULL;
        pthread_setspecific(g_ctx_key, NULL);
    }
    if (!c) {
        c = (DropinCtx *)calloc(1, sizeof(*c));
        if (!c) { *st = pkcu_fail(PKCU_ERR_NOMEM, "host allocation"); return NULL; }
        c->device = dev;
        if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            free(c);
            *st = pkcu_fail(PKCU_ERR_CUDA, "stream creation failed");
            return NULL;
        }
        pthread_setspecific(g_ctx_key, c);
    }
    if (c->cap < bytes) {
        if (c->buf) cudaFree(c->buf);
        c->buf = NULL;
        c->cap = 0;
        size_t want = bytes + bytes / 4;
        if (cudaMalloc(&c->buf, want) != cudaSuccess) {
            cudaGetLastError();
            *st = pkcu_fail(PKCU_ERR_NOMEM, "device workspace of %zu bytes", want);
            return NULL;
        }
        c->cap = want;
    }
    *st = PKCU_OK;
    return c;
}

static size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

static int h2d(void *d, const void *h, size_t bytes, cudaStream_t s)
{
    if (!bytes) return PKCU_OK;
    if (cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return pkcu_fail(PKCU_ERR_CUDA, "host to device copy: %s", cudaGetErrorString(cudaGetLastError()));
    return PKCU_OK;
}

static int d2h_sync(void *h, const void *d, size_t bytes, cudaStream_t s)
{
    if (bytes && cudaMemcpyAsync(h, d, bytes, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return pkcu_fail(PKCU_ERR_CUDA, "device to host copy: %s", cudaGetErrorString(cudaGetLastError()));
    if (cudaStreamSynchronize(s) != cudaSuccess)
        return pkcu_fail(PKCU_ERR_CUDA, "stream synchronize: %s", cudaGetErrorString(cudaGetLastError()));
    return pk_check_wait_timeouts("drop-in call");
}

/* Row LayerNorm of n_rows x D host floats: x (and out, possibly == x). */
static int dropin_ln(const float *x, const float *g, const float *b, float *out, int n_rows, int D)
{
    if (!x || !g || !b || !out) return pkcu_fail(PKCU_ERR_ARG, "NULL pointer");
    if (n_rows <= 0 || D <= 0) return PKCU_OK;
    size_t nx = (size_t)n_rows * D * sizeof(float), nd = (size_t)D * sizeof(float);
    int st;
    DropinCtx *c = dropin_ctx(al256(nx) + 2 * al256(nd), &st);
    if (!c) return st;
    char *base = (char *)c->buf;
    float *dx = (float *)base, *dg = (float *)(base + al256(nx)), *db = (float *)(base + al256(nx) + al256(nd));
    if ((st = h2d(dx, x, nx, c->stream)) || (st = h2d(dg, g, nd, c->stream)) ||
        (st = h2d(db, b, nd, c->stream)))
        return st;
    if ((st = pkcu_layer_norm_rows(dx, dg, db, dx, n_rows, D, c->stream))) return st;
    return d2h_sync(out, dx, nx, c->stream);
}

void pk_layer_norm(const float *x, const float *gamma, const float *beta_, float *out, int len)
{
    dropin_report("pk_layer_norm", dropin_ln(x, gamma, beta_, out, 1, len));
}

void pk_layer_norm_rows(const float *x, const float *gamma, const float *beta_, float *out,
                        int n_rows, int D)
{
    dropin_report("pk_layer_norm_rows", dropin_ln(x, gamma, beta_, out, n_rows, D));
}

void pk_layer_norm_rows_inplace(float *x, const float *gamma, const float *beta_, int n_rows, int D)
{
    dropin_report("pk_layer_norm_rows_inplace", dropin_ln(x, gamma, beta_, x, n_rows, D));
}

enum { FLAT_SWISH, FLAT_RELU };

static int dropin_flat(float *x, long long n, int op)
{
    if (!x) return pkcu_fail(PKCU_ERR_ARG, "NULL pointer");
    if (n <= 0) return PKCU_OK;
    size_t nb = (size_t)n * sizeof(float);
    int st;
    DropinCtx *c = dropin_ctx(nb, &st);
    if (!c) return st;
    float *dx = (float *)c->buf;
    if ((st = h2d(dx, x, nb, c->stream))) return st;
    st = op == FLAT_SWISH ? pkcu_swish(dx, n, c->stream) : pkcu_relu(dx, n, c->stream);
    if (st) return st;
    return d2h_sync(x, dx, nb, c->stream);
}

void pk_swish(float *x, int len) { dropin_report("pk_swish", dropin_flat(x, len, FLAT_SWISH)); }
void pk_relu(float *x, int len) { dropin_report("pk_relu", dropin_flat(x, len, FLAT_RELU)); }

static int dropin_softmax(float *x, int n_rows, int len)
{
    if (!x) return pkcu_fail(PKCU_ERR_ARG, "NULL pointer");
    if (n_rows <= 0 || len <= 0) return PKCU_OK;
    size_t nb = (size_t)n_rows * len * sizeof(float);
    int st;
    DropinCtx *c = dropin_ctx(nb, &st);
    if (!c) return st;
    float *dx = (float *)c->buf;
    if ((st = h2d(dx, x, nb, c->stream))) return st;
    if ((st = pkcu_softmax_rows(dx, n_rows, len, c->stream))) return st;
    return d2h_sync(x, dx, nb, c->stream);
}

void pk_softmax(float *x, int len) { dropin_report("pk_softmax", dropin_softmax(x, 1, len)); }
void pk_softmax_rows(float *x, int n_rows, int len)
{
    dropin_report("pk_softmax_rows", dropin_softmax(x, n_rows, len));
}

static int dropin_bias(float *x, const float *b, int len)
{
    if (!x || !b) return pkcu_fail(PKCU_ERR_ARG, "NULL pointer");
    if (len <= 0) return PKCU_OK;
    size_t nb = (size_t)len * sizeof(float);
    int st;
    DropinCtx *c = dropin_ctx(2 * al256(nb), &st);
    if (!c) return st;
    float *dx = (float *)c->buf, *dbias = (float *)((char *)c->buf + al256(nb));
    if ((st = h2d(dx, x, nb, c->stream)) || (st = h2d(dbias, b, nb, c->stream))) return st;
    if ((st = pkcu_bias_add_rows(dx, dbias, 1, len, c->stream))) return st;
    return d2h_sync(x, dx, nb, c->stream);
}

void pk_bias_add(float *x, const float *b, int len) { dropin_report("pk_bias_add", dropin_bias(x, b, len)); }

static int dropin_dwconv(const float *x, const float *w, const float *b, float *out, int C, int T, int K)
{
    if (!x || !w || !out) return pkcu_fail(PKCU_ERR_ARG, "NULL pointer");
    if (K <= 0 || K > PK_DW_MAX_K)
        return pkcu_fail(PKCU_ERR_ARG, "pk_depthwise_conv1d: K must be 1..%d", PK_DW_MAX_K);
    if (C <= 0 || T <= 0) return PKCU_OK;
    size_t nx = (size_t)C * T * sizeof(float), nw = (size_t)C * K * sizeof(float),
           nbias = (size_t)C * sizeof(float);
    int st;
    DropinCtx *c = dropin_ctx(2 * al256(nx) + al256(nw) + al256(nbias), &st);
    if (!c) return st;
    char *base = (char *)c->buf;
    float *dx = (float *)base, *dout = (float *)(base + al256(nx)),
          *dw = (float *)(base + 2 * al256(nx)), *dbias = (float *)(base + 2 * al256(nx) + al256(nw));
    if ((st = h2d(dx, x, nx, c->stream)) || (st = h2d(dw, w, nw, c->stream))) return st;
    if (b && (st = h2d(dbias, b, nbias, c->stream))) return st;
    if ((st = pkcu_depthwise_conv1d(dx, dw, b ? dbias : NULL, dout, C, T, K, c->stream))) return st;
    return d2h_sync(out, dout, nx, c->stream);
}

void pk_depthwise_conv1d(const float *x, const float *w, const float *b, float *out, int C, int T,
                         int K)
{
    dropin_report("pk_depthwise_conv1d", dropin_dwconv(x, w, b, out, C, T, K));
}

/* ── sequence driver ─────────────────────────────────────────────────────── */

/* The first block's LN_ff1, then per block: bias+Swish (FF1), residual+LN,
 * QKV split, positional split, scores, head concat, residual+LN+transpose,
 * GLU+conv, transpose-add+LN, bias+Swish (FF2), residual+LN+LN. */
int pkcu_encoder_nongemm_launches(int n_blocks) { return n_blocks > 0 ? 1 + 11 * n_blocks : 0; }

#define PK_TRY(call) do { int st_ = (call); if (st_) return st_; } while (0)
#define PK_HOOK(blk, g) do { if (hook) PK_TRY(hook(hook_user, (blk), (g), stream)); } while (0)

int pkcu_encoder_nongemm(float *x, const pkcu_block_params *blocks, int n_blocks,
                         const pkcu_gemm_outputs *go, const pkcu_gemm_inputs *gi,
                         const pkcu_seq *seq, pkcu_gemm_hook hook, void *hook_user,
                         pkcu_stream_t stream)
{
    return pkcu_encoder_nongemm_fused(x, blocks, n_blocks, go, gi, seq, hook, hook_user, 0u, stream);
}

int pkcu_encoder_nongemm_fused(float *x, const pkcu_block_params *blocks, int n_blocks,
                               const pkcu_gemm_outputs *go, const pkcu_gemm_inputs *gi,
                               const pkcu_seq *seq, pkcu_gemm_hook hook, void *hook_user,
                               unsigned fused, pkcu_stream_t stream)
{
    if (!x || !blocks || n_blocks < 0 || !go || !gi || !seq)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_nongemm: NULL argument");
    if (fused & ~(unsigned)(PKCU_FUSED_FF_SWISH | PKCU_FUSED_QKV | PKCU_FUSED_CONV))
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_nongemm: unknown fusion flags 0x%x", fused);
    if (fused && !hook)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_nongemm: fusion flags without a GEMM hook");
    if (n_blocks == 0 || seq->frames == 0) return PKCU_OK;
    if (seq->frames > 0x7fffffffLL / PK_FF)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_nongemm: too many frames in one call");
    const int F = (int)seq->frames;
    /* 1/sqrt(d_k) of csrc/encoder.c:384. */
    const float scale = 1.0f / sqrtf((float)PK_DH);

    PK_TRY(pkcu_layer_norm_rows(x, blocks[0].norm_ff1_w, blocks[0].norm_ff1_b, gi->ln_ff1, F, PK_D,
                                stream));
    for (int b = 0; b < n_blocks; b++) {
        const pkcu_block_params *p = &blocks[b];
        const pkcu_block_params *nx = (b + 1 < n_blocks) ? &blocks[b + 1] : NULL;
        /* FF1 (csrc/encoder.c:179-217) */
        PK_HOOK(b, PKCU_GEMM_FF1_1);
        if (!(fused & PKCU_FUSED_FF_SWISH))
            PK_TRY(pkcu_bias_swish_rows(go->ff1_h, p->ff1_b1, gi->h1, F, PK_FF, stream));
        PK_HOOK(b, PKCU_GEMM_FF1_2);
        PK_TRY(pkcu_residual_layer_norm(x, go->ff1_out, p->ff1_b2, 0.5f, p->norm_sa_w, p->norm_sa_b,
                                        gi->ln_sa, F, stream));
        /* self-attention (csrc/encoder.c:297-435) */
        PK_HOOK(b, PKCU_GEMM_QKV);
        if (!(fused & PKCU_FUSED_QKV))
            PK_TRY(pkcu_qkv_split_uv(go->qkv, p->qkv_b, p->pos_u, p->pos_v, gi->Qu, gi->Qv, gi->K,
                                     gi->V, seq, stream));
        PK_HOOK(b, PKCU_GEMM_POS);
        PK_TRY(pkcu_pos_head_split(go->P, gi->P_h, seq, stream));
        PK_HOOK(b, PKCU_GEMM_AC);
        PK_HOOK(b, PKCU_GEMM_BD);
        PK_TRY(pkcu_relpos_combine_softmax(go->ac, go->bd, gi->S, scale, seq, stream));
        PK_HOOK(b, PKCU_GEMM_AV);
        PK_TRY(pkcu_head_concat(go->attn_h, gi->attn, seq, stream));
        PK_HOOK(b, PKCU_GEMM_OUT);
        if (fused & PKCU_FUSED_CONV) {
            /* conv module with its GEMM epilogues in the hook: LN_conv time-first
             * into cf, the PW1 hook writes the GLU output, the PW2 hook adds
             * pw2 + bias to x */
            PK_TRY(pkcu_residual_layer_norm(x, go->att_out, p->out_b, 1.0f, p->norm_conv_w,
                                            p->norm_conv_b, gi->cf, F, stream));
            PK_HOOK(b, PKCU_GEMM_PW1);
            PK_TRY(pkcu_dwconv_bn_swish(gi->gated, p->dw_w, p->dw_b, NULL, 0.0f, 1, gi->dw, PK_D, 9,
                                        seq, stream));
            PK_HOOK(b, PKCU_GEMM_PW2);
            PK_TRY(pkcu_layer_norm_rows(x, p->norm_ff2_w, p->norm_ff2_b, gi->ln_ff2, F, PK_D, stream));
        } else {
            PK_TRY(pkcu_residual_layer_norm_transpose(x, go->att_out, p->out_b, 1.0f, p->norm_conv_w,
                                                      p->norm_conv_b, gi->cf, seq, stream));
            /* conv module (csrc/encoder.c:439-478) */
            PK_HOOK(b, PKCU_GEMM_PW1);
            PK_TRY(pkcu_glu_dwconv_bn_swish(go->pw1, p->pw1_b, p->dw_w, p->dw_b, NULL, 0.0f, 1, gi->dw,
                                            PK_D, 9, seq, stream));
            PK_HOOK(b, PKCU_GEMM_PW2);
            PK_TRY(pkcu_transpose_add_layer_norm(x, go->pw2, p->pw2_b, p->norm_ff2_w, p->norm_ff2_b,
                                                 gi->ln_ff2, seq, stream));
        }
        /* FF2 and the block's final LN (csrc/encoder.c:489-490) */
        PK_HOOK(b, PKCU_GEMM_FF2_1);
        if (!(fused & PKCU_FUSED_FF_SWISH))
            PK_TRY(pkcu_bias_swish_rows(go->ff2_h, p->ff2_b1, gi->h2, F, PK_FF, stream));
        PK_HOOK(b, PKCU_GEMM_FF2_2);
        PK_TRY(pkcu_residual_layer_norm2(x, go->ff2_out, p->ff2_b2, 0.5f, p->norm_out_w,
                                         p->norm_out_b, nx ? nx->norm_ff1_w : NULL,
                                         nx ? nx->norm_ff1_b : NULL, nx ? gi->ln_ff1 : NULL, F,
                                         stream));
    }
    return PKCU_OK;
}
