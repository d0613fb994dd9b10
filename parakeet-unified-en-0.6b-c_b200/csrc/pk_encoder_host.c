/* pk_encoder_host.c -- host-buffer form of the per-block non-GEMM sequence.
 *
 * The reference's encoder takes host buffers and returns host buffers
 * (pk_encoder, csrc/encoder.c:612-633). pkcu_encoder_nongemm_host does the
 * same for the non-GEMM sequence: the caller keeps x and the GEMM outputs in
 * host memory; a workspace (created once per batch shape) owns the device
 * copies. The batch is split into groups of items and pipelined over three
 * streams: the host-to-device copy of group g+1 and the device-to-host copy of
 * group g-1 run on the copy engines while group g computes. Host buffers
 * should be page-locked (cudaMallocHost / cudaHostRegister); pageable memory
 * works but serialises the copies. */
#include <cuda_runtime_api.h>
#include <stdlib.h>
#include <string.h>

#include "pkcuda_internal.h"

#define N_OUT 12   /* pkcu_gemm_outputs fields */
#define N_IN 15    /* pkcu_gemm_inputs fields  */

/* How a tensor's per-item block scales: elements per frame, per (2T-1) pos
 * row, per score element or per bd element. */
enum { U_FRAME, U_POS, U_SCORE, U_BD };
typedef struct { int unit; long long per; } Extent;

static const Extent OUT_EXT[N_OUT] = {
    {U_FRAME, PK_FF}, {U_FRAME, PK_D}, {U_FRAME, 3 * PK_D}, {U_POS, PK_D}, {U_SCORE, 1},
    {U_BD, 1}, {U_FRAME, PK_D}, {U_FRAME, PK_D}, {U_FRAME, 2 * PK_D}, {U_FRAME, PK_D},
    {U_FRAME, PK_FF}, {U_FRAME, PK_D}};
static const Extent IN_EXT[N_IN] = {
    {U_FRAME, PK_D}, {U_FRAME, PK_FF}, {U_FRAME, PK_D}, {U_FRAME, PK_D}, {U_FRAME, PK_D},
    {U_FRAME, PK_D}, {U_POS, PK_D}, {U_SCORE, 1}, {U_FRAME, PK_D}, {U_FRAME, PK_D},
    {U_FRAME, PK_D}, {U_FRAME, PK_D}, {U_FRAME, PK_D}, {U_FRAME, PK_FF}, {U_FRAME, PK_D}};

struct pkcu_encoder_ws {
    int device;
    int n_groups;
    pkcu_seq **groups;
    long long (*start)[4];      /* per group: first frame, pos row, score, bd element */
    long long total[4];
    void *block;                /* one device allocation for every buffer */
    float *x;
    float *out[N_OUT];
    float *in[N_IN];
    cudaStream_t s_h2d, s_d2h;
    cudaEvent_t *ev_h2d, *ev_comp;
};

static long long ext_elems(Extent e, const long long n[4]) { return e.per * n[e.unit]; }

void pkcu_encoder_ws_destroy(pkcu_encoder_ws *ws)
{
    if (!ws) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(ws->device);
    for (int g = 0; g < ws->n_groups; g++) {
        if (ws->groups && ws->groups[g]) pkcu_seq_destroy(ws->groups[g]);
        if (ws->ev_h2d && ws->ev_h2d[g]) cudaEventDestroy(ws->ev_h2d[g]);
        if (ws->ev_comp && ws->ev_comp[g]) cudaEventDestroy(ws->ev_comp[g]);
    }
    if (ws->s_h2d) cudaStreamDestroy(ws->s_h2d);
    if (ws->s_d2h) cudaStreamDestroy(ws->s_d2h);
    if (ws->block) cudaFree(ws->block);
    free(ws->groups);
    free(ws->start);
    free(ws->ev_h2d);
    free(ws->ev_comp);
    free(ws);
    cudaSetDevice(cur);
}

int pkcu_encoder_ws_create(const pkcu_seq *seq, int n_groups, pkcu_encoder_ws **out)
{
    if (!out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_ws_create: NULL out");
    *out = NULL;
    if (!seq || n_groups <= 0) return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_ws_create: bad argument");
    const int n_items = seq->dev.n_items;
    if (n_groups > n_items) n_groups = n_items;
    pkcu_encoder_ws *ws = (pkcu_encoder_ws *)calloc(1, sizeof(*ws));
    if (!ws) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_encoder_ws_create: host allocation");
    cudaGetDevice(&ws->device);
    ws->n_groups = n_groups;
    ws->groups = (pkcu_seq **)calloc((size_t)n_groups, sizeof(pkcu_seq *));
    ws->start = (long long (*)[4])calloc((size_t)n_groups, sizeof(*ws->start));
    ws->ev_h2d = (cudaEvent_t *)calloc((size_t)n_groups, sizeof(cudaEvent_t));
    ws->ev_comp = (cudaEvent_t *)calloc((size_t)n_groups, sizeof(cudaEvent_t));
    if (!ws->groups || !ws->start || !ws->ev_h2d || !ws->ev_comp) {
        pkcu_encoder_ws_destroy(ws);
        return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_encoder_ws_create: host allocation");
    }
    /* Contiguous groups of items and where each starts in every layout. */
    long long acc[4] = {0, 0, 0, 0};
    int item = 0;
    for (int g = 0; g < n_groups; g++) {
        int i1 = (int)(((long long)n_items * (g + 1)) / n_groups);
        memcpy(ws->start[g], acc, sizeof(acc));
        int st = pkcu_seq_create(seq->lengths + item, i1 - item, &ws->groups[g]);
        if (st) { pkcu_encoder_ws_destroy(ws); return st; }
        for (int i = item; i < i1; i++) {
            long long T = seq->lengths[i];
            acc[U_FRAME] += T;
            acc[U_POS] += 2 * T - 1;
            acc[U_SCORE] += (long long)PK_H * T * T;
            acc[U_BD] += (long long)PK_H * T * (2 * T - 1);
        }
        item = i1;
    }
    memcpy(ws->total, acc, sizeof(acc));
    /* One allocation, every buffer 256-byte aligned. */
    size_t bytes = 0, off_x, off_out[N_OUT], off_in[N_IN];
#define PK_TAKE(off, n) do { (off) = bytes; bytes += (((size_t)(n) * sizeof(float)) + 255) & ~(size_t)255; } while (0)
    PK_TAKE(off_x, acc[U_FRAME] * PK_D);
    for (int r = 0; r < N_OUT; r++) PK_TAKE(off_out[r], ext_elems(OUT_EXT[r], acc));
    for (int r = 0; r < N_IN; r++) PK_TAKE(off_in[r], ext_elems(IN_EXT[r], acc));
#undef PK_TAKE
    if (cudaMalloc(&ws->block, bytes) != cudaSuccess) {
        cudaGetLastError();
        pkcu_encoder_ws_destroy(ws);
        return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_encoder_ws_create: %zu device bytes", bytes);
    }
    char *base = (char *)ws->block;
    ws->x = (float *)(base + off_x);
    for (int r = 0; r < N_OUT; r++) ws->out[r] = (float *)(base + off_out[r]);
    for (int r = 0; r < N_IN; r++) ws->in[r] = (float *)(base + off_in[r]);
    if (cudaStreamCreateWithFlags(&ws->s_h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ws->s_d2h, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        pkcu_encoder_ws_destroy(ws);
        return pkcu_fail(PKCU_ERR_CUDA, "pkcu_encoder_ws_create: stream creation");
    }
    for (int g = 0; g < n_groups; g++)
        if (cudaEventCreateWithFlags(&ws->ev_h2d[g], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ws->ev_comp[g], cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            pkcu_encoder_ws_destroy(ws);
            return pkcu_fail(PKCU_ERR_CUDA, "pkcu_encoder_ws_create: event creation");
        }
    *out = ws;
    return PKCU_OK;
}

/* Device views of the whole batch (for callers that keep data resident). */
int pkcu_encoder_ws_device(pkcu_encoder_ws *ws, float **x, pkcu_gemm_outputs *gemm_out,
                           pkcu_gemm_inputs *gemm_in)
{
    if (!ws) return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_ws_device: NULL ws");
    if (x) *x = ws->x;
    if (gemm_out) {
        const float **o = (const float **)gemm_out;
        for (int r = 0; r < N_OUT; r++) o[r] = ws->out[r];
    }
    if (gemm_in) {
        float **o = (float **)gemm_in;
        for (int r = 0; r < N_IN; r++) o[r] = ws->in[r];
    }
    return PKCU_OK;
}

long long pkcu_encoder_ws_device_bytes(const pkcu_encoder_ws *ws)
{
    if (!ws) return 0;
    long long b = ws->total[U_FRAME] * PK_D;
    for (int r = 0; r < N_OUT; r++) b += ext_elems(OUT_EXT[r], ws->total);
    for (int r = 0; r < N_IN; r++) b += ext_elems(IN_EXT[r], ws->total);
    return b * (long long)sizeof(float);
}

/* Bytes one pkcu_encoder_nongemm_host call moves host->device (x and the
 * twelve GEMM outputs) and device->host (x). */
long long pkcu_encoder_ws_h2d_bytes(const pkcu_encoder_ws *ws)
{
    if (!ws) return 0;
    long long b = ws->total[U_FRAME] * PK_D;
    for (int r = 0; r < N_OUT; r++) b += ext_elems(OUT_EXT[r], ws->total);
    return b * (long long)sizeof(float);
}

long long pkcu_encoder_ws_d2h_bytes(const pkcu_encoder_ws *ws)
{
    return ws ? ws->total[U_FRAME] * PK_D * (long long)sizeof(float) : 0;
}

static int copy(void *dst, const void *src, long long elems, enum cudaMemcpyKind kind, cudaStream_t s)
{
    if (elems <= 0) return PKCU_OK;
    cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)elems * sizeof(float), kind, s);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return pkcu_fail(PKCU_ERR_CUDA, "pkcu_encoder_nongemm_host: copy failed: %s", cudaGetErrorString(e));
    }
    return PKCU_OK;
}

int pkcu_encoder_nongemm_host(pkcu_encoder_ws *ws, float *x_host, const pkcu_gemm_outputs *gemm_out_host,
                              const pkcu_block_params *blocks, int n_blocks, pkcu_stream_t stream)
{
    if (!ws || !x_host || !gemm_out_host || !blocks || n_blocks < 0)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_nongemm_host: NULL argument");
    const float *const *host_out = (const float *const *)gemm_out_host;
    for (int r = 0; r < N_OUT; r++)
        if (!host_out[r]) return pkcu_fail(PKCU_ERR_ARG, "pkcu_encoder_nongemm_host: GEMM output %d is NULL", r);
    cudaStream_t cs = (cudaStream_t)stream;
    int st = PKCU_OK;
    for (int g = 0; g < ws->n_groups && !st; g++) {
        const long long *s0 = ws->start[g];
        const pkcu_seq *gs = ws->groups[g];
        const long long n[4] = {gs->frames, gs->pos_rows, gs->score_elems, gs->bd_elems};
        /* host -> device: x and the GEMM outputs of this group */
        st = copy(ws->x + s0[U_FRAME] * PK_D, x_host + s0[U_FRAME] * PK_D, n[U_FRAME] * PK_D,
                  cudaMemcpyHostToDevice, ws->s_h2d);
        pkcu_gemm_outputs go;
        pkcu_gemm_inputs gi;
        const float **gop = (const float **)&go;
        float **gip = (float **)&gi;
        for (int r = 0; r < N_OUT && !st; r++) {
            long long o = OUT_EXT[r].per * s0[OUT_EXT[r].unit];
            st = copy(ws->out[r] + o, host_out[r] + o, ext_elems(OUT_EXT[r], n), cudaMemcpyHostToDevice,
                      ws->s_h2d);
            gop[r] = ws->out[r] + o;
        }
        for (int r = 0; r < N_IN; r++) gip[r] = ws->in[r] + IN_EXT[r].per * s0[IN_EXT[r].unit];
        if (st) break;
        if (cudaEventRecord(ws->ev_h2d[g], ws->s_h2d) != cudaSuccess ||
            cudaStreamWaitEvent(cs, ws->ev_h2d[g], 0) != cudaSuccess) {
            st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_encoder_nongemm_host: event");
            break;
        }
        /* compute */
        st = pkcu_encoder_nongemm(ws->x + s0[U_FRAME] * PK_D, blocks, n_blocks, &go, &gi, gs, NULL, NULL,
                                  stream);
        if (st) break;
        /* device -> host: x */
        if (cudaEventRecord(ws->ev_comp[g], cs) != cudaSuccess ||
            cudaStreamWaitEvent(ws->s_d2h, ws->ev_comp[g], 0) != cudaSuccess) {
            st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_encoder_nongemm_host: event");
            break;
        }
        st = copy(x_host + s0[U_FRAME] * PK_D, ws->x + s0[U_FRAME] * PK_D, n[U_FRAME] * PK_D,
                  cudaMemcpyDeviceToHost, ws->s_d2h);
    }
    /* Synchronous like the reference's encoder: wait for every stream, also on error. */
    cudaError_t e1 = cudaStreamSynchronize(ws->s_h2d);
    cudaError_t e2 = cudaStreamSynchronize(cs);
    cudaError_t e3 = cudaStreamSynchronize(ws->s_d2h);
    if (!st && (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess))
        st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_encoder_nongemm_host: %s",
                       cudaGetErrorString(e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e3)));
    if (!st) st = pk_check_wait_timeouts("pkcu_encoder_nongemm_host");
    return st;
}
