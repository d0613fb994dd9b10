/* pk_weights.c -- on-device loader for the reference's weights.bin / weights.json
 * checkpoint format (csrc/weights.c:102-402; format written by
 * extract_weights.py:894-945).
 *
 * Format: weights.bin holds every tensor's bytes back to back in name order;
 * weights.json maps each name to {offset, shape, numel, dtype} with dtype
 * "float32", "int8" (plus a per-tensor "scale") or "int4" (packed [K, N/2]
 * bytes, low nibble = even column, followed in the file by K*N/32 fp32 group
 * scales at "scales_offset", "n_scales" of them).
 *
 * Two steps. pkcu_weights_open() is host-only: it parses the manifest and
 * reads the file. pkcu_weights_upload() copies every tensor into its own
 * 256-byte aligned slot of one device allocation (file offsets are not
 * 16-byte aligned in general: a 1025-float bias shifts every later tensor)
 * and then builds, per conformer block, the fused [D, 3D] QKV weight and the
 * [3D] bias the reference builds after loading (csrc/weights.c:403-544):
 *   - q, k, v int8: requantised to the common scale max(sq, sk, sv)
 *     (pkcu_requant_qkv_i8), int8 result;
 *   - q, k, v float32: columns interleaved, fp32 result;
 *   - q, k, v int4: dequantised and interleaved, fp32 result. This is the
 *     reference's int4 branch (:488-544); in the reference itself it is never
 *     reached, because int4 entries carry scale 0 and the float32 test
 *     (:414) catches them first, so this follows the branch's code, not the
 *     reference's behaviour on an int4 checkpoint.
 *
 * The int8 scale is converted from the manifest's decimal text the way the
 * reference's parser does it (:63-94): digits accumulated in a double, the
 * fraction's digits as an integer divided by 10^digits, the exponent applied as
 * a product of tens, then narrowed to float. The double can be off in its last
 * bits for long digit strings; keeping the same steps makes the float equal to
 * the reference's by construction rather than only where the narrowing hides
 * that error. */
#include <cuda_runtime_api.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pkcuda_internal.h"

typedef struct {
    char *name;
    int dtype;                  /* PKCU_DTYPE_* */
    int ndim;
    long long shape[4];
    long long numel;            /* elements (float32, int8) or packed bytes (int4) */
    long long offset;           /* byte offset in weights.bin */
    float scale;                /* int8 */
    long long scales_offset;    /* int4 */
    long long n_scales;         /* int4 */
    long long slot, scales_slot;   /* byte offsets in the device arena, -1 if none */
} Entry;

typedef struct {
    int ok;                     /* fused weight built */
    int bits;                   /* 8 or 32 */
    float scale;                /* int8: the common scale */
    long long w_slot, b_slot;   /* arena byte offsets */
} Fused;

struct pkcu_weights {
    Entry *e;
    int n;
    unsigned char *bin;         /* host copy of weights.bin */
    long long bin_bytes;
    int registered;             /* bin is page-locked by cudaHostRegister */
    int device;
    unsigned char *arena;       /* device allocation, NULL before upload */
    long long arena_bytes;
    int n_blocks;               /* blocks with q, k, v entries */
    Fused *fused;
};

/* ── manifest scanner ─────────────────────────────────────────────────────── */

typedef struct {
    const char *s;
    long long i, n;
    int bad;
} Scan;

static void ws(Scan *p)
{
    while (p->i < p->n && (p->s[p->i] == ' ' || p->s[p->i] == '\n' || p->s[p->i] == '\r' ||
                           p->s[p->i] == '\t'))
        p->i++;
}

static int peek(Scan *p)
{
    ws(p);
    return p->i < p->n ? (unsigned char)p->s[p->i] : -1;
}

static int expect(Scan *p, char c)
{
    if (peek(p) != c) { p->bad = 1; return 0; }
    p->i++;
    return 1;
}

/* A string without escapes (manifest names and keys have none); returns a
 * pointer into the text and its length. */
static int string(Scan *p, const char **at, long long *len)
{
    if (!expect(p, '"')) return 0;
    const long long b = p->i;
    while (p->i < p->n && p->s[p->i] != '"') {
        if (p->s[p->i] == '\\') { p->bad = 1; return 0; }
        p->i++;
    }
    if (p->i >= p->n) { p->bad = 1; return 0; }
    *at = p->s + b;
    *len = p->i - b;
    p->i++;
    return 1;
}

static int integer(Scan *p, long long *v)
{
    ws(p);
    int neg = 0;
    if (p->i < p->n && p->s[p->i] == '-') { neg = 1; p->i++; }
    if (p->i >= p->n || p->s[p->i] < '0' || p->s[p->i] > '9') { p->bad = 1; return 0; }
    long long x = 0;
    while (p->i < p->n && p->s[p->i] >= '0' && p->s[p->i] <= '9') x = x * 10 + (p->s[p->i++] - '0');
    *v = neg ? -x : x;
    return 1;
}

/* The reference's decimal conversion (csrc/weights.c:63-94), step for step. */
static int decimal(Scan *p, double *v)
{
    ws(p);
    int neg = 0;
    if (p->i < p->n && p->s[p->i] == '-') { neg = 1; p->i++; }
    double x = 0.0;
    while (p->i < p->n && p->s[p->i] >= '0' && p->s[p->i] <= '9') x = x * 10 + (p->s[p->i++] - '0');
    if (p->i < p->n && p->s[p->i] == '.') {
        p->i++;
        double frac = 0.0, div = 1.0;
        while (p->i < p->n && p->s[p->i] >= '0' && p->s[p->i] <= '9') {
            frac = frac * 10 + (p->s[p->i++] - '0');
            div *= 10.0;
        }
        x += frac / div;
    }
    if (p->i < p->n && (p->s[p->i] == 'e' || p->s[p->i] == 'E')) {
        p->i++;
        int eneg = 0, e = 0;
        if (p->i < p->n && p->s[p->i] == '-') { eneg = 1; p->i++; }
        else if (p->i < p->n && p->s[p->i] == '+') p->i++;
        while (p->i < p->n && p->s[p->i] >= '0' && p->s[p->i] <= '9') e = e * 10 + (p->s[p->i++] - '0');
        double mul = 1.0;
        for (int k = 0; k < e; k++) mul *= 10.0;
        x = eneg ? x / mul : x * mul;
    }
    *v = neg ? -x : x;
    return 1;
}

/* Skips any JSON value. */
static void skip_value(Scan *p, int depth)
{
    const int c = peek(p);
    if (depth > 64) { p->bad = 1; return; }
    if (c == '"') {
        const char *a; long long l;
        string(p, &a, &l);
    } else if (c == '{' || c == '[') {
        const char close = c == '{' ? '}' : ']';
        p->i++;
        if (peek(p) == close) { p->i++; return; }
        while (!p->bad) {
            if (c == '{') {
                const char *a; long long l;
                if (!string(p, &a, &l) || !expect(p, ':')) return;
            }
            skip_value(p, depth + 1);
            if (peek(p) == ',') { p->i++; continue; }
            expect(p, close);
            return;
        }
    } else {
        while (p->i < p->n && p->s[p->i] != ',' && p->s[p->i] != '}' && p->s[p->i] != ']' &&
               p->s[p->i] != ' ' && p->s[p->i] != '\n' && p->s[p->i] != '\r' && p->s[p->i] != '\t')
            p->i++;
    }
}

static int key_is(const char *a, long long l, const char *k)
{
    return (long long)strlen(k) == l && memcmp(a, k, (size_t)l) == 0;
}

static int parse_entry(Scan *p, Entry *e)
{
    e->dtype = PKCU_DTYPE_F32;
    e->ndim = 0;
    e->numel = -1;
    e->offset = -1;
    e->scale = 0.0f;
    e->scales_offset = -1;
    e->n_scales = 0;
    if (!expect(p, '{')) return 0;
    if (peek(p) == '}') { p->i++; return 1; }
    while (!p->bad) {
        const char *k; long long kl;
        if (!string(p, &k, &kl) || !expect(p, ':')) return 0;
        if (key_is(k, kl, "offset")) {
            integer(p, &e->offset);
        } else if (key_is(k, kl, "numel")) {
            integer(p, &e->numel);
        } else if (key_is(k, kl, "scales_offset")) {
            integer(p, &e->scales_offset);
        } else if (key_is(k, kl, "n_scales")) {
            integer(p, &e->n_scales);
        } else if (key_is(k, kl, "scale")) {
            double v;
            decimal(p, &v);
            e->scale = (float)v;
        } else if (key_is(k, kl, "dtype")) {
            const char *v; long long vl;
            if (!string(p, &v, &vl)) return 0;
            if (key_is(v, vl, "int8")) e->dtype = PKCU_DTYPE_I8;
            else if (key_is(v, vl, "int4")) e->dtype = PKCU_DTYPE_I4;
            else if (key_is(v, vl, "float32")) e->dtype = PKCU_DTYPE_F32;
            else { p->bad = 1; return 0; }
        } else if (key_is(k, kl, "shape")) {
            if (!expect(p, '[')) return 0;
            if (peek(p) == ']') { p->i++; }
            else {
                while (!p->bad) {
                    long long d;
                    if (!integer(p, &d)) return 0;
                    if (e->ndim < 4) e->shape[e->ndim] = d;
                    e->ndim++;
                    if (peek(p) == ',') { p->i++; continue; }
                    if (!expect(p, ']')) return 0;
                    break;
                }
            }
        } else {
            skip_value(p, 0);
        }
        if (peek(p) == ',') { p->i++; continue; }
        return expect(p, '}');
    }
    return 0;
}

static long long elem_bytes(const Entry *e)
{
    return e->dtype == PKCU_DTYPE_F32 ? 4 * e->numel : e->numel;   /* int8: 1 B; int4: packed */
}

/* ── open / close ─────────────────────────────────────────────────────────── */

void pkcu_weights_destroy(pkcu_weights *w)
{
    if (!w) return;
    if (w->arena) {
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(w->device);
        cudaFree(w->arena);
        cudaSetDevice(cur);
    }
    if (w->registered) cudaHostUnregister(w->bin);
    for (int i = 0; i < w->n; i++) free(w->e[i].name);
    free(w->e);
    free(w->fused);
    free(w->bin);
    free(w);
}

static unsigned char *read_file(const char *path, long long *bytes)
{
    FILE *f = fopen(path, "rb");
    if (!f) return NULL;
    if (fseek(f, 0, SEEK_END) != 0) { fclose(f); return NULL; }
    const long long n = ftell(f);
    if (n < 0 || fseek(f, 0, SEEK_SET) != 0) { fclose(f); return NULL; }
    unsigned char *buf = (unsigned char *)malloc((size_t)n + 1);
    if (!buf) { fclose(f); return NULL; }
    const size_t got = n ? fread(buf, 1, (size_t)n, f) : 0;
    fclose(f);
    if ((long long)got != n) { free(buf); return NULL; }
    buf[n] = 0;
    *bytes = n;
    return buf;
}

int pkcu_weights_open(const char *bin_path, const char *json_path, pkcu_weights **out)
{
    if (!bin_path || !json_path || !out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_open: NULL argument");
    *out = NULL;
    long long jn = 0;
    unsigned char *json = read_file(json_path, &jn);
    if (!json) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_open: cannot read %s", json_path);
    pkcu_weights *w = (pkcu_weights *)calloc(1, sizeof(*w));
    if (!w) { free(json); return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_weights_open: host allocation"); }
    Scan p = {(const char *)json, 0, jn, 0};
    int cap = 0;
    int st = PKCU_OK;
    if (!expect(&p, '{')) st = PKCU_ERR_ARG;
    if (!st && peek(&p) != '}') {
        while (!p.bad) {
            const char *nm; long long nl;
            if (!string(&p, &nm, &nl) || !expect(&p, ':')) break;
            if (w->n == cap) {
                cap = cap ? 2 * cap : 1024;
                Entry *ne = (Entry *)realloc(w->e, (size_t)cap * sizeof(Entry));
                if (!ne) { st = PKCU_ERR_NOMEM; break; }
                w->e = ne;
            }
            Entry *e = &w->e[w->n];
            memset(e, 0, sizeof(*e));
            e->name = (char *)malloc((size_t)nl + 1);
            if (!e->name) { st = PKCU_ERR_NOMEM; break; }
            memcpy(e->name, nm, (size_t)nl);
            e->name[nl] = 0;
            w->n++;
            if (!parse_entry(&p, e)) break;
            if (peek(&p) == ',') { p.i++; continue; }
            expect(&p, '}');
            break;
        }
    }
    free(json);
    if (!st && p.bad) st = PKCU_ERR_ARG;
    if (st) {
        pkcu_weights_destroy(w);
        return pkcu_fail(st, "pkcu_weights_open: %s is not a weights manifest (near byte %lld)",
                         json_path, p.i);
    }
    w->bin = read_file(bin_path, &w->bin_bytes);
    if (!w->bin) {
        pkcu_weights_destroy(w);
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_open: cannot read %s", bin_path);
    }
    for (int i = 0; i < w->n; i++) {
        const Entry *e = &w->e[i];
        const long long nb = elem_bytes(e);
        int bad = e->offset < 0 || e->numel < 0 || e->offset + nb > w->bin_bytes;
        if (e->dtype == PKCU_DTYPE_I4)
            bad |= e->scales_offset < 0 || e->n_scales <= 0 ||
                   e->scales_offset + 4 * e->n_scales > w->bin_bytes || e->ndim != 2 ||
                   e->shape[0] * e->shape[1] != e->numel;
        if (bad) {
            const int idx = i;
            char name[128];
            snprintf(name, sizeof name, "%s", w->e[idx].name);
            pkcu_weights_destroy(w);
            return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_open: entry '%s' lies outside %s or is malformed",
                             name, bin_path);
        }
    }
    while (1) {   /* conformer blocks: layers.0 .. with a linear_q weight */
        char name[64];
        snprintf(name, sizeof name, "layers.%d.self_attn.linear_q.weight", w->n_blocks);
        int found = 0;
        for (int i = 0; i < w->n && !found; i++) found = strcmp(w->e[i].name, name) == 0;
        if (!found) break;
        w->n_blocks++;
    }
    *out = w;
    return PKCU_OK;
}

int pkcu_weights_count(const pkcu_weights *w) { return w ? w->n : 0; }

const char *pkcu_weights_name(const pkcu_weights *w, int index)
{
    return (w && index >= 0 && index < w->n) ? w->e[index].name : NULL;
}

static const Entry *find(const pkcu_weights *w, const char *name)
{
    for (int i = 0; i < w->n; i++)
        if (strcmp(w->e[i].name, name) == 0) return &w->e[i];
    return NULL;
}

int pkcu_weights_find(const pkcu_weights *w, const char *name, pkcu_tensor *t)
{
    if (!w || !name || !t) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_find: NULL argument");
    const Entry *e = find(w, name);
    if (!e) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_find: no tensor '%s'", name);
    memset(t, 0, sizeof(*t));
    t->dtype = e->dtype;
    t->ndim = e->ndim < 4 ? e->ndim : 4;
    for (int d = 0; d < t->ndim; d++) t->shape[d] = e->shape[d];
    t->numel = e->numel;
    t->scale = e->scale;
    t->n_scales = e->n_scales;
    t->host = w->bin + e->offset;
    t->host_scales = e->dtype == PKCU_DTYPE_I4 ? (const float *)(w->bin + e->scales_offset) : NULL;
    if (w->arena) {
        t->dev = w->arena + e->slot;
        t->dev_scales = e->scales_slot >= 0 ? (const float *)(w->arena + e->scales_slot) : NULL;
    }
    return PKCU_OK;
}

/* ── upload ──────────────────────────────────────────────────────────────── */

static long long align256(long long x) { return (x + 255) & ~255LL; }

static const Entry *block_entry(const pkcu_weights *w, int b, const char *suffix)
{
    char name[160];
    snprintf(name, sizeof name, "layers.%d.%s", b, suffix);
    return find(w, name);
}

/* q, k, v of block b share one dtype and a square [D, D] shape. */
static int qkv_layout(const pkcu_weights *w, int b, const Entry *q[3], const Entry *bias[3],
                      int *D)
{
    static const char *wn[3] = {"self_attn.linear_q.weight", "self_attn.linear_k.weight",
                                "self_attn.linear_v.weight"};
    static const char *bn[3] = {"self_attn.linear_q.bias", "self_attn.linear_k.bias",
                                "self_attn.linear_v.bias"};
    for (int m = 0; m < 3; m++) {
        q[m] = block_entry(w, b, wn[m]);
        bias[m] = block_entry(w, b, bn[m]);
        if (!q[m] || !bias[m]) return 0;
    }
    const int dt = q[0]->dtype;
    if (q[1]->dtype != dt || q[2]->dtype != dt || q[0]->ndim != 2) return 0;
    const long long d = q[0]->shape[0];
    const long long cols = dt == PKCU_DTYPE_I4 ? 2 * q[0]->shape[1] : q[0]->shape[1];
    if (cols != d || d <= 0 || d % 32) return 0;
    for (int m = 0; m < 3; m++) {
        if (q[m]->ndim != 2 || q[m]->shape[0] != q[0]->shape[0] || q[m]->shape[1] != q[0]->shape[1])
            return 0;
        if (bias[m]->dtype != PKCU_DTYPE_F32 || bias[m]->numel != d) return 0;
        if (dt == PKCU_DTYPE_I8 && !(q[m]->scale > 0.0f)) return 0;
        if (dt == PKCU_DTYPE_I4 && q[m]->n_scales != d * (d / 32)) return 0;
    }
    *D = (int)d;
    return 1;
}

int pkcu_weights_upload(pkcu_weights *w, pkcu_stream_t stream)
{
    if (!w) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_upload: NULL weights");
    if (w->arena) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_upload: already uploaded");
    cudaStream_t s = (cudaStream_t)stream;
    /* slots for every tensor (and int4 scales) */
    long long at = 0;
    for (int i = 0; i < w->n; i++) {
        Entry *e = &w->e[i];
        e->slot = at;
        at = align256(at + elem_bytes(e));
        e->scales_slot = -1;
        if (e->dtype == PKCU_DTYPE_I4) {
            e->scales_slot = at;
            at = align256(at + 4 * e->n_scales);
        }
    }
    /* fused QKV per block, for the blocks that have q, k and v */
    const int nb = w->n_blocks;
    w->fused = nb ? (Fused *)calloc((size_t)nb, sizeof(Fused)) : NULL;
    if (nb && !w->fused) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_weights_upload: host allocation");
    for (int b = 0; b < nb; b++) {
        const Entry *q[3], *bias[3];
        int D = 0;
        Fused *f = &w->fused[b];
        if (!qkv_layout(w, b, q, bias, &D)) continue;
        f->ok = 1;
        f->bits = q[0]->dtype == PKCU_DTYPE_I8 ? 8 : 32;
        f->w_slot = at;
        at = align256(at + (long long)D * 3 * D * (f->bits == 8 ? 1 : 4));
        f->b_slot = at;
        at = align256(at + 4LL * 3 * D);
    }
    w->arena_bytes = at;
    cudaGetDevice(&w->device);
    if (cudaMalloc((void **)&w->arena, (size_t)(at ? at : 256)) != cudaSuccess) {
        cudaGetLastError();
        w->arena = NULL;
        return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_weights_upload: %lld bytes of device memory", at);
    }
    /* Page-lock the host copy for full-speed copies; pageable memory still works. */
    if (!w->registered && w->bin_bytes > 0) {
        if (cudaHostRegister(w->bin, (size_t)w->bin_bytes, cudaHostRegisterDefault) == cudaSuccess)
            w->registered = 1;
        else
            cudaGetLastError();
    }
    for (int i = 0; i < w->n; i++) {
        const Entry *e = &w->e[i];
        if (cudaMemcpyAsync(w->arena + e->slot, w->bin + e->offset, (size_t)elem_bytes(e),
                            cudaMemcpyHostToDevice, s) != cudaSuccess ||
            (e->dtype == PKCU_DTYPE_I4 &&
             cudaMemcpyAsync(w->arena + e->scales_slot, w->bin + e->scales_offset,
                             (size_t)(4 * e->n_scales), cudaMemcpyHostToDevice, s) != cudaSuccess))
            return pkcu_launch_status("pkcu_weights_upload: copy");
    }
    for (int b = 0; b < nb; b++) {
        Fused *f = &w->fused[b];
        if (!f->ok) continue;
        const Entry *q[3], *bias[3];
        int D = 0;
        qkv_layout(w, b, q, bias, &D);
        void *fw = w->arena + f->w_slot;
        float *fb = (float *)(w->arena + f->b_slot);
        int st = PKCU_OK;
        if (q[0]->dtype == PKCU_DTYPE_I8) {
            st = pkcu_requant_qkv_i8((const int8_t *)(w->arena + q[0]->slot),
                                     (const int8_t *)(w->arena + q[1]->slot),
                                     (const int8_t *)(w->arena + q[2]->slot), q[0]->scale,
                                     q[1]->scale, q[2]->scale, (int8_t *)fw, &f->scale, D, D,
                                     stream);
        } else if (q[0]->dtype == PKCU_DTYPE_I4) {
            st = pkcu_dequant_i4_qkv(w->arena + q[0]->slot, w->arena + q[1]->slot,
                                     w->arena + q[2]->slot,
                                     (const float *)(w->arena + q[0]->scales_slot),
                                     (const float *)(w->arena + q[1]->scales_slot),
                                     (const float *)(w->arena + q[2]->scales_slot), (float *)fw, D,
                                     D, 32, stream);
        } else {
            for (int m = 0; m < 3 && !st; m++)
                if (cudaMemcpy2DAsync((float *)fw + (size_t)m * D, (size_t)3 * D * 4,
                                      w->arena + q[m]->slot, (size_t)D * 4, (size_t)D * 4,
                                      (size_t)D, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
                    st = pkcu_launch_status("pkcu_weights_upload: QKV interleave");
        }
        for (int m = 0; m < 3 && !st; m++)
            if (cudaMemcpyAsync(fb + (size_t)m * D, w->arena + bias[m]->slot, (size_t)D * 4,
                                cudaMemcpyDeviceToDevice, s) != cudaSuccess)
                st = pkcu_launch_status("pkcu_weights_upload: bias concat");
        if (st) return st;
    }
    if (cudaStreamSynchronize(s) != cudaSuccess)
        return pkcu_launch_status("pkcu_weights_upload");
    return PKCU_OK;
}

/* ── device views ─────────────────────────────────────────────────────────── */

static int need_upload(const pkcu_weights *w, const char *what)
{
    if (!w) return pkcu_fail(PKCU_ERR_ARG, "%s: NULL weights", what);
    if (!w->arena) return pkcu_fail(PKCU_ERR_ARG, "%s: weights not uploaded", what);
    return PKCU_OK;
}

int pkcu_weights_dequant(const pkcu_weights *w, const char *name, float *out, pkcu_stream_t stream)
{
    int st = need_upload(w, "pkcu_weights_dequant");
    if (st) return st;
    if (!name || !out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_dequant: NULL argument");
    const Entry *e = find(w, name);
    if (!e) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_dequant: no tensor '%s'", name);
    const void *src = w->arena + e->slot;
    if (e->dtype == PKCU_DTYPE_F32) {
        if (cudaMemcpyAsync(out, src, (size_t)(4 * e->numel), cudaMemcpyDeviceToDevice,
                            (cudaStream_t)stream) != cudaSuccess)
            return pkcu_launch_status("pkcu_weights_dequant");
        return PKCU_OK;
    }
    if (e->dtype == PKCU_DTYPE_I8) return pkcu_dequant_i8((const int8_t *)src, e->scale, out, e->numel, stream);
    /* int4: packed [K, N/2], scales [K, N/32] (the exporter's G = 32 along N) */
    const long long K = e->shape[0], N = 2 * e->shape[1];
    if (N % 32 || e->n_scales != K * (N / 32) || K > 0x7fffffff || N > 0x7fffffff)
        return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_dequant: int4 '%s' has %lld scales for [%lld, %lld]",
                         name, e->n_scales, K, N);
    return pkcu_dequant_i4((const uint8_t *)src, (const float *)(w->arena + e->scales_slot), out,
                           (int)K, (int)N, 32, PKCU_GROUP_ALONG_N, stream);
}

int pkcu_weights_fused_qkv(const pkcu_weights *w, int block, const void **weight, int *bits,
                           float *scale, const float **bias)
{
    int st = need_upload(w, "pkcu_weights_fused_qkv");
    if (st) return st;
    if (block < 0 || block >= w->n_blocks || !w->fused[block].ok)
        return pkcu_fail(PKCU_ERR_ARG,
                         "pkcu_weights_fused_qkv: block %d has no q/k/v of one dtype and square shape",
                         block);
    const Fused *f = &w->fused[block];
    if (weight) *weight = w->arena + f->w_slot;
    if (bits) *bits = f->bits;
    if (scale) *scale = f->bits == 8 ? f->scale : 0.0f;
    if (bias) *bias = (const float *)(w->arena + f->b_slot);
    return PKCU_OK;
}

int pkcu_weights_block_params(const pkcu_weights *w, int block, pkcu_block_params *p)
{
    int st = need_upload(w, "pkcu_weights_block_params");
    if (st) return st;
    if (!p) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_block_params: NULL params");
    static const char *names[22] = {
        "norm_feed_forward1.weight", "norm_feed_forward1.bias", "feed_forward1.linear1.bias",
        "feed_forward1.linear2.bias", "norm_self_att.weight", "norm_self_att.bias", NULL,
        "self_attn.pos_bias_u", "self_attn.pos_bias_v", "self_attn.linear_out.bias",
        "norm_conv.weight", "norm_conv.bias", "conv.pointwise_conv1.bias",
        "conv.depthwise_conv.weight", "conv.depthwise_conv.bias", "conv.pointwise_conv2.bias",
        "norm_feed_forward2.weight", "norm_feed_forward2.bias", "feed_forward2.linear1.bias",
        "feed_forward2.linear2.bias", "norm_out.weight", "norm_out.bias"};
    const float *v[22];
    for (int i = 0; i < 22; i++) {
        if (!names[i]) {   /* qkv_b: the concatenated [Bq | Bk | Bv] */
            const float *fb = NULL;
            st = pkcu_weights_fused_qkv(w, block, NULL, NULL, NULL, &fb);
            if (st) return st;
            v[i] = fb;
            continue;
        }
        const Entry *e = block_entry(w, block, names[i]);
        if (!e || e->dtype != PKCU_DTYPE_F32)
            return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_block_params: block %d has no float32 '%s'",
                             block, names[i]);
        v[i] = (const float *)(w->arena + e->slot);
    }
    p->norm_ff1_w = v[0];  p->norm_ff1_b = v[1];  p->ff1_b1 = v[2];      p->ff1_b2 = v[3];
    p->norm_sa_w = v[4];   p->norm_sa_b = v[5];   p->qkv_b = v[6];       p->pos_u = v[7];
    p->pos_v = v[8];       p->out_b = v[9];       p->norm_conv_w = v[10]; p->norm_conv_b = v[11];
    p->pw1_b = v[12];      p->dw_w = v[13];       p->dw_b = v[14];       p->pw2_b = v[15];
    p->norm_ff2_w = v[16]; p->norm_ff2_b = v[17]; p->ff2_b1 = v[18];     p->ff2_b2 = v[19];
    p->norm_out_w = v[20]; p->norm_out_b = v[21];
    return PKCU_OK;
}

int pkcu_weights_blocks(const pkcu_weights *w) { return w ? w->n_blocks : 0; }

int pkcu_weights_pre_params(const pkcu_weights *w, pkcu_pre_params *p)
{
    int st = need_upload(w, "pkcu_weights_pre_params");
    if (st) return st;
    if (!p) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_pre_params: NULL params");
    static const char *names[9] = {
        "pre_encode.conv.0.weight", "pre_encode.conv.0.bias", "pre_encode.conv.2.weight",
        "pre_encode.conv.2.bias", "pre_encode.conv.3.bias", "pre_encode.conv.5.weight",
        "pre_encode.conv.5.bias", "pre_encode.conv.6.bias", "pre_encode.out.bias"};
    const float *v[9];
    for (int i = 0; i < 9; i++) {
        const Entry *e = find(w, names[i]);
        if (!e || e->dtype != PKCU_DTYPE_F32)
            return pkcu_fail(PKCU_ERR_ARG, "pkcu_weights_pre_params: no float32 '%s'", names[i]);
        v[i] = (const float *)(w->arena + e->slot);
    }
    p->conv0_w = v[0]; p->conv0_b = v[1]; p->conv2_w = v[2]; p->conv2_b = v[3];
    p->conv3_b = v[4]; p->conv5_w = v[5]; p->conv5_b = v[6]; p->conv6_b = v[7];
    p->out_b = v[8];
    return PKCU_OK;
}
