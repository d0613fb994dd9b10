/*  pk_oracle_weights.c -- CPU restatement of the reference's weight
 *  dequantisation (TEST INFRASTRUCTURE ONLY, see pk_oracle.h).
 *
 *  Built like the reference's csrc/weights.c: without -ffast-math
 *  (csrc/Makefile:22-25). Every result here is one integer-to-float
 *  conversion and one rounding, so the GPU kernels must match bit for bit.
 */
#include "pk_oracle.h"
#include <math.h>
#include <string.h>

/* int8 per-tensor dequant, as packed by pack_B_panel_q (csrc/blas.c:526-558):
 * w = (float)q * scale. */
void or_dequant_i8(const int8_t *q, float scale, float *out, long long n)
{
    for (long long i = 0; i < n; i++) out[i] = (float)q[i] * scale;
}

static void requant_slice(const int8_t *src, float s, float ms, int8_t *dst, int D)
{
    if (s == ms) { memcpy(dst, src, (size_t)D); return; }
    float r = s / ms;
    for (int n = 0; n < D; n++) {
        int v = (int)roundf(src[n] * r);
        dst[n] = (int8_t)(v < -127 ? -127 : v > 127 ? 127 : v);
    }
}

/* Fused-QKV int8 build (csrc/weights.c:437-487): common scale
 * ms = max(sq, sk, sv); each of Wq|Wk|Wv [K, D] is requantised to ms
 * (q' = clamp(roundf(q * (s/ms)), -127, 127), copied when s == ms) and the
 * three are interleaved per row into [K, 3D]. Returns ms. */
float or_requant_qkv_i8(const int8_t *q, const int8_t *k, const int8_t *v,
                        float sq, float sk, float sv, int8_t *fused, int K, int D)
{
    float ms = sq;
    if (sk > ms) ms = sk;
    if (sv > ms) ms = sv;
    for (int r = 0; r < K; r++) {
        int8_t *dst = fused + (size_t)r * 3 * D;
        requant_slice(q + (size_t)r * D, sq, ms, dst, D);
        requant_slice(k + (size_t)r * D, sk, ms, dst + D, D);
        requant_slice(v + (size_t)r * D, sv, ms, dst + 2 * D, D);
    }
    return ms;
}

/* Signed nibbles of one packed byte (csrc/blas.c:836-839,
 * extract_weights.py:589-594): low nibble is the even column. */
static inline int nib_lo(uint8_t b) { return (int)(signed char)((b & 0x0F) << 4) >> 4; }
static inline int nib_hi(uint8_t b) { return (int)(signed char)(b & 0xF0) >> 4; }

/* int4 group dequant of W [K, N] packed as [K, N/2] bytes.
 *   axis 1 (the reference layout, csrc/blas.c:785-794, csrc/weights.c:505-515):
 *     groups of `group` columns along N, scales [K, N/group],
 *     s = scales[k*(N/group) + col/group].
 *   axis 0 (groups of `group` rows along K): scales [K/group, N],
 *     s = scales[(k/group)*N + col].
 * w = (float)q * s. */
void or_dequant_i4(const uint8_t *packed, const float *scales, float *out,
                   int K, int N, int group, int axis)
{
    int half = N / 2, n_groups = N / group;
    for (int k = 0; k < K; k++)
        for (int j = 0; j < half; j++) {
            uint8_t byte = packed[(size_t)k * half + j];
            int c0 = 2 * j, c1 = 2 * j + 1;
            float s0, s1;
            if (axis == 1) {
                s0 = scales[(size_t)k * n_groups + c0 / group];
                s1 = scales[(size_t)k * n_groups + c1 / group];
            } else {
                s0 = scales[(size_t)(k / group) * N + c0];
                s1 = scales[(size_t)(k / group) * N + c1];
            }
            out[(size_t)k * N + c0] = (float)nib_lo(byte) * s0;
            out[(size_t)k * N + c1] = (float)nib_hi(byte) * s1;
        }
}

/* Fused-QKV int4 path (csrc/weights.c:488-544): Wq|Wk|Wv each [K, D] int4
 * with [K, D/group] scales, dequantised to fp32 and interleaved into [K, 3D]. */
void or_dequant_i4_qkv(const uint8_t *pq, const uint8_t *pk, const uint8_t *pv,
                       const float *sq, const float *sk, const float *sv,
                       float *fused, int K, int D, int group)
{
    const uint8_t *src[3] = {pq, pk, pv};
    const float *sc[3] = {sq, sk, sv};
    int half = D / 2, n_groups = D / group;
    for (int r = 0; r < K; r++)
        for (int m = 0; m < 3; m++) {
            float *dst = fused + (size_t)r * 3 * D + (size_t)m * D;
            const uint8_t *s = src[m] + (size_t)r * half;
            for (int j = 0; j < half; j++) {
                int col = 2 * j;
                float g = sc[m][(size_t)r * n_groups + col / group];
                dst[col] = (float)nib_lo(s[j]) * g;
                dst[col + 1] = (float)nib_hi(s[j]) * g;
            }
        }
}
