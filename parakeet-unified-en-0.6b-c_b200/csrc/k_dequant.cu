// k_dequant.cu -- weight dequantisation (int8 per tensor, int4 per group, the
// fused-QKV int8 requantisation) and the RNN-T greedy argmax.
//
// Every output here is one int->float conversion and one IEEE rounding, the
// same operations the reference performs, so results are bit-identical:
//   int8  w = (float)q * scale                 csrc/blas.c:526-558
//   QKV   q' = clamp(roundf((float)q * (s/ms)), -127, 127)   csrc/weights.c:437-487
//   int4  w = (float)nibble * scale[group]     csrc/blas.c:780-843, csrc/weights.c:488-544
// Dequant reads 1 (int8) or 0.5 + 4/G (int4) bytes and writes 4 bytes per
// weight; the kernels move 16 weights per thread per step (128-bit loads of
// int8, 64-bit loads of packed int4, four 128-bit stores).
//
// Argmax (csrc/decoder.c:106-114): one warp per row of V logits; lanes keep
// (value, index) of their strided entries, NaN entries never become the best,
// ties keep the lower index, and a NaN at index 0 returns 0, which is what the
// reference's strict '>' scan from index 0 does.
#include <math.h>

#include "pk_common.cuh"

namespace pk {

constexpr int DQ_THREADS = 256;

__device__ __forceinline__ float4 i8x4_to_f4(uint32_t w, float s) {
  return make_float4((float)(int8_t)(w & 0xff) * s, (float)(int8_t)((w >> 8) & 0xff) * s,
                     (float)(int8_t)((w >> 16) & 0xff) * s, (float)(int8_t)(w >> 24) * s);
}

__global__ void __launch_bounds__(DQ_THREADS)
dequant_i8_kernel(const int8_t *__restrict__ q, float scale, float *__restrict__ out, long long n,
                  int vec) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long done = 0;
  if (vec) {
    const long long n16 = n >> 4;
    for (; i < n16; i += stride) {
      const uint4 raw = __ldcs(reinterpret_cast<const uint4 *>(q) + i);
      float *o = out + 16 * i;
      st4(o, i8x4_to_f4(raw.x, scale));
      st4(o + 4, i8x4_to_f4(raw.y, scale));
      st4(o + 8, i8x4_to_f4(raw.z, scale));
      st4(o + 12, i8x4_to_f4(raw.w, scale));
    }
    done = n16 << 4;
    i = done + (long long)blockIdx.x * blockDim.x + threadIdx.x;
  }
  for (; i < n; i += stride) out[i] = (float)q[i] * scale;
}

// r[m] = s_m / ms, copy[m] = (s_m == ms) for the Q, K, V slices.
struct Requant {
  float r[3];
  int copy[3];
};

__device__ __forceinline__ int8_t requant1(int8_t v, float r, int copy) {
  if (copy) return v;
  int t = (int)roundf((float)v * r);
  t = t < -127 ? -127 : (t > 127 ? 127 : t);
  return (int8_t)t;
}

__global__ void __launch_bounds__(DQ_THREADS)
requant_qkv_kernel(const int8_t *__restrict__ q, const int8_t *__restrict__ k,
                   const int8_t *__restrict__ v, Requant rq, int8_t *__restrict__ fused, int K,
                   int D, int vec) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int8_t *src[3] = {q, k, v};
  if (vec) {
    const int per_row = 3 * D / 16;
    const long long n = (long long)K * per_row;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const int r = (int)(i / per_row);
      const int col = (int)(i - (long long)r * per_row) * 16;
      const int m = col / D, c = col - m * D;
      uint4 raw = __ldcs(reinterpret_cast<const uint4 *>(src[m] + (long long)r * D + c));
      int8_t *b = reinterpret_cast<int8_t *>(&raw);
#pragma unroll
      for (int e = 0; e < 16; e++) b[e] = requant1(b[e], rq.r[m], rq.copy[m]);
      *reinterpret_cast<uint4 *>(fused + (long long)r * 3 * D + col) = raw;
    }
  } else {
    const long long n = (long long)K * 3 * D;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const int r = (int)(i / (3 * D));
      const int col = (int)(i - (long long)r * 3 * D);
      const int m = col / D, c = col - m * D;
      fused[i] = requant1(src[m][(long long)r * D + c], rq.r[m], rq.copy[m]);
    }
  }
}

__device__ __forceinline__ int nib_lo(uint32_t b) { return ((int)((b & 0x0F) << 28)) >> 28; }
__device__ __forceinline__ int nib_hi(uint32_t b) { return ((int)((b & 0xF0) << 24)) >> 28; }

// 16 weights of row k starting at column col0 (col0 % 16 == 0) from 8 packed bytes.
__device__ __forceinline__ void dq4_16(uint2 raw, const float *scales, int k, int col0, int N,
                                       int G, int axis, float *o) {
  const uint32_t w[2] = {raw.x, raw.y};
  float sc[16];
  if (axis == PKCU_GROUP_ALONG_N) {
    const int ng = N / G;
    if (G % 16 == 0) {
      const float s = __ldg(scales + (long long)k * ng + col0 / G);
#pragma unroll
      for (int e = 0; e < 16; e++) sc[e] = s;
    } else {
#pragma unroll
      for (int e = 0; e < 16; e++) sc[e] = __ldg(scales + (long long)k * ng + (col0 + e) / G);
    }
  } else {
    const float *sr = scales + (long long)(k / G) * N + col0;
#pragma unroll
    for (int e = 0; e < 16; e++) sc[e] = __ldg(sr + e);
  }
  float f[16];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const uint32_t byte = (w[j >> 2] >> (8 * (j & 3))) & 0xff;
    f[2 * j] = (float)nib_lo(byte) * sc[2 * j];
    f[2 * j + 1] = (float)nib_hi(byte) * sc[2 * j + 1];
  }
#pragma unroll
  for (int e = 0; e < 16; e += 4) st4(o + e, make_float4(f[e], f[e + 1], f[e + 2], f[e + 3]));
}

__global__ void __launch_bounds__(DQ_THREADS)
dequant_i4_kernel(const uint8_t *__restrict__ packed, const float *__restrict__ scales,
                  float *__restrict__ out, int K, int N, int G, int axis, int vec) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  if (vec) {
    const int per_row = N / 16;
    const long long n = (long long)K * per_row;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const int k = (int)(i / per_row);
      const int col0 = (int)(i - (long long)k * per_row) * 16;
      const uint2 raw = __ldcs(reinterpret_cast<const uint2 *>(packed + (long long)k * (N / 2) + col0 / 2));
      dq4_16(raw, scales, k, col0, N, G, axis, out + (long long)k * N + col0);
    }
  } else {
    const long long n = (long long)K * N;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const int k = (int)(i / N);
      const int col = (int)(i - (long long)k * N);
      const uint32_t byte = packed[(long long)k * (N / 2) + col / 2];
      const int q4 = (col & 1) ? nib_hi(byte) : nib_lo(byte);
      const float s = axis == PKCU_GROUP_ALONG_N ? scales[(long long)k * (N / G) + col / G]
                                                 : scales[(long long)(k / G) * N + col];
      out[i] = (float)q4 * s;
    }
  }
}

__global__ void __launch_bounds__(DQ_THREADS)
dequant_i4_qkv_kernel(const uint8_t *__restrict__ pq, const uint8_t *__restrict__ pk,
                      const uint8_t *__restrict__ pv, const float *__restrict__ sq,
                      const float *__restrict__ sk, const float *__restrict__ sv,
                      float *__restrict__ fused, int K, int D, int G) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const int per_row = 3 * D / 16;
  const long long n = (long long)K * per_row;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int k = (int)(i / per_row);
    const int col = (int)(i - (long long)k * per_row) * 16;
    const int m = col / D, c0 = col - m * D;
    const uint8_t *p = m == 0 ? pq : (m == 1 ? pk : pv);
    const float *s = m == 0 ? sq : (m == 1 ? sk : sv);
    const uint2 raw = __ldcs(reinterpret_cast<const uint2 *>(p + (long long)k * (D / 2) + c0 / 2));
    dq4_16(raw, s, k, c0, D, G, PKCU_GROUP_ALONG_N, fused + (long long)k * 3 * D + col);
  }
}

constexpr int AM_ROWS_PER_CTA = 8;

__global__ void __launch_bounds__(32 * AM_ROWS_PER_CTA)
argmax_rows_kernel(const float *__restrict__ logits, int32_t *__restrict__ out, long long n_rows,
                   int V) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * AM_ROWS_PER_CTA + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const float *l = logits + row * V;
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int j = lane; j < V; j += 32) {
    const float v = __ldcs(l + j);
    if (!isnan(v) && (v > bv || (v == bv && j < bi))) { bv = v; bi = j; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(PK_FULL_MASK, bv, o);
    const int oi = __shfl_xor_sync(PK_FULL_MASK, bi, o);
    if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
  }
  if (lane == 0) out[row] = (isnan(__ldg(l)) || bi == INT_MAX) ? 0 : bi;
}

static unsigned dq_grid(long long work) {
  long long g = (work + DQ_THREADS - 1) / DQ_THREADS;
  const long long cap = (long long)pkcu_sm_count() * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

}  // namespace pk

using namespace pk;

extern "C" int pkcu_dequant_i8(const int8_t *q, float scale, float *out, long long n,
                               pkcu_stream_t stream) {
  if (!q || !out || n < 0) return pkcu_fail(PKCU_ERR_ARG, "pkcu_dequant_i8: bad argument");
  if (n == 0) return PKCU_OK;
  const int vec = PK_ALIGNED16(q) && PK_ALIGNED16(out);
  dequant_i8_kernel<<<dq_grid(vec ? n / 16 : n), DQ_THREADS, 0, (cudaStream_t)stream>>>(q, scale, out,
                                                                                       n, vec);
  return pkcu_launch_status("pkcu_dequant_i8");
}

extern "C" int pkcu_requant_qkv_i8(const int8_t *q, const int8_t *k, const int8_t *v, float sq,
                                   float sk, float sv, int8_t *fused, float *ms_out, int K, int D,
                                   pkcu_stream_t stream) {
  if (!q || !k || !v || !fused || K < 0 || D <= 0 || !(sq > 0.0f) || !(sk > 0.0f) ||
      !(sv > 0.0f))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_requant_qkv_i8: bad argument (scales must be > 0)");
  /* Common scale and per-slice ratios, as csrc/weights.c:440-447 computes them. */
  float ms = sq;
  if (sk > ms) ms = sk;
  if (sv > ms) ms = sv;
  Requant rq;
  const float s[3] = {sq, sk, sv};
  for (int m = 0; m < 3; m++) {
    rq.copy[m] = (s[m] == ms);
    rq.r[m] = s[m] / ms;
  }
  if (ms_out) *ms_out = ms;
  if (K == 0) return PKCU_OK;
  const int vec = (D % 16 == 0) && PK_ALIGNED16(q) && PK_ALIGNED16(k) && PK_ALIGNED16(v) &&
                  PK_ALIGNED16(fused);
  const long long work = vec ? (long long)K * 3 * D / 16 : (long long)K * 3 * D;
  requant_qkv_kernel<<<dq_grid(work), DQ_THREADS, 0, (cudaStream_t)stream>>>(q, k, v, rq, fused,
                                                                            K, D, vec);
  return pkcu_launch_status("pkcu_requant_qkv_i8");
}

extern "C" int pkcu_dequant_i4(const uint8_t *packed, const float *scales, float *out, int K,
                               int N, int group, int axis, pkcu_stream_t stream) {
  if (!packed || !scales || !out || K < 0 || N <= 0 || (N & 1) || group <= 0 ||
      (axis != PKCU_GROUP_ALONG_K && axis != PKCU_GROUP_ALONG_N) ||
      (axis == PKCU_GROUP_ALONG_N && N % group) || (axis == PKCU_GROUP_ALONG_K && K % group))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_dequant_i4: bad argument (N even, group divides the axis)");
  if (K == 0) return PKCU_OK;
  const int vec = (N % 16 == 0) && (((uintptr_t)packed & 7u) == 0) && PK_ALIGNED16(out);
  const long long work = vec ? (long long)K * N / 16 : (long long)K * N;
  dequant_i4_kernel<<<dq_grid(work), DQ_THREADS, 0, (cudaStream_t)stream>>>(packed, scales, out, K,
                                                                           N, group, axis, vec);
  return pkcu_launch_status("pkcu_dequant_i4");
}

extern "C" int pkcu_dequant_i4_qkv(const uint8_t *pq, const uint8_t *pk, const uint8_t *pv,
                                   const float *sq, const float *sk, const float *sv,
                                   float *fused, int K, int D, int group, pkcu_stream_t stream) {
  if (!pq || !pk || !pv || !sq || !sk || !sv || !fused || K < 0 || D <= 0 || D % 16 ||
      group <= 0 || D % group)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_dequant_i4_qkv: bad argument (D % 16 == 0, group | D)");
  if ((((uintptr_t)pq | (uintptr_t)pk | (uintptr_t)pv) & 7u) || !PK_ALIGNED16(fused))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_dequant_i4_qkv: misaligned pointer");
  if (K == 0) return PKCU_OK;
  dequant_i4_qkv_kernel<<<dq_grid((long long)K * 3 * D / 16), DQ_THREADS, 0,
                          (cudaStream_t)stream>>>(pq, pk, pv, sq, sk, sv, fused, K, D, group);
  return pkcu_launch_status("pkcu_dequant_i4_qkv");
}

extern "C" int pkcu_argmax_rows(const float *logits, int32_t *out, long long n_rows, int V,
                                pkcu_stream_t stream) {
  if (!logits || !out || n_rows < 0 || V <= 0)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_argmax_rows: bad argument");
  if (n_rows == 0) return PKCU_OK;
  argmax_rows_kernel<<<(unsigned)((n_rows + AM_ROWS_PER_CTA - 1) / AM_ROWS_PER_CTA),
                       32 * AM_ROWS_PER_CTA, 0, (cudaStream_t)stream>>>(logits, out, n_rows, V);
  return pkcu_launch_status("pkcu_argmax_rows");
}
