// k_dequant.cu -- weight dequantisation (int8 per tensor, int4 per group, the
// fused-QKV int8 requantisation) and the RNN-T greedy argmax.
//
// Every output here is one int->float conversion and one IEEE rounding, the
// same operations the reference performs, so results are bit-identical:
//   int8  w = (float)q * scale                 csrc/blas.c:526-558
//   QKV   q' = clamp(roundf((float)q * (s/ms)), -127, 127)   csrc/weights.c:437-487
//   int4  w = (float)nibble * scale[group]     csrc/blas.c:780-843, csrc/weights.c:488-544
// Dequant reads 1 (int8) or 0.5 + 4/G (int4) bytes and writes 4 bytes per
// weight. The stores dominate, so the kernels are laid out for them: every
// warp store instruction writes 32 consecutive float4s (512 bytes). int8:
// each lane loads the 4 bytes of its own float4 (a warp load is 128
// consecutive bytes). int4: each lane loads one 32-bit word (8 weights) and a
// shuffle hands every lane the two packed bytes of the float4 it stores.
//
// Argmax (csrc/decoder.c:106-114): one warp per row of V logits; lanes keep
// (value, index) of their strided entries, NaN entries never become the best,
// ties keep the lower index, and a NaN at index 0 returns 0, which is what the
// reference's strict '>' scan from index 0 does.
#include <math.h>

#include "pk_common.cuh"

namespace pk {

constexpr int DQ_THREADS = 256;

// The four int8 values of w (byte i = weight i) times s. After w ^ 0x80808080
// each byte is q + 128 in [0, 255]; a byte permute places it under the
// exponent bits of 2^23, giving the float 2^23 + q + 128 exactly, and
// subtracting 2^23 + 128 leaves q exactly: (float)q * s with its single
// rounding, without integer-to-float conversions.
__device__ __forceinline__ float4 i8x4_to_f4(uint32_t w, float s) {
  constexpr float kVal = 8388736.0f;   // 2^23 + 128
  const uint32_t u = w ^ 0x80808080u;
  const float2 q01 = sub2(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)),
                                      __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441))),
                          splat2(kVal));
  const float2 q23 = sub2(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)),
                                      __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443))),
                          splat2(kVal));
  const float2 o01 = mul2(q01, splat2(s)), o23 = mul2(q23, splat2(s));
  return make_float4(o01.x, o01.y, o23.x, o23.y);
}

__global__ void __launch_bounds__(DQ_THREADS)
dequant_i8_kernel(const int8_t *__restrict__ q, float scale, float *__restrict__ out, long long n,
                  int vec) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long done = 0;
  if (vec) {   // q 4-byte, out 16-byte aligned: unit u = weights [4u, 4u + 4)
    const long long n4 = n >> 2;
    const uint32_t *q4 = reinterpret_cast<const uint32_t *>(q);
    for (; i + 3 * stride < n4; i += 4 * stride) {   // 4 loads in flight per thread
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; j++) w[j] = __ldcs(q4 + i + j * stride);
#pragma unroll
      for (int j = 0; j < 4; j++) st4(out + 4 * (i + j * stride), i8x4_to_f4(w[j], scale));
    }
    for (; i < n4; i += stride) st4(out + 4 * i, i8x4_to_f4(__ldcs(q4 + i), scale));
    done = n4 << 2;
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

// The four signed 4-bit values held in the 16 bits h (nibble i = bits
// 4i..4i+3, two's complement) times their scales. nibble ^ 8 is q + 8 in
// [0, 15]; placed in the mantissa of 2^23 it gives the float 2^23 + q + 8
// exactly, and subtracting 2^23 + 8 leaves q exactly, so the result is the
// reference's (float)q * scale with its single rounding.
__device__ __forceinline__ float4 nib4_scaled(uint32_t h, float4 s) {
  constexpr uint32_t kBits = 0x4B000008u;   // 2^23 + 8
  constexpr float kVal = 8388616.0f;
  const float2 q01 = sub2(make_float2(__uint_as_float((h & 0xFu) ^ kBits),
                                      __uint_as_float(((h >> 4) & 0xFu) ^ kBits)),
                          splat2(kVal));
  const float2 q23 = sub2(make_float2(__uint_as_float(((h >> 8) & 0xFu) ^ kBits),
                                      __uint_as_float(((h >> 12) & 0xFu) ^ kBits)),
                          splat2(kVal));
  const float2 o01 = mul2(q01, make_float2(s.x, s.y));
  const float2 o23 = mul2(q23, make_float2(s.z, s.w));
  return make_float4(o01.x, o01.y, o23.x, o23.y);
}

// The scales of the 4 weights at columns col .. col + 3 (col % 4 == 0) of a
// row whose scale row is srow: [K/G, N] layout (G along K, srow = scales +
// (k / G) * N) or [K, N/G] (G along N, srow = scales + k * N/G).
__device__ __forceinline__ float4 scales4(const float *__restrict__ srow, int col, int G, int axis,
                                          FastDiv div_G) {
  if (axis == PKCU_GROUP_ALONG_K) return __ldg(reinterpret_cast<const float4 *>(srow + col));
  if (G % 4 == 0) {
    const float t = __ldg(srow + fast_div((unsigned)col, div_G));
    return make_float4(t, t, t, t);
  }
  return make_float4(__ldg(srow + fast_div((unsigned)col, div_G)),
                     __ldg(srow + fast_div((unsigned)col + 1, div_G)),
                     __ldg(srow + fast_div((unsigned)col + 2, div_G)),
                     __ldg(srow + fast_div((unsigned)col + 3, div_G)));
}

__device__ __forceinline__ const float *scale_row(const float *scales, unsigned k, int N, int ng,
                                                  int axis, FastDiv div_G) {
  return axis == PKCU_GROUP_ALONG_K ? scales + (long long)fast_div(k, div_G) * N
                                    : scales + (long long)k * ng;
}

// Vector form (N % 8 == 0, packed 4-byte and out 16-byte aligned, fewer than
// 2^32 packed words). A warp chunk is 32 packed words = 256 weights; lane l
// loads word l of the chunk, then for store j in {0, 1} takes the 16 bits
// holding the chunk's float4 32j + l from word 16j + l/2, so every warp store
// writes 512 consecutive bytes. With N % 256 == 0 a chunk is a 256-column
// block of one row (one division per chunk); otherwise chunks run over the
// flat array and each float4 finds its row. Four chunks per warp per
// iteration, their loads issued together.
template <bool BLOCKS, bool PRE, bool NPRE = false>
__global__ void __launch_bounds__(DQ_THREADS)
dequant_i4_vec_kernel(const uint8_t *__restrict__ packed, const float *__restrict__ scales,
                      float *__restrict__ out, int K, int N, int G, int axis, FastDiv div_wpr,
                      FastDiv div_bpr, FastDiv div_G) {
  const int lane = threadIdx.x & 31;
  const unsigned wpr = (unsigned)N / 8;   // packed words per row
  const unsigned bpr = (unsigned)N / 256; // 256-column blocks per row
  const unsigned n_words = (unsigned)K * wpr;
  const unsigned n_chunks = (n_words + 31) >> 5;
  const unsigned warps = gridDim.x * (blockDim.x >> 5);
  const uint32_t *pw = reinterpret_cast<const uint32_t *>(packed);
  const int ng = N / G;
  constexpr int U = 8;
  for (unsigned c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); c < n_chunks;
       c += U * warps) {
    uint32_t w[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const unsigned wi = 32 * (c + u * warps) + lane;
      w[u] = wi < n_words ? __ldcs(pw + wi) : 0u;
    }
    // PRE (block chunks, scales along K: a float4 of scales per float4 of
    // weights): every chunk's scales requested before the first store, so their
    // (L2) latencies overlap instead of one per chunk (0.73 -> 0.88 of the copy
    // bandwidth at G = 128; along N, a broadcast float4 per float4 of weights
    // prefetched this way measured worse: see NPRE)
    float4 sv[PRE ? U : 1][2];
    // NPRE (block chunks, scales along N with G dividing 256, G >= 8): a chunk's
    // 256 / G scales are one load by lanes 0 .. 256 / G - 1, every chunk's
    // requested before the first store; each float4 then takes its group's scale
    // from the lane holding it (G = 32: 0.80 -> 0.82 of the copy bandwidth).
    float sn[NPRE ? U : 1];
    if (NPRE) {
      const unsigned gpc = 256u / (unsigned)G;
#pragma unroll
      for (int u = 0; u < U; u++) {
        const unsigned cu = c + u * warps;
        sn[u] = 0.0f;
        if (cu < n_chunks && (unsigned)lane < gpc) {
          const unsigned k = fast_div(cu, div_bpr);
          sn[u] = __ldg(scales + (long long)k * ng + fast_div(256 * (cu - k * bpr), div_G) + lane);
        }
      }
    }
    if (PRE) {
#pragma unroll
      for (int u = 0; u < U; u++) {
        const unsigned cu = c + u * warps;
        if (cu < n_chunks) {
          const unsigned k = fast_div(cu, div_bpr);
          const float *srow = scale_row(scales, k, N, ng, axis, div_G);
#pragma unroll
          for (int j = 0; j < 2; j++)
            sv[u][j] = scales4(srow, (int)(256 * (cu - k * bpr)) + 128 * j + 4 * lane, G, axis, div_G);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const unsigned cu = c + u * warps;
      if (cu >= n_chunks) break;   // warp-uniform
      unsigned k = 0, col0 = 0;
      const float *srow = nullptr;
      if (BLOCKS) {
        k = fast_div(cu, div_bpr);
        col0 = 256 * (cu - k * bpr);
        if (!PRE && !NPRE) srow = scale_row(scales, k, N, ng, axis, div_G);
      }
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const uint32_t src = __shfl_sync(PK_FULL_MASK, w[u], 16 * j + (lane >> 1));
        int col;
        if (NPRE) {
          col = (int)col0 + 128 * j + 4 * lane;
          const float t = __shfl_sync(PK_FULL_MASK, sn[NPRE ? u : 0],
                                      (int)fast_div((unsigned)(128 * j + 4 * lane), div_G));
          const uint32_t h = (lane & 1) ? src >> 16 : src & 0xffffu;
          st4(out + (long long)k * N + col, nib4_scaled(h, make_float4(t, t, t, t)));
          continue;
        }
        if (PRE) {
          col = (int)col0 + 128 * j + 4 * lane;
          const uint32_t h = (lane & 1) ? src >> 16 : src & 0xffffu;
          st4(out + (long long)k * N + col, nib4_scaled(h, sv[PRE ? u : 0][j]));
          continue;
        }
        if (BLOCKS) {
          col = (int)col0 + 128 * j + 4 * lane;
        } else {
          const unsigned ws = 32 * cu + 16 * j + (lane >> 1);   // word holding this float4
          if (ws >= n_words) continue;
          k = fast_div(ws, div_wpr);
          col = (int)(8 * (ws - k * wpr)) + 4 * (lane & 1);
          srow = scale_row(scales, k, N, ng, axis, div_G);
        }
        const uint32_t h = (lane & 1) ? src >> 16 : src & 0xffffu;
        st4(out + (long long)k * N + col, nib4_scaled(h, scales4(srow, col, G, axis, div_G)));
      }
    }
  }
}

// Any alignment: one weight per thread.
__global__ void __launch_bounds__(DQ_THREADS)
dequant_i4_kernel(const uint8_t *__restrict__ packed, const float *__restrict__ scales,
                  float *__restrict__ out, int K, int N, int G, int axis) {
  const long long stride = (long long)gridDim.x * blockDim.x;
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
  // each lane scans its entries in increasing order, so a strict '>' keeps the
  // first maximum, and a NaN never compares greater; 16 loads per lane in
  // flight (a 1025-logit row is 33 per lane)
#pragma unroll 16
  for (int j = lane; j < V; j += 32) {
    const float v = __ldcs(l + j);
    if (v > bv) { bv = v; bi = j; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(PK_FULL_MASK, bv, o);
    const int oi = __shfl_xor_sync(PK_FULL_MASK, bi, o);
    if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
  }
  if (lane == 0) out[row] = (isnan(__ldg(l)) || bi == INT_MAX) ? 0 : bi;
}

// Grid-stride kernels: at most one full wave of resident CTAs (from the
// kernel's occupancy), at most one CTA per DQ_THREADS units of work.
template <typename Kern>
static unsigned dq_grid(Kern kernel, long long work) {
  long long g = (work + DQ_THREADS - 1) / DQ_THREADS;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, DQ_THREADS, 0) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const long long cap = (long long)pkcu_sm_count() * per_sm;
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
  const int vec = (((uintptr_t)q & 3u) == 0) && PK_ALIGNED16(out);
  // aligned: four float4 units per thread, an uncapped grid (measured faster
  // than one wave striding over the array)
  long long g = vec ? (n / 4 + DQ_THREADS * 4 - 1) / (DQ_THREADS * 4) : 0;
  if (g > 0x7fffffffLL) g = 0x7fffffffLL;   // the kernel strides over the rest
  dequant_i8_kernel<<<vec ? (unsigned)(g < 1 ? 1 : g) : dq_grid(dequant_i8_kernel, n), DQ_THREADS, 0,
                      (cudaStream_t)stream>>>(q, scale, out, n, vec);
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
  requant_qkv_kernel<<<dq_grid(requant_qkv_kernel, work), DQ_THREADS, 0, (cudaStream_t)stream>>>(q, k, v, rq, fused,
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
  const bool vec = (N % 8 == 0) && (((uintptr_t)packed & 3u) == 0) && PK_ALIGNED16(out) &&
                   (axis == PKCU_GROUP_ALONG_N || PK_ALIGNED16(scales)) &&
                   (long long)K * N / 8 < (1LL << 32) - 64;
  if (vec && N % 256 == 0 && axis == PKCU_GROUP_ALONG_K)
    dequant_i4_vec_kernel<true, true><<<dq_grid(dequant_i4_vec_kernel<true, true>, (long long)K * N / 8),
                                        DQ_THREADS, 0, (cudaStream_t)stream>>>(
        packed, scales, out, K, N, group, axis, make_fastdiv((unsigned)(N / 8)),
        make_fastdiv((unsigned)(N / 256)), make_fastdiv((unsigned)group));
  else if (vec && N % 256 == 0 && group >= 8 && 256 % group == 0)
    dequant_i4_vec_kernel<true, false, true><<<dq_grid(dequant_i4_vec_kernel<true, false, true>,
                                                       (long long)K * N / 8),
                                               DQ_THREADS, 0, (cudaStream_t)stream>>>(
        packed, scales, out, K, N, group, axis, make_fastdiv((unsigned)(N / 8)),
        make_fastdiv((unsigned)(N / 256)), make_fastdiv((unsigned)group));
  else if (vec && N % 256 == 0)
    dequant_i4_vec_kernel<true, false><<<dq_grid(dequant_i4_vec_kernel<true, false>, (long long)K * N / 8),
                                         DQ_THREADS, 0, (cudaStream_t)stream>>>(
        packed, scales, out, K, N, group, axis, make_fastdiv((unsigned)(N / 8)),
        make_fastdiv((unsigned)(N / 256)), make_fastdiv((unsigned)group));
  else if (vec)
    dequant_i4_vec_kernel<false, false><<<dq_grid(dequant_i4_vec_kernel<false, false>, (long long)K * N / 8), DQ_THREADS, 0,
                                   (cudaStream_t)stream>>>(packed, scales, out, K, N, group, axis,
                                                           make_fastdiv((unsigned)(N / 8)),
                                                           make_fastdiv(1u),
                                                           make_fastdiv((unsigned)group));
  else
    dequant_i4_kernel<<<dq_grid(dequant_i4_kernel, (long long)K * N), DQ_THREADS, 0, (cudaStream_t)stream>>>(
        packed, scales, out, K, N, group, axis);
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
  dequant_i4_qkv_kernel<<<dq_grid(dequant_i4_qkv_kernel, (long long)K * 3 * D / 16), DQ_THREADS, 0,
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
