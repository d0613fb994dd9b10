// k_split.cu -- fp32 operands as sums of three bf16 parts, for fp32-accurate
// products on the bf16 tensor cores through plain library GEMMs
// (pk_encoder_model.c).
//
// x = x0 + x1 + x2 with x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1)
// (round to nearest; each difference is exact in fp32, and the three 8-bit
// significands cover the 24 of an fp32 value, so the sum is x for normal
// values). A product sum_k a_k w_k is then the sum of the nine part products
// a_i w_j, each exact in fp32; the six with i + j <= 2 are kept (the other
// three are below 2^-23 of |a||w| together, under fp32 rounding). They are
// summed band by band, one GEMM per band so that every GEMM adds products of
// one magnitude (the tensor cores align the products of a step to the largest
// before adding), the bands joined in fp32, smallest first:
//   band 2 = [a0 a1 a2] . [w2; w1; w0],  band 1 = [a0 a1] . [w1; w0],  band 0 = a0 . w0
// -- the activation split writes each row as [a0 | a1 | a2], the weight split
// writes the stack [w2; w1; w0] once at load, and each band reads a slice of
// both.
#include <cuda_bf16.h>

#include "pk_common.cuh"

namespace pk {

__device__ __forceinline__ void split3(float x, __nv_bfloat16 &p0, __nv_bfloat16 &p1, __nv_bfloat16 &p2) {
  p0 = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(p0);
  p1 = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(p1);
  p2 = __float2bfloat16_rn(r2);
}

struct __align__(8) bf16x4 {
  __nv_bfloat16 v[4];
};

// A [M, K] fp32 -> out [M, 3K] bf16, row m = [a0 | a1 | a2]; K % 4 == 0.
__global__ void split_rows_kernel(const float *__restrict__ A, __nv_bfloat16 *__restrict__ out, long long M,
                                  int K) {
  const int K4 = K / 4;
  const long long n4 = M * K4;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n4;
       e += (long long)gridDim.x * blockDim.x) {
    const long long m = e / K4;
    const int k = (int)(e - m * K4) * 4;
    const float4 a = __ldg(reinterpret_cast<const float4 *>(A) + e);
    bf16x4 q0, q1, q2;
    split3(a.x, q0.v[0], q1.v[0], q2.v[0]);
    split3(a.y, q0.v[1], q1.v[1], q2.v[1]);
    split3(a.z, q0.v[2], q1.v[2], q2.v[2]);
    split3(a.w, q0.v[3], q1.v[3], q2.v[3]);
    __nv_bfloat16 *row = out + m * 3 * K + k;
    *reinterpret_cast<bf16x4 *>(row) = q0;
    *reinterpret_cast<bf16x4 *>(row + K) = q1;
    *reinterpret_cast<bf16x4 *>(row + 2 * K) = q2;
  }
}

// W [K, N] fp32 -> S [3K, N] bf16 = [w2; w1; w0]; N % 4 == 0.
__global__ void split_stack_kernel(const float *__restrict__ W, __nv_bfloat16 *__restrict__ S, int K, int N) {
  const int N4 = N / 4;
  const long long n4 = (long long)K * N4;
  const long long part = (long long)K * N;   // elements per stacked copy
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n4;
       e += (long long)gridDim.x * blockDim.x) {
    const float4 w = __ldg(reinterpret_cast<const float4 *>(W) + e);
    bf16x4 q0, q1, q2;
    split3(w.x, q0.v[0], q1.v[0], q2.v[0]);
    split3(w.y, q0.v[1], q1.v[1], q2.v[1]);
    split3(w.z, q0.v[2], q1.v[2], q2.v[2]);
    split3(w.w, q0.v[3], q1.v[3], q2.v[3]);
    __nv_bfloat16 *p = S + 4 * e;
    *reinterpret_cast<bf16x4 *>(p) = q2;
    *reinterpret_cast<bf16x4 *>(p + part) = q1;
    *reinterpret_cast<bf16x4 *>(p + 2 * part) = q0;
  }
}

// items x [K, T] fp32 (channel-first) -> items x [3K, Tp] bf16 = [x2; x1; x0]
// per item, rows padded to the pitch Tp >= T (the pad columns are left as they
// are: they only feed output columns that are dropped). A warp per channel row
// (rows of T floats are not 16-byte aligned): lane-strided, coalesced loads and
// stores, four in flight.
__global__ void split_cols_kernel(const float *__restrict__ X, __nv_bfloat16 *__restrict__ out, long long items,
                                  int K, int T, int Tp) {
  const int lane = threadIdx.x & 31;
  const long long rows = items * K, part = (long long)K * Tp;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
    const long long it = r / K, k = r - it * K;
    const float *src = X + r * T;
    __nv_bfloat16 *o = out + it * 3 * part + k * Tp;
    for (int t0 = 0; t0 < T; t0 += 128) {
      float x[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int t = t0 + 32 * u + lane;
        x[u] = t < T ? __ldg(src + t) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int t = t0 + 32 * u + lane;
        if (t < T) {
          __nv_bfloat16 p0, p1, p2;
          split3(x[u], p0, p1, p2);
          o[t] = p2;
          o[part + t] = p1;
          o[2 * part + t] = p0;
        }
      }
    }
  }
}

// int8 -> bf16 (exact: |q| <= 128 fits the 8-bit significand).
__global__ void i8_to_bf16_kernel(const int8_t *__restrict__ q, __nv_bfloat16 *__restrict__ out, long long n) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x)
    out[e] = __float2bfloat16_rn((float)q[e]);
}

// rows x [Tp] -> rows x [T]: drops the pad columns; a warp per row, four
// accesses in flight per lane.
__global__ void depad_kernel(const float *__restrict__ src, float *__restrict__ dst, long long rows, int T,
                             int Tp) {
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
    const float *s = src + r * Tp;
    float *d = dst + r * T;
    for (int t0 = 0; t0 < T; t0 += 128) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int t = t0 + 32 * u + lane;
        v[u] = t < T ? __ldg(s + t) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int t = t0 + 32 * u + lane;
        if (t < T) d[t] = v[u];
      }
    }
  }
}

static unsigned split_grid(long long work) {
  long long g = (work + 255) / 256;
  const long long cap = (long long)pkcu_sm_count() * 16;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace pk

using namespace pk;

extern "C" int pk_split_rows_bf16x3(const float *A, void *out, long long M, int K, pkcu_stream_t stream) {
  if (!A || !out || M <= 0 || K <= 0 || K % 4 || !PK_ALIGNED16(A) || !PK_ALIGNED16(out))
    return pkcu_fail(PKCU_ERR_ARG, "pk_split_rows_bf16x3: bad argument");
  split_rows_kernel<<<split_grid(M * (K / 4)), 256, 0, (cudaStream_t)stream>>>(
      A, static_cast<__nv_bfloat16 *>(out), M, K);
  return pkcu_launch_status("pk_split_rows_bf16x3");
}

extern "C" int pk_split_stack_bf16x3(const float *W, void *S, int K, int N, pkcu_stream_t stream) {
  if (!W || !S || K <= 0 || N <= 0 || N % 4 || !PK_ALIGNED16(W) || !PK_ALIGNED16(S))
    return pkcu_fail(PKCU_ERR_ARG, "pk_split_stack_bf16x3: bad argument");
  split_stack_kernel<<<split_grid((long long)K * (N / 4)), 256, 0, (cudaStream_t)stream>>>(
      W, static_cast<__nv_bfloat16 *>(S), K, N);
  return pkcu_launch_status("pk_split_stack_bf16x3");
}

extern "C" int pk_split_cols_bf16x3(const float *X, void *out, long long items, int K, int T, int Tp,
                                    pkcu_stream_t stream) {
  if (!X || !out || items <= 0 || K <= 0 || T <= 0 || Tp < T)
    return pkcu_fail(PKCU_ERR_ARG, "pk_split_cols_bf16x3: bad argument");
  split_cols_kernel<<<split_grid(items * K * 32), 256, 0, (cudaStream_t)stream>>>(
      X, static_cast<__nv_bfloat16 *>(out), items, K, T, Tp);
  return pkcu_launch_status("pk_split_cols_bf16x3");
}

extern "C" int pk_depad_rows(const float *src, float *dst, long long rows, int T, int Tp, pkcu_stream_t stream) {
  if (!src || !dst || rows <= 0 || T <= 0 || Tp < T) return pkcu_fail(PKCU_ERR_ARG, "pk_depad_rows: bad argument");
  depad_kernel<<<split_grid(rows * 32), 256, 0, (cudaStream_t)stream>>>(src, dst, rows, T, Tp);
  return pkcu_launch_status("pk_depad_rows");
}

extern "C" int pk_i8_to_bf16(const int8_t *q, void *out, long long n, pkcu_stream_t stream) {
  if (!q || !out || n <= 0) return pkcu_fail(PKCU_ERR_ARG, "pk_i8_to_bf16: bad argument");
  i8_to_bf16_kernel<<<split_grid(n), 256, 0, (cudaStream_t)stream>>>(q, static_cast<__nv_bfloat16 *>(out), n);
  return pkcu_launch_status("pk_i8_to_bf16");
}
