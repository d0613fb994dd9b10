// k_split.cu -- fp32 activations as sums of three bf16 parts, the left-hand
// operand of the library's tcgen05 GEMM (k_tcgemm.cu).
//
// x = x0 + x1 + x2 with x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1)
// (round to nearest; each difference is exact in fp32, and the three 8-bit
// significands cover the 24 of an fp32 value, so the sum is x for normal
// values). A product sum_k a_k w_k is then a sum of part products a_i w_j,
// each exact in fp32; those with i + j <= 2 are kept (the others are below
// 2^-23 of |a||w| together, under fp32 rounding). The activation split writes
// each row as [a0 | a1 | a2], one K-major matrix of 3K columns.
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
