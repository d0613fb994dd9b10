// k_selftest.cu -- on-device checks of what the kernels rely on:
//  * rcp_1_2e126 (hardware reciprocal approximation + one fused Newton step)
//    equals the correctly rounded reciprocal __frcp_rn for every float d in
//    [1, 2^126) (bit-exact Swish and GLU gates);
//  * the bounded mbarrier wait of the bulk-copy kernels gives up and reports
//    when a phase never completes (a barrier that expects 16 bytes no copy
//    will deliver), leaving the context usable.
#include "pk_common.cuh"

namespace pk {

__global__ void __launch_bounds__(256)
selftest_rcp_kernel(unsigned lo, unsigned hi, unsigned long long *mismatches) {
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  unsigned long long bad = 0;
  for (unsigned long long u = lo + (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; u < hi;
       u += stride) {
    const float d = __uint_as_float((unsigned)u);
    bad += __float_as_uint(rcp_1_2e126(d)) != __float_as_uint(__frcp_rn(d));
  }
  if (bad) atomicAdd(mismatches, bad);
}

// One warp; no copy is ever issued, so nothing is in flight when it returns.
__global__ void selftest_wait_kernel(unsigned long long limit_ns, int *timed_out) {
  __shared__ unsigned long long bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_init_fence();
  }
  __syncwarp();
  if (threadIdx.x == 0) mbar_arrive_tx(&bar, 16);
  __syncwarp();
  const bool ok = mbar_wait(&bar, 0, limit_ns);
  if (threadIdx.x == 0) *timed_out = ok ? 0 : 1;
}

}  // namespace pk

using namespace pk;

extern "C" int pkcu_selftest_wait(int *timed_out) {
  if (!timed_out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_selftest_wait: NULL argument");
  int *d = nullptr;
  if (cudaMalloc(&d, sizeof(*d)) != cudaSuccess) {
    cudaGetLastError();
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_selftest_wait: device allocation");
  }
  int st = PKCU_OK;
  if (cudaMemset(d, 0xff, sizeof(*d)) != cudaSuccess)
    st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_selftest_wait: memset");
  if (!st) {
    selftest_wait_kernel<<<1, 32>>>(20000000ULL, d);   // 20 ms limit
    st = pkcu_launch_status("pkcu_selftest_wait");
  }
  if (!st && cudaMemcpy(timed_out, d, sizeof(*d), cudaMemcpyDeviceToHost) != cudaSuccess)
    st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_selftest_wait: %s", cudaGetErrorString(cudaGetLastError()));
  cudaFree(d);
  return st;
}

extern "C" int pkcu_selftest(unsigned long long *mismatches) {
  if (!mismatches) return pkcu_fail(PKCU_ERR_ARG, "pkcu_selftest: NULL argument");
  unsigned long long *d = nullptr;
  if (cudaMalloc(&d, sizeof(*d)) != cudaSuccess) {
    cudaGetLastError();
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_selftest: device allocation");
  }
  int st = PKCU_OK;
  if (cudaMemset(d, 0, sizeof(*d)) != cudaSuccess) st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_selftest: memset");
  if (!st) {
    selftest_rcp_kernel<<<pkcu_sm_count() * 8, 256>>>(0x3F800000u, 0x7E800000u, d);   // [1, 2^126)
    st = pkcu_launch_status("pkcu_selftest");
  }
  if (!st && cudaMemcpy(mismatches, d, sizeof(*d), cudaMemcpyDeviceToHost) != cudaSuccess)
    st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_selftest: %s", cudaGetErrorString(cudaGetLastError()));
  cudaFree(d);
  return st;
}
