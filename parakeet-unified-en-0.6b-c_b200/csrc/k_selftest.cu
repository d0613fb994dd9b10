// k_selftest.cu -- on-device check of the arithmetic assumption the kernels
// rely on for bit-exact results: rcp_1_2e126 (hardware reciprocal
// approximation + one fused Newton step) equals the correctly rounded
// reciprocal __frcp_rn for every float d in [1, 2^126).
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

}  // namespace pk

using namespace pk;

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
