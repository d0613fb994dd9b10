// k_gemm.cu -- the GEMMs next to the tensor_ops path with their non-GEMM
// epilogues fused into them, so the GEMM output never makes the extra round
// trip through HBM that a separate bias / activation / residual kernel costs:
//
//   pkcu_gemm_bias_swish     D = Swish(A W + b)       FF linear1 + bias + Swish
//                                                     (csrc/encoder.c:193-196)
//   pkcu_gemm_bias_residual  X = X + s (A W + b)      FF linear2 + bias + the
//                                                     0.5-scaled macaron residual
//                                                     (:198-216, s = 0.5), the
//                                                     attention output projection
//                                                     + residual (:418-434, s = 1)
//   pk_gemm_f32_rm           C = A B                  the plain projections of the
//                                                     library's own encoder forward
//                                                     (pk_encoder_model.c)
//
// A [M, K], W [K, N] (row-major, the reference's weight layout), fp32 in and
// out like the reference's sgemm. The products run on the 5th-generation
// tensor cores through CUTLASS's sm100 FastFP32 collective: every fp32
// operand is split into three bf16 parts and each product is the sum of the
// nine bf16 MMAs (tcgen05.mma, accumulators in TMEM), which keeps fp32-level
// accuracy. Operand tiles are staged by TMA into shared memory, one CTA per
// cluster (no multicast). The epilogue reads the accumulator tile from TMEM,
// adds the bias (and for the residual form the tile of X) and applies the
// activation before the single store.
#include <cuda_runtime.h>

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/epilogue/fusion/operations.hpp"
#include "cutlass/epilogue/thread/activation.h"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/dispatch_policy.hpp"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

#include "pkcuda_internal.h"

namespace pk_gemm {
using namespace cute;

// x -> s * x (s = the call's residual scale)
template <class T>
using ScaledIdentity = cutlass::epilogue::thread::Scale<cutlass::epilogue::thread::Identity<T>>;

template <class FusionOp>
struct FastF32 {
  using Layout = cutlass::layout::RowMajor;
  static constexpr int kAlign = 4;   // 16 bytes of fp32
  using MmaTileShape = Shape<_128, _128, _32>;
  using ClusterShape = Shape<_1, _1, _1>;
  using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, MmaTileShape, ClusterShape,
      cutlass::epilogue::collective::EpilogueTileAuto, float, float, float, Layout, kAlign, float,
      Layout, kAlign, cutlass::epilogue::TmaWarpSpecialized1Sm, FusionOp>::CollectiveOp;
  using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, float, Layout, kAlign, float, Layout,
      kAlign, float, MmaTileShape, ClusterShape,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(
          sizeof(typename Epilogue::SharedStorage))>,
      cutlass::gemm::KernelTmaWarpSpecialized1SmFastFP32Sm100>::CollectiveOp;
  using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue, void>;
  using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
};

using SwishGemm = FastF32<cutlass::epilogue::fusion::LinCombPerColBiasEltAct<
    cutlass::epilogue::thread::SiLu, float, float, float, float>>::Gemm;
using ResidualGemm = FastF32<cutlass::epilogue::fusion::PerColResAddPerColBiasEltAct<
    ScaledIdentity, float, float, float, float>>::Gemm;
using PlainGemm = FastF32<cutlass::epilogue::fusion::LinearCombination<float, float, float, float>>::Gemm;

// Per-device workspace for kernels that ask for one (grown, never shrunk).
static void *g_ws[64];
static size_t g_ws_bytes[64];

static int workspace(size_t bytes, void **out) {
  *out = nullptr;
  if (bytes == 0) return PKCU_OK;
  const int dev = pkcu_device();
  if (dev >= 64) return pkcu_fail(PKCU_ERR_ARG, "pkcu_gemm: device index %d", dev);
  if (g_ws_bytes[dev] < bytes) {
    if (g_ws[dev]) cudaFree(g_ws[dev]);
    g_ws[dev] = nullptr;
    g_ws_bytes[dev] = 0;
    if (cudaMalloc(&g_ws[dev], bytes) != cudaSuccess) {
      cudaGetLastError();
      return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_gemm: workspace of %zu bytes", bytes);
    }
    g_ws_bytes[dev] = bytes;
  }
  *out = g_ws[dev];
  return PKCU_OK;
}

template <class Gemm>
static int run(typename Gemm::Arguments &args, cudaStream_t s, const char *what) {
  Gemm gemm;
  if (gemm.can_implement(args) != cutlass::Status::kSuccess)
    return pkcu_fail(PKCU_ERR_ARG, "%s: shape or alignment not supported", what);
  void *ws = nullptr;
  int st = workspace(Gemm::get_workspace_size(args), &ws);
  if (st) return st;
  if (gemm.initialize(args, ws, s) != cutlass::Status::kSuccess)
    return pkcu_fail(PKCU_ERR_CUDA, "%s: initialisation failed", what);
  if (gemm.run(s) != cutlass::Status::kSuccess) return pkcu_launch_status(what);
  return pkcu_launch_status(what);
}

static int check(const void *A, const void *W, const void *bias, const void *D, int M, int N, int K,
                 const char *what) {
  if (!A || !W || !bias || !D || M <= 0 || N <= 0 || K <= 0)
    return pkcu_fail(PKCU_ERR_ARG, "%s: NULL pointer or empty shape", what);
  if (N % 4 || K % 4)
    return pkcu_fail(PKCU_ERR_ARG, "%s: N and K must be multiples of 4 (16-byte rows)", what);
  if (!PK_ALIGNED16(A) || !PK_ALIGNED16(W) || !PK_ALIGNED16(bias) || !PK_ALIGNED16(D))
    return pkcu_fail(PKCU_ERR_ARG, "%s: A, W, bias and the output must be 16-byte aligned", what);
  return PKCU_OK;
}

template <class Gemm>
static auto strides(int M, int N, int K) {
  using Kn = typename Gemm::GemmKernel;
  return cute::make_tuple(
      cutlass::make_cute_packed_stride(typename Kn::StrideA{}, make_shape(M, K, 1)),
      cutlass::make_cute_packed_stride(typename Kn::StrideB{}, make_shape(N, K, 1)),
      cutlass::make_cute_packed_stride(typename Kn::StrideC{}, make_shape(M, N, 1)));
}

}  // namespace pk_gemm

using namespace pk_gemm;

extern "C" int pkcu_gemm_bias_swish(const float *A, const float *W, const float *bias, float *D,
                                    int M, int N, int K, pkcu_stream_t stream) {
  const char *what = "pkcu_gemm_bias_swish";
  int st = check(A, W, bias, D, M, N, K, what);
  if (st) return st;
  auto sd = strides<SwishGemm>(M, N, K);
  typename SwishGemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                     {M, N, K, 1},
                                     {A, get<0>(sd), W, get<1>(sd)},
                                     {{}, D, get<2>(sd), D, get<2>(sd)}};
  args.epilogue.thread.alpha = 1.0f;
  args.epilogue.thread.beta = 0.0f;
  args.epilogue.thread.bias_ptr = bias;
  return run<SwishGemm>(args, (cudaStream_t)stream, what);
}

extern "C" int pkcu_gemm_bias_residual(const float *A, const float *W, const float *bias, float *X,
                                       float scale, int M, int N, int K, pkcu_stream_t stream) {
  const char *what = "pkcu_gemm_bias_residual";
  int st = check(A, W, bias, X, M, N, K, what);
  if (st) return st;
  auto sd = strides<ResidualGemm>(M, N, K);
  typename ResidualGemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                        {M, N, K, 1},
                                        {A, get<0>(sd), W, get<1>(sd)},
                                        {{}, X, get<2>(sd), X, get<2>(sd)}};
  args.epilogue.thread.alpha = 1.0f;
  args.epilogue.thread.beta = 1.0f;
  args.epilogue.thread.bias_ptr = bias;
  args.epilogue.thread.activation.scale = scale;
  return run<ResidualGemm>(args, (cudaStream_t)stream, what);
}

// C[M, N] = A[M, K] B[K, N], row-major with packed rows (the library's own
// projections, pk_encoder_model.c). Returns PKCU_ERR_ARG when the shape does
// not suit the kernel (N or K not a multiple of 4, misaligned pointers) so the
// caller can take another GEMM.
extern "C" int pk_gemm_f32_rm(const float *A, const float *B, float *C, int M, int N, int K,
                              pkcu_stream_t stream) {
  const char *what = "pk_gemm_f32_rm";
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || N % 4 || K % 4 || !PK_ALIGNED16(A) ||
      !PK_ALIGNED16(B) || !PK_ALIGNED16(C))
    return PKCU_ERR_ARG;
  auto sd = strides<PlainGemm>(M, N, K);
  typename PlainGemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                     {M, N, K, 1},
                                     {A, get<0>(sd), B, get<1>(sd)},
                                     {{}, C, get<2>(sd), C, get<2>(sd)}};
  args.epilogue.thread.alpha = 1.0f;
  args.epilogue.thread.beta = 0.0f;
  return run<PlainGemm>(args, (cudaStream_t)stream, what);
}
