// k_preencode.cu -- pre-encode subsampling and input scaling (csrc/encoder.c:103-175,
// 578-593) for a batch of utterances: the non-GEMM steps as kernels, the two
// 1x1 convolutions and the output projection at GEMM hooks.
//
// Per utterance of T mel frames (mel [128, T], as the reference receives it):
//   conv0  1 -> 256, 3x3, stride 2, pad 1, + bias, ReLU   -> [256, H1, 64]
//   dw2    depthwise 3x3 stride 2 + bias                  -> [256, H2, 32]   (GEMM pw1 input)
//   pw1    1x1 conv = GEMM; + bias, ReLU
//   dw5    depthwise 3x3 stride 2 + bias                  -> [256, H3, 16]   (GEMM pw2 input)
//   pw2    1x1 conv = GEMM; + bias, ReLU
//   flat   [256, H3, 16] -> [H3, 4096]                                        (GEMM out input)
//   out    projection = GEMM; x = (proj + bias) * sqrt(1024)  -> [H3, 1024]   (the blocks' x)
// H1 = ceil(T/2), H2 = ceil(H1/2), H3 = ceil(H2/2). Every convolution output
// starts from its bias and adds tap products as fused multiply-adds in (kh, kw)
// order, taps outside the input skipped: the reference's pk_conv2d
// (csrc/tensor_ops.c:439-475) under its build's contraction, so the results are
// bit-identical to it.
//
// Layout: the [256, *, W] tensors are channel-major across the whole batch --
// row c holds every utterance's plane, utterance after utterance -- so each
// 1x1 convolution is one [256 x 256] x [256 x P] GEMM for the batch. The time-
// first tensors (flat, proj, x) are frames of every utterance, utterance after
// utterance, as the encoder blocks take x.
//
// conv0's output (the largest tensor of the stage, 256 x 64 floats per two mel
// frames) is never written: front_kernel computes it tile by tile in shared
// memory and applies dw2 there.
#include "pk_common.cuh"

namespace pk {

constexpr int PRE_C = 256, PRE_MELS = 128;
constexpr int PF_R2 = 4;                        // dw2 output rows per CTA
constexpr int PF_S1 = 2 * PF_R2 + 1;            // conv0 rows they read
constexpr int PF_MEL = 2 * PF_S1 + 1;           // mel frames those read
constexpr int PF_CG = 8;                        // channels per pass
constexpr int PF_THREADS = 256;

__device__ __forceinline__ int half_up(int h) { return (h + 1) >> 1; }   // (h + 2 - 3) / 2 + 1

// conv0 + bias + ReLU + dw2 + bias for dw2 rows [a, a + PF_R2) of one item.
__global__ void __launch_bounds__(PF_THREADS)
pre_front_kernel(const float *__restrict__ mel, const float *__restrict__ w0,
                 const float *__restrict__ b0, const float *__restrict__ w2,
                 const float *__restrict__ b2, float *__restrict__ s2d, SeqDev seq_mel,
                 SeqDev seq2, long long P2) {
  __shared__ float tile[PF_MEL][PRE_MELS];
  __shared__ float s1[PF_CG][PF_S1][64];
  const int item = blockIdx.y;
  const int T = seq_T(seq_mel, item);
  const int H1 = half_up(T), H2 = half_up(H1);
  const int a = blockIdx.x * PF_R2;
  if (a >= H2) return;
  const long long mel0 = seq_frame_off(seq_mel, item) * PRE_MELS;   // item's [128, T] block
  const long long q0 = seq_frame_off(seq2, item) * 32;              // item's first s2d column
  // mel frames t = 4a - 3 + j, j < PF_MEL, transposed into tile[j][m]
  const int t0 = 4 * a - 3;
  for (int e = threadIdx.x; e < PF_MEL * PRE_MELS; e += PF_THREADS) {
    const int m = e / PF_MEL, j = e - m * PF_MEL;
    const int t = t0 + j;
    tile[j][m] = (t >= 0 && t < T) ? __ldg(mel + mel0 + (long long)m * T + t) : 0.0f;
  }
  const int r1_0 = 2 * a - 1;   // conv0 row of s1[.][0]
  for (int cg = 0; cg < PRE_C; cg += PF_CG) {
    __syncthreads();   // tile loaded / previous pass's s1 consumed
    for (int e = threadIdx.x; e < PF_CG * PF_S1 * 64; e += PF_THREADS) {
      const int w1 = e & 63, i = (e >> 6) % PF_S1, cl = e / (64 * PF_S1);
      const int c = cg + cl, r1 = r1_0 + i;
      if (r1 < 0 || r1 >= H1) continue;   // never read below
      const float *wc = w0 + c * 9;
      float val = __ldg(b0 + c);
#pragma unroll
      for (int kh = 0; kh < 3; kh++) {
        const int t = 2 * r1 - 1 + kh;   // tile row 2i + kh
        if (t < 0 || t >= T) continue;
#pragma unroll
        for (int kw = 0; kw < 3; kw++) {
          const int m = 2 * w1 - 1 + kw;
          if (m >= 0 && m < PRE_MELS) val = fmaf(tile[2 * i + kh][m], __ldg(wc + kh * 3 + kw), val);
        }
      }
      s1[cl][i][w1] = val < 0.0f ? 0.0f : val;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < PF_CG * PF_R2 * 32; e += PF_THREADS) {
      const int ow = e & 31, r = (e >> 5) % PF_R2, cl = e / (32 * PF_R2);
      const int c = cg + cl, oh = a + r;
      if (oh >= H2) continue;
      const float *wc = w2 + c * 9;
      float val = __ldg(b2 + c);
#pragma unroll
      for (int kh = 0; kh < 3; kh++) {
        const int r1 = 2 * oh - 1 + kh;   // s1 row 2r + kh
        if (r1 < 0 || r1 >= H1) continue;
#pragma unroll
        for (int kw = 0; kw < 3; kw++) {
          const int w1 = 2 * ow - 1 + kw;
          if (w1 >= 0 && w1 < 64) val = fmaf(s1[cl][2 * r + kh][w1], __ldg(wc + kh * 3 + kw), val);
        }
      }
      s2d[(long long)c * P2 + q0 + oh * 32 + ow] = val;
    }
  }
}

// The item holding global row g of a sequence of per-item row counts.
__device__ __forceinline__ int seq_item_of(const SeqDev &s, long long g) {
  if (s.uniform_T > 0) return (int)(g / s.uniform_T);
  int lo = 0, hi = s.n_items;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(s.frame_off + mid) <= g) lo = mid; else hi = mid;
  }
  return lo;
}

// s3d[c, 16 g3 + ow] = b5[c] + taps of relu(y2 + b3) (dw5 on the pw1 output):
// one output per thread.
__global__ void __launch_bounds__(256)
pre_dw5_kernel(const float *__restrict__ y2, const float *__restrict__ b3,
               const float *__restrict__ w5, const float *__restrict__ b5, float *__restrict__ s3d,
               SeqDev seq2, SeqDev seq3, long long P2, long long P3) {
  const long long n = (long long)PRE_C * P3;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(e / P3);
    const long long q = e - (long long)c * P3;
    const long long g3 = q >> 4;
    const int ow = (int)(q & 15);
    const int item = seq_item_of(seq3, g3);
    const int oh = (int)(g3 - seq_frame_off(seq3, item));
    const int H2 = seq_T(seq2, item);
    const float *yc = y2 + (long long)c * P2 + seq_frame_off(seq2, item) * 32;
    const float bc = __ldg(b3 + c);
    const float *wc = w5 + c * 9;
    float val = __ldg(b5 + c);
#pragma unroll
    for (int kh = 0; kh < 3; kh++) {
      const int r2 = 2 * oh - 1 + kh;
      if (r2 < 0 || r2 >= H2) continue;
#pragma unroll
      for (int kw = 0; kw < 3; kw++) {
        const int w2 = 2 * ow - 1 + kw;
        if (w2 < 0 || w2 >= 32) continue;
        float v = __ldg(yc + r2 * 32 + w2) + bc;
        v = v < 0.0f ? 0.0f : v;
        val = fmaf(v, __ldg(wc + kh * 3 + kw), val);
      }
    }
    s3d[e] = val;
  }
}

// flat[g, 16c + w] = relu(y3[c, 16g + w] + b6[c]), four floats per thread.
__global__ void __launch_bounds__(256)
pre_flatten_kernel(const float *__restrict__ y3, const float *__restrict__ b6,
                   float *__restrict__ flat, long long rows, long long P3) {
  const long long n = rows * PRE_C * 4;   // float4s
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const long long g = e / (PRE_C * 4);
    const int r = (int)(e - g * PRE_C * 4), c = r >> 2, j = r & 3;
    const float bc = __ldg(b6 + c);
    float4 v = ldg4_stream(y3 + (long long)c * P3 + 16 * g + 4 * j);
    v = make_float4(v.x + bc, v.y + bc, v.z + bc, v.w + bc);
    v = make_float4(v.x < 0.0f ? 0.0f : v.x, v.y < 0.0f ? 0.0f : v.y, v.z < 0.0f ? 0.0f : v.z,
                    v.w < 0.0f ? 0.0f : v.w);
    st4(flat + g * (PRE_C * 16) + 16 * c + 4 * j, v);
  }
}

// x = (proj + bias) * sqrt(1024): the bias add of csrc/encoder.c:163-164, then
// the scaling of :582-586 (a power of two, exact).
__global__ void __launch_bounds__(256)
pre_out_kernel(const float *__restrict__ proj, const float *__restrict__ b, float *__restrict__ x,
               long long rows) {
  const long long n = rows * (PK_D / 4);
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const int d4 = (int)(e % (PK_D / 4));
    const float4 p = ldg4_stream(proj + 4 * e), bb = __ldg(reinterpret_cast<const float4 *>(b) + d4);
    st4(x + 4 * e, make_float4((p.x + bb.x) * 32.0f, (p.y + bb.y) * 32.0f, (p.z + bb.z) * 32.0f,
                               (p.w + bb.w) * 32.0f));
  }
}

static unsigned flat_grid(long long work) {
  long long g = (work + 255) / 256;
  const long long cap = (long long)pkcu_sm_count() * 8;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace pk

using namespace pk;

struct pkcu_pre_plan {
  pkcu_seq *mel, *rows2, *rows3;   // per item: T, H2, H3 (rows3 = the blocks' frames)
  long long P2, P3, frames;        // 32 x sum H2, 16 x sum H3, sum H3
};

extern "C" void pkcu_pre_plan_destroy(pkcu_pre_plan *p) {
  if (!p) return;
  pkcu_seq_destroy(p->mel);
  pkcu_seq_destroy(p->rows2);
  pkcu_seq_destroy(p->rows3);
  free(p);
}

extern "C" int pkcu_pre_plan_create(const int *mel_lengths, int n_items, pkcu_pre_plan **out) {
  if (!mel_lengths || n_items <= 0 || n_items > 65535 || !out)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_pre_plan_create: bad argument (1..65535 items)");
  *out = nullptr;
  for (int i = 0; i < n_items; i++)
    if (mel_lengths[i] <= 0)
      return pkcu_fail(PKCU_ERR_ARG, "pkcu_pre_plan_create: item %d has %d mel frames", i,
                       mel_lengths[i]);
  pkcu_pre_plan *p = (pkcu_pre_plan *)calloc(1, sizeof(*p));
  int *h2 = (int *)malloc(sizeof(int) * n_items), *h3 = (int *)malloc(sizeof(int) * n_items);
  if (!p || !h2 || !h3) {
    free(p); free(h2); free(h3);
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_pre_plan_create: host allocation");
  }
  for (int i = 0; i < n_items; i++) {
    const int a = (mel_lengths[i] + 1) / 2, b = (a + 1) / 2;
    h2[i] = b;
    h3[i] = (b + 1) / 2;
    p->P2 += 32LL * h2[i];
    p->P3 += 16LL * h3[i];
    p->frames += h3[i];
  }
  int st = pkcu_seq_create(mel_lengths, n_items, &p->mel);
  if (!st) st = pkcu_seq_create(h2, n_items, &p->rows2);
  if (!st) st = pkcu_seq_create(h3, n_items, &p->rows3);
  free(h2);
  free(h3);
  if (st) {
    pkcu_pre_plan_destroy(p);
    return st;
  }
  *out = p;
  return PKCU_OK;
}

extern "C" long long pkcu_pre_plan_p2(const pkcu_pre_plan *p) { return p ? p->P2 : 0; }
extern "C" long long pkcu_pre_plan_p3(const pkcu_pre_plan *p) { return p ? p->P3 : 0; }
extern "C" long long pkcu_pre_plan_frames(const pkcu_pre_plan *p) { return p ? p->frames : 0; }
extern "C" const pkcu_seq *pkcu_pre_plan_out_seq(const pkcu_pre_plan *p) {
  return p ? p->rows3 : nullptr;
}

extern "C" int pkcu_pre_encode(const float *mel, const pkcu_pre_params *prm,
                               const pkcu_pre_gemm_outputs *go, const pkcu_pre_gemm_inputs *gi,
                               float *x, const pkcu_pre_plan *plan, pkcu_gemm_hook hook,
                               void *hook_user, pkcu_stream_t stream) {
  if (!mel || !prm || !go || !gi || !x || !plan)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_pre_encode: NULL argument");
  const float *need[] = {prm->conv0_w, prm->conv0_b, prm->conv2_w, prm->conv2_b, prm->conv3_b,
                         prm->conv5_w, prm->conv5_b, prm->conv6_b, prm->out_b,
                         go->pw1, go->pw2, go->proj, gi->s2d, gi->s3d, gi->flat};
  for (const float *q : need)
    if (!q) return pkcu_fail(PKCU_ERR_ARG, "pkcu_pre_encode: NULL parameter or buffer");
  if (!PK_ALIGNED16(go->pw2) || !PK_ALIGNED16(go->proj) || !PK_ALIGNED16(gi->flat) ||
      !PK_ALIGNED16(x) || !PK_ALIGNED16(prm->out_b))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_pre_encode: pw2, proj, flat, x, out_b must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const SeqDev sm = plan->mel->dev, s2 = plan->rows2->dev, s3 = plan->rows3->dev;
  const unsigned tiles = (unsigned)((s2.max_T + PF_R2 - 1) / PF_R2);
  pre_front_kernel<<<dim3(tiles, (unsigned)sm.n_items), PF_THREADS, 0, s>>>(
      mel, prm->conv0_w, prm->conv0_b, prm->conv2_w, prm->conv2_b, gi->s2d, sm, s2, plan->P2);
  int st = pkcu_launch_status("pkcu_pre_encode: conv0 + dw2");
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_PRE_PW1, stream);
  if (st) return st;
  pre_dw5_kernel<<<flat_grid((long long)PRE_C * plan->P3), 256, 0, s>>>(
      go->pw1, prm->conv3_b, prm->conv5_w, prm->conv5_b, gi->s3d, s2, s3, plan->P2, plan->P3);
  st = pkcu_launch_status("pkcu_pre_encode: dw5");
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_PRE_PW2, stream);
  if (st) return st;
  pre_flatten_kernel<<<flat_grid(plan->frames * PRE_C * 4), 256, 0, s>>>(
      go->pw2, prm->conv6_b, gi->flat, plan->frames, plan->P3);
  st = pkcu_launch_status("pkcu_pre_encode: flatten");
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_PRE_OUT, stream);
  if (st) return st;
  pre_out_kernel<<<flat_grid(plan->frames * (PK_D / 4)), 256, 0, s>>>(go->proj, prm->out_b, x,
                                                                      plan->frames);
  return pkcu_launch_status("pkcu_pre_encode: out");
}
