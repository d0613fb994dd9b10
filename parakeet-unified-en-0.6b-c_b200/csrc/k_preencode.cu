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
// frames) is never written: pre_front_kernel computes it row by row in
// registers and feeds each value straight into the dw2 accumulators.
#include "pk_common.cuh"

namespace pk {

constexpr int PRE_C = 256, PRE_MELS = 128;
constexpr int PF_R2 = 16;                       // dw2 output rows per CTA
constexpr int PF_MEL = 4 * PF_R2 + 3;           // mel frames their conv0 rows read
constexpr int PF_LD = 132;                      // float2 per staged frame: mel bin m at m + 4
constexpr int PF_THREADS = 256;                 // 64 channel pairs x 4 column quarters

__device__ __forceinline__ int half_up(int h) { return (h + 1) >> 1; }   // (h + 2 - 3) / 2 + 1

__device__ __forceinline__ float relu1(float v) { return v < 0.0f ? 0.0f : v; }

// One conv0 output row (staged-frame row pair 2 li .. 2 li + 2), + bias,
// ReLU, for this thread's channel pair and column quarter q, each value fed at
// once to the dw2 accumulators of that quarter (dw2 columns 8q .. 8q + 7):
//   MODE 1: row 2 oh      -> tap row kh = 1 of dw2 row oh (A)
//   MODE 2: row 2 oh + 1  -> kh = 2 of row oh (A) and kh = 0 of row oh + 1 (B)
// Quarter q produces conv0 columns 16q - 1 .. 16q + 15 (column -1 does not
// exist). Columns are visited left to right and rows top to bottom, so every
// output's taps arrive in the reference's (kh, kw) order. With EDGE, tap rows
// outside the mel frames are skipped as the reference skips them.
template <int MODE, bool EDGE>
__device__ __forceinline__ void pf_row(const float2 (*__restrict__ tile)[PF_LD], int li, int t0,
                                       int T, int q, const float2 (&w0)[9], float2 b0,
                                       const float2 (&w2)[9], float2 (&A)[8], float2 (&B)[8]) {
  bool ok[3];
  float2 cm[3], c0[3], c1[3];
#pragma unroll
  for (int kh = 0; kh < 3; kh++) {
    const int t = t0 + 2 * li + kh;
    ok[kh] = !EDGE || (t >= 0 && t < T);
    const float2 *row = tile[2 * li + kh];
    cm[kh] = row[32 * q + 1];                                          // mel bin 32q - 3
    const float4 v = *reinterpret_cast<const float4 *>(row + 32 * q + 2);   // bins 32q - 2, 32q - 1
    c0[kh] = make_float2(v.x, v.y);
    c1[kh] = make_float2(v.z, v.w);
  }
  constexpr int KA = MODE == 1 ? 3 : 6;   // tap row of A
#pragma unroll
  for (int u = 0; u < 17; u++) {
    if (u > 0 || q > 0) {                 // conv0 column w1 = 16q - 1 + u exists
      float2 s = b0;
#pragma unroll
      for (int kh = 0; kh < 3; kh++) {
        if (!ok[kh]) continue;
        if (u != 1 || q > 0) s = fma2(cm[kh], w0[kh * 3 + 0], s);   // mel bin 2 w1 - 1 >= 0
        s = fma2(c0[kh], w0[kh * 3 + 1], s);
        s = fma2(c1[kh], w0[kh * 3 + 2], s);
      }
      s = make_float2(relu1(s.x), relu1(s.y));
      const int v = u - 1;                // column within the quarter's 16
      if (v >= 0 && (v & 1) == 0) {       // even: kw = 1 of dw2 column v / 2
        A[v / 2] = fma2(s, w2[KA + 1], A[v / 2]);
        if (MODE == 2) B[v / 2] = fma2(s, w2[1], B[v / 2]);
      } else {                            // odd: kw = 2 of (v - 1) / 2, kw = 0 of (v + 1) / 2
        if (v >= 1) {
          A[(v - 1) / 2] = fma2(s, w2[KA + 2], A[(v - 1) / 2]);
          if (MODE == 2) B[(v - 1) / 2] = fma2(s, w2[2], B[(v - 1) / 2]);
        }
        if (v + 1 < 16) {
          A[(v + 1) / 2] = fma2(s, w2[KA + 0], A[(v + 1) / 2]);
          if (MODE == 2) B[(v + 1) / 2] = fma2(s, w2[0], B[(v + 1) / 2]);
        }
      }
    }
    if (u + 1 < 17) {                     // slide to column w1 + 1: bins 2 w1 + 2, 2 w1 + 3
#pragma unroll
      for (int kh = 0; kh < 3; kh++) {
        cm[kh] = c1[kh];
        const float4 v =
            *reinterpret_cast<const float4 *>(tile[2 * li + kh] + 32 * q + 2 * u + 4);
        c0[kh] = make_float2(v.x, v.y);
        c1[kh] = make_float2(v.z, v.w);
      }
    }
  }
}

constexpr int PF_SLD = 36;   // floats per channel row of the output stage (32 + pad)
constexpr size_t PF_SMEM = sizeof(float2) * PF_MEL * PF_LD + sizeof(float) * 128 * PF_SLD;

// dw2 row oh of this CTA's 128 channels, written through the shared stage so
// that every 8 lanes store one whole 128-byte channel row: a thread's own
// outputs (8 columns x 2 channels) would otherwise be 32 scattered 16-byte
// pieces per warp store.
__device__ __forceinline__ void pf_store(float *__restrict__ stage, float *__restrict__ s2d,
                                         long long P2, long long col0, int q, int cp,
                                         const float2 (&acc)[8]) {
  __syncthreads();   // the previous row's copy-out has read the stage
  float *r0 = stage + cp * PF_SLD + 8 * q, *r1 = stage + (64 + cp) * PF_SLD + 8 * q;
  *reinterpret_cast<float4 *>(r0) = make_float4(acc[0].x, acc[1].x, acc[2].x, acc[3].x);
  *reinterpret_cast<float4 *>(r0 + 4) = make_float4(acc[4].x, acc[5].x, acc[6].x, acc[7].x);
  *reinterpret_cast<float4 *>(r1) = make_float4(acc[0].y, acc[1].y, acc[2].y, acc[3].y);
  *reinterpret_cast<float4 *>(r1 + 4) = make_float4(acc[4].y, acc[5].y, acc[6].y, acc[7].y);
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int e = threadIdx.x + i * PF_THREADS, r = e >> 3, j = e & 7;
    const int c = (r < 64 ? 0 : 64) + 64 * blockIdx.z + r;   // stage row r -> channel
    st4(s2d + (long long)c * P2 + col0 + 4 * j,
        *reinterpret_cast<const float4 *>(stage + r * PF_SLD + 4 * j));
  }
}

// conv0 rows 2a - 1 .. 2(a + nrows) - 1 in order: odd rows finish the previous
// dw2 row and start the next, even rows add the middle tap row.
template <bool EDGE>
__device__ __forceinline__ void pf_tile(const float2 (*__restrict__ tile)[PF_LD], int a, int nrows,
                                        int T, int H1, int q, const float2 (&w0)[9], float2 b0,
                                        const float2 (&w2)[9], float2 b2, float *__restrict__ stage,
                                        float *__restrict__ s2d, long long P2, long long q0,
                                        int cp) {
  const int t0 = 4 * a - 3;
  float2 prev[8], cur[8];
#pragma unroll
  for (int j = 0; j < 8; j++) prev[j] = b2;
  for (int k = 0; k <= nrows; k++) {
    const int oh = a + k;
#pragma unroll
    for (int j = 0; j < 8; j++) cur[j] = b2;
    if (!EDGE || (2 * oh - 1 >= 0 && 2 * oh - 1 < H1))
      pf_row<2, EDGE>(tile, 2 * k, t0, T, q, w0, b0, w2, prev, cur);
    if (k < nrows) pf_row<1, EDGE>(tile, 2 * k + 1, t0, T, q, w0, b0, w2, cur, cur);
    if (k > 0) pf_store(stage, s2d, P2, q0 + 32LL * (oh - 1), q, cp, prev);
#pragma unroll
    for (int j = 0; j < 8; j++) prev[j] = cur[j];
  }
}

// conv0 (1 -> 256, 3x3 stride 2) + bias + ReLU + dw2 (depthwise 3x3 stride 2)
// + bias for dw2 rows [a, a + PF_R2) of one item and channels c, c + 128 for
// c in [64 z, 64 z + 64) (z = blockIdx.z). conv0's output never leaves
// registers. Thread = (column quarter, channel pair c, c + 128): warps 2q and
// 2q + 1 take quarter q, so every lane of a warp reads the same staged mel
// value (a shared-memory broadcast) and the pair shares it through
// fma.rn.f32x2. Staged frames hold each mel bin twice (v, v) for that.
__global__ void __launch_bounds__(PF_THREADS, 2)
pre_front_kernel(const float *__restrict__ mel, const float *__restrict__ w0g,
                 const float *__restrict__ b0g, const float *__restrict__ w2g,
                 const float *__restrict__ b2g, float *__restrict__ s2d, SeqDev seq_mel,
                 SeqDev seq2, long long P2) {
  extern __shared__ float4 pf_smem4[];
  float2 (*tile)[PF_LD] = reinterpret_cast<float2 (*)[PF_LD]>(pf_smem4);
  float *stage = reinterpret_cast<float *>(tile + PF_MEL);
  const int item = blockIdx.y;
  const int T = seq_T(seq_mel, item);
  const int H1 = half_up(T), H2 = half_up(H1);
  const int a = blockIdx.x * PF_R2;
  if (a >= H2) return;
  const int nrows = min(PF_R2, H2 - a);
  const long long mel0 = seq_frame_off(seq_mel, item) * PRE_MELS;   // item's [128, T] block
  const long long q0 = seq_frame_off(seq2, item) * 32;              // item's first s2d column
  const int t0 = 4 * a - 3;
  constexpr int BATCH = 5;   // loads in flight per thread
  for (int e0 = threadIdx.x; e0 < PF_MEL * PRE_MELS; e0 += BATCH * PF_THREADS) {
    float v[BATCH];
#pragma unroll
    for (int b = 0; b < BATCH; b++) {
      const int e = e0 + b * PF_THREADS, m = e / PF_MEL, t = t0 + e - m * PF_MEL;
      v[b] = (e < PF_MEL * PRE_MELS && t >= 0 && t < T)
                 ? __ldg(mel + mel0 + (long long)m * T + t) : 0.0f;
    }
#pragma unroll
    for (int b = 0; b < BATCH; b++) {
      const int e = e0 + b * PF_THREADS, m = e / PF_MEL;
      if (e < PF_MEL * PRE_MELS) tile[e - m * PF_MEL][m + 4] = make_float2(v[b], v[b]);
    }
  }
  const int warp = threadIdx.x >> 5, q = warp >> 1;
  const int cp = (warp & 1) * 32 + (threadIdx.x & 31);   // channel pair within the CTA
  const int c_lo = 64 * blockIdx.z + cp, c_hi = c_lo + 128;
  float2 w0[9], w2[9];
#pragma unroll
  for (int k = 0; k < 9; k++) {
    w0[k] = make_float2(__ldg(w0g + c_lo * 9 + k), __ldg(w0g + c_hi * 9 + k));
    w2[k] = make_float2(__ldg(w2g + c_lo * 9 + k), __ldg(w2g + c_hi * 9 + k));
  }
  const float2 b0 = make_float2(__ldg(b0g + c_lo), __ldg(b0g + c_hi));
  const float2 b2 = make_float2(__ldg(b2g + c_lo), __ldg(b2g + c_hi));
  __syncthreads();
  if (a == 0 || 4 * (a + nrows) > T)
    pf_tile<true>(tile, a, nrows, T, H1, q, w0, b0, w2, b2, stage, s2d, P2, q0, cp);
  else
    pf_tile<false>(tile, a, nrows, T, H1, q, w0, b0, w2, b2, stage, s2d, P2, q0, cp);
}

constexpr int P5_R3 = 64;                  // dw5 output rows per CTA
constexpr int P5_IN = 2 * P5_R3 + 1;       // input rows they read
constexpr int P5_LD = 32;                  // floats per staged row

// s3d[c, item, oh, ow] = b5[c] + taps of relu(y2 + b3[c]) (dw5 applied to the
// pw1 product): one CTA per (64 output rows, channel, item). The input rows
// are contiguous in y2's channel row: they arrive as 16-byte asynchronous
// copies (the whole slab in flight at once), 16-byte chunk k of staged row R
// at chunk k ^ ((R >> 1) & 1), so that the two output rows of a quarter-warp
// read disjoint banks. Thread = output row ol (tid / 4) x output columns
// ow = 4q..4q+3 (q = tid % 4): per input row the two float4 of columns
// 8q..8q+7 and the column 8q - 1, bias + ReLU applied as they are read; each
// output's taps in the reference's order (kh, then kw), column -1 being the
// zero padding.
__global__ void __launch_bounds__(256)
pre_dw5_kernel(const float *__restrict__ y2, const float *__restrict__ b3,
               const float *__restrict__ w5, const float *__restrict__ b5, float *__restrict__ s3d,
               SeqDev seq2, SeqDev seq3, long long P2, long long P3) {
  __shared__ __align__(16) float tile[P5_IN * P5_LD];
  const int c = blockIdx.y, item = blockIdx.z;
  const int H2 = seq_T(seq2, item), H3 = seq_T(seq3, item);
  const int o0 = blockIdx.x * P5_R3;
  if (o0 >= H3) return;
  const int nout = min(P5_R3, H3 - o0);
  const int r0 = 2 * o0 - 1;                                 // input row of staged row 0
  const int rlo = max(r0, 0), rhi = min(2 * (o0 + nout) - 1, H2 - 1);
  const float *src = y2 + (long long)c * P2 + seq_frame_off(seq2, item) * 32;
  for (int e = threadIdx.x; e < (rhi - rlo + 1) * 8; e += 256) {
    const int r = rlo + (e >> 3), k = e & 7, R = r - r0;
    cp_async16(tile + R * P5_LD + 4 * (k ^ ((R >> 1) & 1)), src + (long long)r * 32 + 4 * k);
  }
  cp_async_commit();
  const float bc = __ldg(b3 + c);
  float w[9];
#pragma unroll
  for (int k = 0; k < 9; k++) w[k] = __ldg(w5 + c * 9 + k);
  const float bias = __ldg(b5 + c);
  cp_async_wait<0>();
  __syncthreads();
  const int ol = threadIdx.x >> 2, q = threadIdx.x & 3, oh = o0 + ol;
  if (ol >= nout) return;
  float acc0 = bias, acc1 = bias, acc2 = bias, acc3 = bias;
#pragma unroll
  for (int kh = 0; kh < 3; kh++) {
    const int r = 2 * oh - 1 + kh;
    if (r < 0 || r >= H2) continue;
    const int R = 2 * ol + kh, sw = (R >> 1) & 1;
    const float *row = tile + R * P5_LD;
    float4 a = ld4(row + 4 * ((2 * q) ^ sw)), b = ld4(row + 4 * ((2 * q + 1) ^ sw));
    a = make_float4(relu1(a.x + bc), relu1(a.y + bc), relu1(a.z + bc), relu1(a.w + bc));
    b = make_float4(relu1(b.x + bc), relu1(b.y + bc), relu1(b.z + bc), relu1(b.w + bc));
    const float w0 = w[kh * 3 + 0], w1 = w[kh * 3 + 1], w2 = w[kh * 3 + 2];
    if (q > 0) acc0 = fmaf(relu1(row[4 * ((2 * q - 1) ^ sw) + 3] + bc), w0, acc0);
    acc0 = fmaf(a.x, w1, acc0);
    acc0 = fmaf(a.y, w2, acc0);
    acc1 = fmaf(a.y, w0, acc1);
    acc1 = fmaf(a.z, w1, acc1);
    acc1 = fmaf(a.w, w2, acc1);
    acc2 = fmaf(a.w, w0, acc2);
    acc2 = fmaf(b.x, w1, acc2);
    acc2 = fmaf(b.y, w2, acc2);
    acc3 = fmaf(b.y, w0, acc3);
    acc3 = fmaf(b.z, w1, acc3);
    acc3 = fmaf(b.w, w2, acc3);
  }
  float *o = s3d + (long long)c * P3 + (seq_frame_off(seq3, item) + oh) * 16 + 4 * q;
  o[0] = acc0;
  o[1] = acc1;
  o[2] = acc2;
  o[3] = acc3;
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
  if (!PK_ALIGNED16(go->pw1) || !PK_ALIGNED16(go->pw2) || !PK_ALIGNED16(go->proj) ||
      !PK_ALIGNED16(gi->s2d) || !PK_ALIGNED16(gi->flat) || !PK_ALIGNED16(x) ||
      !PK_ALIGNED16(prm->out_b))
    return pkcu_fail(PKCU_ERR_ARG,
                     "pkcu_pre_encode: pw1, pw2, proj, s2d, flat, x, out_b must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const SeqDev sm = plan->mel->dev, s2 = plan->rows2->dev, s3 = plan->rows3->dev;
  const unsigned tiles = (unsigned)((s2.max_T + PF_R2 - 1) / PF_R2);
  static int optin[64];
  smem_optin(pre_front_kernel, PF_SMEM, optin);
  pre_front_kernel<<<dim3(tiles, (unsigned)sm.n_items, 2), PF_THREADS, PF_SMEM, s>>>(
      mel, prm->conv0_w, prm->conv0_b, prm->conv2_w, prm->conv2_b, gi->s2d, sm, s2, plan->P2);
  int st = pkcu_launch_status("pkcu_pre_encode: conv0 + dw2");
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_PRE_PW1, stream);
  if (st) return st;
  const unsigned tiles3 = (unsigned)((s3.max_T + P5_R3 - 1) / P5_R3);
  pre_dw5_kernel<<<dim3(tiles3, PRE_C, (unsigned)s3.n_items), 256, 0, s>>>(
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
