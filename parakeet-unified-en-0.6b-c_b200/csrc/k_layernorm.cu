// k_layernorm.cu -- LayerNorm and the ops fused around it.
//
// Reference: pk_layer_norm / _rows / _rows_inplace (csrc/tensor_ops.c:151-280):
// mean, biased variance of (x - mean), inv_std = 1/sqrtf(var + 1e-5),
// out = fma((x - mean) * inv_std, gamma, beta). The reductions run in a
// different order than the reference's 8-lane AVX2 sums (compared within
// 2e-6 abs / 1e-5 rel); everything after the two sums is the same sequence of
// IEEE operations.
//
// D = 1024 rows (every LN of the encoder, csrc/encoder.c:191,308,447,490) take
// the register path: one warp per row, each lane holding 8 float4 (columns
// 4*(lane + 32j)), so a row is read once and written once: 8 bytes per element
// of HBM traffic. Other widths or unaligned pointers take a CTA-per-row
// kernel that re-reads the row from L1/L2.
//
// Fusions (each saves a full read+write of the [frames, 1024] residual stream):
//   residual + LN         x += a*(y+bias); ln = LN(x)                 (FF1 -> MHSA)
//   residual + LN + LN    x = LN_out(x + a*(y+bias)); ln = LN_ff1'(x) (FF2 -> next block)
//   residual + LN + T     x += y + bias; cf = LN(x)^T per item        (MHSA -> conv)
//   T-add + LN            x[t,d] += y[d,t] + bias[d]; ln = LN(x)      (conv -> FF2)
#include <math.h>

#include "pk_common.cuh"

namespace pk {

constexpr int LN_VEC = PK_D / 128;      // float4 per lane for a 1024-wide row
constexpr int LN_ROWS_PER_CTA = 8;      // one warp per row, 256 threads
constexpr int LT_STRIDE = PK_D + 4;     // smem row stride (keeps float4 alignment)
// The transposing kernels take TT frames per CTA, one warp per frame: 32
// (128 KB tile, one CTA per SM) when the batch gives every SM a tile, else 16
// (64 KB, two per SM), so that short batches still spread over the SMs.
template <int TT>
constexpr size_t lt_smem() { return sizeof(float) * TT * LT_STRIDE; }

// Normalises one 1024-wide row held in a warp's registers.
__device__ __forceinline__ void ln_regs(float4 (&v)[LN_VEC], const float *__restrict__ g,
                                        const float *__restrict__ b, int lane) {
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < LN_VEC; j++) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  s = warp_sum(s);
  const float mean = s / (float)PK_D;
  float q = 0.0f;
#pragma unroll
  for (int j = 0; j < LN_VEC; j++) {
    float d;
    d = v[j].x - mean; q = fmaf(d, d, q);
    d = v[j].y - mean; q = fmaf(d, d, q);
    d = v[j].z - mean; q = fmaf(d, d, q);
    d = v[j].w - mean; q = fmaf(d, d, q);
  }
  q = warp_sum(q);
  const float inv = 1.0f / sqrtf(q / (float)PK_D + 1e-5f);
#pragma unroll
  for (int j = 0; j < LN_VEC; j++) {
    const int c = 4 * (lane + 32 * j);
    const float4 gg = __ldg(reinterpret_cast<const float4 *>(g + c));
    const float4 bb = __ldg(reinterpret_cast<const float4 *>(b + c));
    v[j].x = fmaf((v[j].x - mean) * inv, gg.x, bb.x);
    v[j].y = fmaf((v[j].y - mean) * inv, gg.y, bb.y);
    v[j].z = fmaf((v[j].z - mean) * inv, gg.z, bb.z);
    v[j].w = fmaf((v[j].w - mean) * inv, gg.w, bb.w);
  }
}

__device__ __forceinline__ void load_row(float4 (&v)[LN_VEC], const float *r, int lane) {
#pragma unroll
  for (int j = 0; j < LN_VEC; j++) v[j] = ld4(r + 4 * (lane + 32 * j));
}

__device__ __forceinline__ void store_row(float *r, const float4 (&v)[LN_VEC], int lane) {
#pragma unroll
  for (int j = 0; j < LN_VEC; j++) st4(r + 4 * (lane + 32 * j), v[j]);
}

// v += alpha * (y + bias), the residual add of csrc/encoder.c:202-216 / :422-434
// after the GEMM-output bias add (pk_bias_add): (y + bias) rounds first, then
// one fused multiply-add (exact for alpha = 0.5 and 1).
__device__ __forceinline__ void add_residual(float4 (&v)[LN_VEC], const float *yr,
                                             const float *bias, float alpha, int lane) {
#pragma unroll
  for (int j = 0; j < LN_VEC; j++) {
    const int c = 4 * (lane + 32 * j);
    float4 t = ldg4_stream(yr + c);
    if (bias) t = add4(t, __ldg(reinterpret_cast<const float4 *>(bias + c)));
    v[j].x = fmaf(t.x, alpha, v[j].x);
    v[j].y = fmaf(t.y, alpha, v[j].y);
    v[j].z = fmaf(t.z, alpha, v[j].z);
    v[j].w = fmaf(t.w, alpha, v[j].w);
  }
}

enum { LN_PLAIN = 0, LN_RESID = 1, LN_RESID2 = 2 };

// MODE LN_PLAIN : out = LN(x; g1,b1)                         (out may be x)
// MODE LN_RESID : x += alpha*(y+bias); out = LN(x; g1,b1)
// MODE LN_RESID2: x = LN(x + alpha*(y+bias); g1,b1); out = LN(x; g2,b2) if g2
// (LN_RESID2 held to 64 registers, four CTAs = 32 warps per SM: 0.98 of the copy
// bandwidth against 0.92-0.93 at 75 registers and three CTAs, despite a few
// spilled bytes; residual + LN already runs at the copy bandwidth unbounded.)
template <int MODE>
__global__ void __launch_bounds__(32 * LN_ROWS_PER_CTA, MODE == LN_RESID2 ? 4 : 1)
ln1024_kernel(float *x, const float *__restrict__ y, const float *__restrict__ bias, float alpha,
              const float *__restrict__ g1, const float *__restrict__ b1,
              const float *__restrict__ g2, const float *__restrict__ b2, float *out,
              long long n_rows) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * LN_ROWS_PER_CTA + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  float *xr = x + row * PK_D;
  float4 v[LN_VEC];
  load_row(v, xr, lane);
  if (MODE != LN_PLAIN) {
    add_residual(v, y + row * PK_D, bias, alpha, lane);
    if (MODE == LN_RESID) store_row(xr, v, lane);
  }
  ln_regs(v, g1, b1, lane);
  if (MODE == LN_RESID2) {
    store_row(xr, v, lane);
    if (g2 == nullptr) return;
    ln_regs(v, g2, b2, lane);
  }
  store_row(out + row * PK_D, v, lane);
}

// Any width, any alignment: one CTA per row, three passes over the row.
// Columns below 8*floor(D/8) use the fused form of the reference's vector
// body, the rest its scalar tail ((x-mean)*inv*g + b, :215-216).
__global__ void __launch_bounds__(256)
ln_generic_kernel(const float *x, const float *__restrict__ g, const float *__restrict__ b,
                  float *out, int D) {
  __shared__ float red[33];
  const float *xr = x + (long long)blockIdx.x * D;
  float *orow = out + (long long)blockIdx.x * D;
  float s = 0.0f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) s += xr[i];
  s = block_sum(s, red);
  const float mean = s / (float)D;
  float q = 0.0f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float d = xr[i] - mean;
    q = fmaf(d, d, q);
  }
  q = block_sum(q, red);
  const float inv = 1.0f / sqrtf(q / (float)D + 1e-5f);
  const int D8 = D & ~7;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    const float xn = (xr[i] - mean) * inv;
    orow[i] = (i < D8) ? fmaf(xn, g[i], b[i]) : xn * g[i] + b[i];
  }
}

// LayerNorm of frames [t0, t0 + TT) of one item, optionally after the attention
// residual, written channel-first: cf[d, t] per item [D, T_b]
// (csrc/encoder.c:447-452). The normalised rows are staged in shared memory
// and leave as 128-byte runs of 32 consecutive frames per channel: one warp
// store per channel. (Channel-first runs of 16 frames moved measurably less:
// 3.9 against 5.1 TB/s for the bare transposed write of 256 x 375 frames.
// Persistent forms of both transposing kernels, one CTA per SM with the next
// tile's rows prefetched into L2, measured slower still: 0.64 / 0.60 of the
// copy bandwidth against 0.85 / 0.84. So did two cures for the 4-way bank
// conflict of the column reads (row stride 1028): warp instructions over 4
// channels x 8 frames (0.80 / 0.44: 32-byte pieces per instruction), and rows
// held as scalars with an odd stride (0.80 / 0.86). A tile without any bank
// conflict (16-byte chunks at chunk index q ^ (row & 7), each lane moving a
// float4 of four channels of one frame, still 128-byte runs per warp store)
// gained nothing either: 0.87 / 0.82 against 0.87 / 0.84 on the same box. Nor
// did two 512-thread CTAs per tile as a thread-block cluster (16 frames in each
// CTA's 64 KB, two CTAs per SM, each CTA moving half the channels of all 32
// frames through distributed shared memory): 0.35 / 0.44, the 4-byte accesses
// to the peer's shared memory costing far more than the overlap gained.
// Requesting transpose-add's x row before its channel-first reads measured
// 0.71 against 0.86.)
template <int TT, bool RESID>
__global__ void __launch_bounds__(32 * TT, 32 / TT)
ln_transpose_kernel(float *x, const float *__restrict__ y, const float *__restrict__ bias,
                    float alpha, const float *__restrict__ g, const float *__restrict__ b,
                    float *__restrict__ cf, SeqDev seq) {
  extern __shared__ float4 lt_smem4[];
  float *tile = reinterpret_cast<float *>(lt_smem4);
  const int item = blockIdx.y;
  const int T = seq_T(seq, item);
  const int t0 = blockIdx.x * TT;
  if (t0 >= T) return;
  const int nrows = min(TT, T - t0);
  const long long f0 = seq_frame_off(seq, item);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < nrows) {
    const long long row = f0 + t0 + warp;
    float *xr = x + row * PK_D;
    float4 v[LN_VEC];
    load_row(v, xr, lane);
    if (RESID) {
      add_residual(v, y + row * PK_D, bias, alpha, lane);
      store_row(xr, v, lane);
    }
    ln_regs(v, g, b, lane);
#pragma unroll
    for (int j = 0; j < LN_VEC; j++)
      st4(tile + warp * LT_STRIDE + 4 * (lane + 32 * j), v[j]);
  }
  __syncthreads();
  const int t = threadIdx.x & (TT - 1), dsub = threadIdx.x / TT;
  if (t < nrows) {
    float *dst = cf + f0 * PK_D + t0 + t;
    const float *src = tile + t * LT_STRIDE;
#pragma unroll 8
    for (int d = dsub; d < PK_D; d += 32) dst[(long long)d * T] = src[d];
  }
}

// Conv-module residual x[t,d] += y[d,t] + bias[d] (csrc/encoder.c:475-477,
// y per item [D, T_b] with the pointwise bias of csrc/tensor_ops.c:585-589),
// optionally followed by the FF2 LayerNorm of the updated rows.
template <int TT, bool WITH_LN>
__global__ void __launch_bounds__(32 * TT, 32 / TT)
transpose_add_kernel(float *x, const float *__restrict__ y, const float *__restrict__ bias,
                     const float *__restrict__ g, const float *__restrict__ b,
                     float *__restrict__ ln, SeqDev seq) {
  extern __shared__ float4 lt_smem4[];
  float *tile = reinterpret_cast<float *>(lt_smem4);
  const int item = blockIdx.y;
  const int T = seq_T(seq, item);
  const int t0 = blockIdx.x * TT;
  if (t0 >= T) return;
  const int nrows = min(TT, T - t0);
  const long long f0 = seq_frame_off(seq, item);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    const int t = threadIdx.x & (TT - 1), dsub = threadIdx.x / TT;
    if (t < nrows) {
      const float *src = y + f0 * PK_D + t0 + t;
      float *dst = tile + t * LT_STRIDE;
#pragma unroll 8
      for (int d = dsub; d < PK_D; d += 32) dst[d] = __ldcs(src + (long long)d * T);
    }
  }
  __syncthreads();
  if (warp >= nrows) return;
  const long long row = f0 + t0 + warp;
  float *xr = x + row * PK_D;
  float4 v[LN_VEC];
  load_row(v, xr, lane);
#pragma unroll
  for (int j = 0; j < LN_VEC; j++) {
    const int c = 4 * (lane + 32 * j);
    float4 t = *reinterpret_cast<const float4 *>(tile + warp * LT_STRIDE + c);
    if (bias) t = add4(t, __ldg(reinterpret_cast<const float4 *>(bias + c)));
    v[j] = add4(v[j], t);
  }
  store_row(xr, v, lane);
  if (WITH_LN) {
    ln_regs(v, g, b, lane);
    store_row(ln + row * PK_D, v, lane);
  }
}

static int g_lt_flags[8][64];

static unsigned ln_grid(long long n_rows) {
  return (unsigned)((n_rows + LN_ROWS_PER_CTA - 1) / LN_ROWS_PER_CTA);
}

}  // namespace pk

using namespace pk;

extern "C" int pkcu_layer_norm_rows(const float *x, const float *gamma, const float *beta,
                                    float *out, int n_rows, int D, pkcu_stream_t stream) {
  if (!x || !gamma || !beta || !out || n_rows < 0 || D <= 0)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_layer_norm_rows: bad argument");
  if (n_rows == 0) return PKCU_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (D == PK_D && PK_ALIGNED16(x) && PK_ALIGNED16(gamma) && PK_ALIGNED16(beta) &&
      PK_ALIGNED16(out)) {
    ln1024_kernel<LN_PLAIN><<<ln_grid(n_rows), 32 * LN_ROWS_PER_CTA, 0, s>>>(
        const_cast<float *>(x), nullptr, nullptr, 0.0f, gamma, beta, nullptr, nullptr, out,
        n_rows);
  } else {
    ln_generic_kernel<<<n_rows, 256, 0, s>>>(x, gamma, beta, out, D);
  }
  return pkcu_launch_status("pkcu_layer_norm_rows");
}

extern "C" int pkcu_residual_layer_norm(float *x, const float *y, const float *bias, float alpha,
                                        const float *gamma, const float *beta, float *ln,
                                        int n_rows, pkcu_stream_t stream) {
  if (!x || !y || !gamma || !beta || !ln || n_rows < 0)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_residual_layer_norm: bad argument");
  if (!PK_ALIGNED16(x) || !PK_ALIGNED16(y) || !PK_ALIGNED16(gamma) || !PK_ALIGNED16(beta) ||
      !PK_ALIGNED16(ln) || (bias && !PK_ALIGNED16(bias)))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_residual_layer_norm: pointers must be 16-byte aligned");
  if (n_rows == 0) return PKCU_OK;
  ln1024_kernel<LN_RESID><<<ln_grid(n_rows), 32 * LN_ROWS_PER_CTA, 0, (cudaStream_t)stream>>>(
      x, y, bias, alpha, gamma, beta, nullptr, nullptr, ln, n_rows);
  return pkcu_launch_status("pkcu_residual_layer_norm");
}

extern "C" int pkcu_residual_layer_norm2(float *x, const float *y, const float *bias,
                                         float alpha, const float *g_out, const float *b_out,
                                         const float *g_next, const float *b_next,
                                         float *ln_next, int n_rows, pkcu_stream_t stream) {
  if (!x || !y || !g_out || !b_out || n_rows < 0 || (g_next && (!b_next || !ln_next)))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_residual_layer_norm2: bad argument");
  if (!PK_ALIGNED16(x) || !PK_ALIGNED16(y) || !PK_ALIGNED16(g_out) || !PK_ALIGNED16(b_out) ||
      (bias && !PK_ALIGNED16(bias)) ||
      (g_next && (!PK_ALIGNED16(g_next) || !PK_ALIGNED16(b_next) || !PK_ALIGNED16(ln_next))))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_residual_layer_norm2: pointers must be 16-byte aligned");
  if (n_rows == 0) return PKCU_OK;
  ln1024_kernel<LN_RESID2><<<ln_grid(n_rows), 32 * LN_ROWS_PER_CTA, 0, (cudaStream_t)stream>>>(
      x, y, bias, alpha, g_out, b_out, g_next, b_next, ln_next, n_rows);
  return pkcu_launch_status("pkcu_residual_layer_norm2");
}

static int check_seq_tile(const pkcu_seq *seq, const char *what) {
  if (!seq) return pkcu_fail(PKCU_ERR_ARG, "%s: NULL seq", what);
  if (seq->dev.n_items > 65535)
    return pkcu_fail(PKCU_ERR_ARG, "%s: at most 65535 items per call", what);
  return PKCU_OK;
}

static bool lt_wide(const pkcu_seq *seq) {
  return (long long)((seq->dev.max_T + 31) / 32) * seq->dev.n_items >= pkcu_sm_count();
}

template <int TT>
static dim3 lt_grid(const pkcu_seq *seq) {
  return dim3((unsigned)((seq->dev.max_T + TT - 1) / TT), (unsigned)seq->dev.n_items);
}

// Launches kernel<32, FLAG> or kernel<16, FLAG> (flags slot k or k + 4).
#define PK_LT_LAUNCH(KERNEL, FLAG, k, stream, ...)                                             \
  do {                                                                                         \
    if (lt_wide(seq)) {                                                                        \
      smem_optin(KERNEL<32, FLAG>, lt_smem<32>(), g_lt_flags[k]);                              \
      KERNEL<32, FLAG><<<lt_grid<32>(seq), 32 * 32, lt_smem<32>(), (cudaStream_t)(stream)>>>(  \
          __VA_ARGS__);                                                                        \
    } else {                                                                                   \
      smem_optin(KERNEL<16, FLAG>, lt_smem<16>(), g_lt_flags[(k) + 4]);                        \
      KERNEL<16, FLAG><<<lt_grid<16>(seq), 32 * 16, lt_smem<16>(), (cudaStream_t)(stream)>>>(  \
          __VA_ARGS__);                                                                        \
    }                                                                                          \
  } while (0)

extern "C" int pkcu_layer_norm_transpose(const float *x, const float *gamma, const float *beta,
                                         float *cf, const pkcu_seq *seq,
                                         pkcu_stream_t stream) {
  int st = check_seq_tile(seq, "pkcu_layer_norm_transpose");
  if (st) return st;
  if (!x || !gamma || !beta || !cf || !PK_ALIGNED16(x) || !PK_ALIGNED16(gamma) ||
      !PK_ALIGNED16(beta))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_layer_norm_transpose: bad or misaligned pointer");
  if (seq->frames == 0) return PKCU_OK;
  PK_LT_LAUNCH(ln_transpose_kernel, false, 0, stream, const_cast<float *>(x), nullptr, nullptr,
               0.0f, gamma, beta, cf, seq->dev);
  return pkcu_launch_status("pkcu_layer_norm_transpose");
}

extern "C" int pkcu_residual_layer_norm_transpose(float *x, const float *y, const float *bias,
                                                  float alpha, const float *gamma,
                                                  const float *beta, float *cf,
                                                  const pkcu_seq *seq, pkcu_stream_t stream) {
  int st = check_seq_tile(seq, "pkcu_residual_layer_norm_transpose");
  if (st) return st;
  if (!x || !y || !gamma || !beta || !cf || !PK_ALIGNED16(x) || !PK_ALIGNED16(y) ||
      !PK_ALIGNED16(gamma) || !PK_ALIGNED16(beta) || (bias && !PK_ALIGNED16(bias)))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_residual_layer_norm_transpose: bad or misaligned pointer");
  if (seq->frames == 0) return PKCU_OK;
  PK_LT_LAUNCH(ln_transpose_kernel, true, 1, stream, x, y, bias, alpha, gamma, beta, cf,
               seq->dev);
  return pkcu_launch_status("pkcu_residual_layer_norm_transpose");
}

extern "C" int pkcu_transpose_add(float *x, const float *y, const float *bias,
                                  const pkcu_seq *seq, pkcu_stream_t stream) {
  int st = check_seq_tile(seq, "pkcu_transpose_add");
  if (st) return st;
  if (!x || !y || !PK_ALIGNED16(x) || (bias && !PK_ALIGNED16(bias)))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_transpose_add: bad or misaligned pointer");
  if (seq->frames == 0) return PKCU_OK;
  PK_LT_LAUNCH(transpose_add_kernel, false, 2, stream, x, y, bias, nullptr, nullptr, nullptr,
               seq->dev);
  return pkcu_launch_status("pkcu_transpose_add");
}

extern "C" int pkcu_transpose_add_layer_norm(float *x, const float *y, const float *bias,
                                             const float *gamma, const float *beta, float *ln,
                                             const pkcu_seq *seq, pkcu_stream_t stream) {
  int st = check_seq_tile(seq, "pkcu_transpose_add_layer_norm");
  if (st) return st;
  if (!x || !y || !gamma || !beta || !ln || !PK_ALIGNED16(x) || !PK_ALIGNED16(gamma) ||
      !PK_ALIGNED16(beta) || !PK_ALIGNED16(ln) || (bias && !PK_ALIGNED16(bias)))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_transpose_add_layer_norm: bad or misaligned pointer");
  if (seq->frames == 0) return PKCU_OK;
  PK_LT_LAUNCH(transpose_add_kernel, true, 3, stream, x, y, bias, gamma, beta, ln, seq->dev);
  return pkcu_launch_status("pkcu_transpose_add_layer_norm");
}
