// k_elementwise.cu -- streaming elementwise ops: Swish, bias add, residual add,
// ReLU, the RNN-T joint add + activation.
//
// Every op here is 8-12 bytes of HBM traffic per element and no reuse, so the
// kernels are 128-bit loads/stores with several independent loads in flight
// per thread; row ops run one warp per row (bias index = column, no division).
//
// Swish keeps the reference's split (csrc/tensor_ops.c:380-389): the first
// 8*floor(n/8) elements of the flat array use the polynomial form
// v * (1/(1 + exp_poly(-v))), bit-identical to the restated pk_exp_avx2; the
// remaining n % 8 elements use x / (1 + expf(-x)).
#include <math.h>

#include "pk_common.cuh"

namespace pk {

constexpr int EW_THREADS = 256;
constexpr int ROWS_PER_CTA = 8;

__device__ __forceinline__ float4 swish4(float4 v) {
  const float2 a = swish_poly2(make_float2(v.x, v.y)), b = swish_poly2(make_float2(v.z, v.w));
  return make_float4(a.x, a.y, b.x, b.y);
}

// ── flat Swish ───────────────────────────────────────────────────────────────

__global__ void __launch_bounds__(EW_THREADS) swish_vec_kernel(float *x, long long n) {
  const long long n8 = n & ~7LL, n4 = n8 >> 2;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 7 * stride < n4; i += 8 * stride) {   // 8 float4 loads in flight per thread
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = ld4(x + 4 * (i + j * stride));
#pragma unroll
    for (int j = 0; j < 8; j++) st4(x + 4 * (i + j * stride), swish4(v[j]));
  }
  for (; i < n4; i += stride) st4(x + 4 * i, swish4(ld4(x + 4 * i)));
  if (blockIdx.x == 0 && threadIdx.x < n - n8) x[n8 + threadIdx.x] = swish_tail(x[n8 + threadIdx.x]);
}

__global__ void __launch_bounds__(EW_THREADS) swish_scalar_kernel(float *x, long long n) {
  const long long n8 = n & ~7LL;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x)
    x[e] = (e < n8) ? swish_poly(x[e]) : swish_tail(x[e]);
}

// ── ReLU: x < 0 ? 0 : x (NaN and -0 kept) ───────────────────────────────────
// csrc/tensor_ops.c:401-416. The scalar tail states this form and the
// reference's -ffast-math build gives its vector body the same result.

__device__ __forceinline__ float relu1(float v) { return (v < 0.0f) ? 0.0f : v; }

__global__ void __launch_bounds__(EW_THREADS) relu_kernel(float *x, long long n, int vec) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long done = 0;
  if (vec) {
    const long long n4 = n >> 2;
    for (; i + 3 * stride < n4; i += 4 * stride) {   // 4 float4 loads in flight per thread
      float4 v[4];
#pragma unroll
      for (int j = 0; j < 4; j++) v[j] = ld4(x + 4 * (i + j * stride));
#pragma unroll
      for (int j = 0; j < 4; j++)
        st4(x + 4 * (i + j * stride), make_float4(relu1(v[j].x), relu1(v[j].y), relu1(v[j].z),
                                                  relu1(v[j].w)));
    }
    for (; i < n4; i += stride) {
      float4 v = ld4(x + 4 * i);
      st4(x + 4 * i, make_float4(relu1(v.x), relu1(v.y), relu1(v.z), relu1(v.w)));
    }
    done = n4 << 2;
    i = done + (long long)blockIdx.x * blockDim.x + threadIdx.x;
  }
  for (; i < n; i += stride) x[i] = relu1(x[i]);
}

// ── row ops: one warp per row ────────────────────────────────────────────────

enum { ROW_BIAS = 0, ROW_BIAS_SWISH = 1, ROW_RESID = 2 };

// ROW_BIAS      : x[r,c] += b[c]                    (pk_bias_add per row)
// ROW_BIAS_SWISH: out[r,c] = swish(in[r,c] + b[c])  (csrc/encoder.c:194-196)
// ROW_RESID     : x[r,c] = fma(y[r,c] + b[c], alpha, x[r,c])
// Vector path: len % 4 == 0 and 16-byte aligned pointers. TAIL: the flat
// length is not a multiple of 8, so the last elements take Swish's scalar form.
// One warp per segment of a row: the row's float4s [seg * seg4, (seg + 1) * seg4),
// segs segments per row (1 for large batches; short batches split rows so that
// more warps share the latency).
template <int OP, bool TAIL>
__global__ void __launch_bounds__(32 * ROWS_PER_CTA)
row_vec_kernel(const float *in, const float *__restrict__ b, const float *__restrict__ y,
               float alpha, float *out, long long n_rows, int len, long long n8, int segs) {
  const int lane = threadIdx.x & 31;
  const long long wid = (long long)blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  const long long row = wid / segs;
  if (row >= n_rows) return;
  const long long base = row * len;
  const int len4 = len >> 2;
  const int seg4 = (len4 + segs - 1) / segs;
  const int seg0 = (int)(wid - row * segs) * seg4;
  const int seg_end = min(len4, seg0 + seg4);
  constexpr int U = 8;
  for (int c0 = seg0 + lane; c0 < seg_end; c0 += 32 * U) {
    float4 v[U], t[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int c = c0 + 32 * u;
      if (c < seg_end) {
        v[u] = ld4(in + base + 4 * c);
        if (OP == ROW_RESID) t[u] = ldg4_stream(y + base + 4 * c);
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int c = c0 + 32 * u;
      if (c >= seg_end) continue;
      float4 bb = b ? __ldg(reinterpret_cast<const float4 *>(b) + c) : make_float4(0, 0, 0, 0);
      float4 r;
      if (OP == ROW_BIAS) {
        r = add4(v[u], bb);
      } else if (OP == ROW_BIAS_SWISH) {
        r = add4(v[u], bb);
        const long long e = base + 4 * c;
        if (!TAIL || e + 4 <= n8) {
          r = swish4(r);
        } else {   // only the last float4s of a flat array whose length is not a multiple of 8
          r = make_float4(e < n8 ? swish_poly(r.x) : swish_tail(r.x),
                          e + 1 < n8 ? swish_poly(r.y) : swish_tail(r.y),
                          e + 2 < n8 ? swish_poly(r.z) : swish_tail(r.z),
                          e + 3 < n8 ? swish_poly(r.w) : swish_tail(r.w));
        }
      } else {
        const float4 yy = b ? add4(t[u], bb) : t[u];
        r = make_float4(fmaf(yy.x, alpha, v[u].x), fmaf(yy.y, alpha, v[u].y),
                        fmaf(yy.z, alpha, v[u].z), fmaf(yy.w, alpha, v[u].w));
      }
      st4(out + base + 4 * c, r);
    }
  }
}

// Any length / alignment.
template <int OP>
__global__ void __launch_bounds__(EW_THREADS)
row_scalar_kernel(const float *in, const float *__restrict__ b, const float *__restrict__ y,
                  float alpha, float *out, long long n, int len, long long n8) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(e % len);
    const float bb = b ? b[c] : 0.0f;
    float r;
    if (OP == ROW_BIAS) r = in[e] + bb;
    else if (OP == ROW_BIAS_SWISH) {
      const float v = in[e] + bb;
      r = (e < n8) ? swish_poly(v) : swish_tail(v);
    } else {
      const float yy = b ? y[e] + bb : y[e];
      r = fmaf(yy, alpha, in[e]);
    }
    out[e] = r;
  }
}

// ── RNN-T joint: out[b,t,j] = act(enc[b,t,j] + pred[b,j]) ────────────────────

template <int ACT>
__device__ __forceinline__ float joint_act(float h) {
  if (ACT == PKCU_ACT_RELU) return (h < 0.0f) ? 0.0f : h;   // csrc/decoder.c:65-66
  return tanhf(h);
}

template <int ACT>
__global__ void __launch_bounds__(32 * ROWS_PER_CTA)
joint_vec_kernel(const float *__restrict__ enc, const float *__restrict__ pred,
                 float *__restrict__ out, long long n_rows, int T, int J) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const float4 *e4 = reinterpret_cast<const float4 *>(enc + row * J);
  const float4 *p4 = reinterpret_cast<const float4 *>(pred + (row / T) * J);
  float4 *o4 = reinterpret_cast<float4 *>(out + row * J);
  for (int c = lane; c < (J >> 2); c += 32) {
    const float4 h = add4(__ldcs(e4 + c), __ldg(p4 + c));
    o4[c] = make_float4(joint_act<ACT>(h.x), joint_act<ACT>(h.y), joint_act<ACT>(h.z),
                        joint_act<ACT>(h.w));
  }
}

template <int ACT>
__global__ void __launch_bounds__(EW_THREADS)
joint_scalar_kernel(const float *enc, const float *pred, float *out, long long n, int T, int J) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / J;
    const int j = (int)(e - row * J);
    out[e] = joint_act<ACT>(enc[e] + pred[(row / T) * J + j]);
  }
}

static unsigned flat_grid(long long work, long long per_cta) {
  long long g = (work + per_cta - 1) / per_cta;
  const long long cap = (long long)pkcu_sm_count() * 32;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

template <int OP>
static int launch_rows(const float *in, const float *b, const float *y, float alpha, float *out,
                       long long n_rows, int len, cudaStream_t s) {
  const long long n = n_rows * len;
  const long long n8 = n & ~7LL;
  const bool vec = (len % 4 == 0) && PK_ALIGNED16(in) && PK_ALIGNED16(out) &&
                   (!b || PK_ALIGNED16(b)) && (!y || PK_ALIGNED16(y));
  if (vec) {
    // rows of 256+ float4s split into segments of at least 256 when fewer
    // than 48 row-warps per SM would run
    int segs = 1;
    if (n_rows < (long long)pkcu_sm_count() * 48) segs = (len / 4 + 255) / 256;
    if (segs < 1) segs = 1;
    const unsigned grid = (unsigned)((n_rows * segs + ROWS_PER_CTA - 1) / ROWS_PER_CTA);
    if (n8 == n)
      row_vec_kernel<OP, false><<<grid, 32 * ROWS_PER_CTA, 0, s>>>(in, b, y, alpha, out, n_rows, len, n8, segs);
    else
      row_vec_kernel<OP, true><<<grid, 32 * ROWS_PER_CTA, 0, s>>>(in, b, y, alpha, out, n_rows, len, n8, segs);
  } else {
    row_scalar_kernel<OP><<<flat_grid(n, EW_THREADS * 4), EW_THREADS, 0, s>>>(
        in, b, y, alpha, out, n, len, n8);
  }
  return PKCU_OK;
}

}  // namespace pk

using namespace pk;

extern "C" int pkcu_swish(float *x, long long n, pkcu_stream_t stream) {
  if (!x || n < 0) return pkcu_fail(PKCU_ERR_ARG, "pkcu_swish: bad argument");
  if (n == 0) return PKCU_OK;
  cudaStream_t s = (cudaStream_t)stream;
  // one 8-float4 chunk per thread: no grid-stride cap (measured faster than
  // a capped grid striding over the array)
  if (PK_ALIGNED16(x)) {
    long long g = (n / 4 + EW_THREADS * 8 - 1) / (EW_THREADS * 8);
    if (g > 0x7fffffffLL) g = 0x7fffffffLL;   // the kernel strides over the rest
    swish_vec_kernel<<<(unsigned)(g < 1 ? 1 : g), EW_THREADS, 0, s>>>(x, n);
  }
  if (!PK_ALIGNED16(x)) swish_scalar_kernel<<<flat_grid(n, EW_THREADS * 4), EW_THREADS, 0, s>>>(x, n);
  return pkcu_launch_status("pkcu_swish");
}

extern "C" int pkcu_relu(float *x, long long n, pkcu_stream_t stream) {
  if (!x || n < 0) return pkcu_fail(PKCU_ERR_ARG, "pkcu_relu: bad argument");
  if (n == 0) return PKCU_OK;
  const int vec = PK_ALIGNED16(x);
  relu_kernel<<<flat_grid(vec ? n / 4 : n, EW_THREADS * 4), EW_THREADS, 0, (cudaStream_t)stream>>>(
      x, n, vec);
  return pkcu_launch_status("pkcu_relu");
}

extern "C" int pkcu_bias_add_rows(float *x, const float *b, int n_rows, int len,
                                  pkcu_stream_t stream) {
  if (!x || !b || n_rows < 0 || len <= 0)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_bias_add_rows: bad argument");
  if (n_rows == 0) return PKCU_OK;
  launch_rows<ROW_BIAS>(x, b, nullptr, 0.0f, x, n_rows, len, (cudaStream_t)stream);
  return pkcu_launch_status("pkcu_bias_add_rows");
}

extern "C" int pkcu_bias_swish_rows(const float *in, const float *b, float *out, int n_rows,
                                    int len, pkcu_stream_t stream) {
  if (!in || !b || !out || n_rows < 0 || len <= 0)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_bias_swish_rows: bad argument");
  if (n_rows == 0) return PKCU_OK;
  launch_rows<ROW_BIAS_SWISH>(in, b, nullptr, 0.0f, out, n_rows, len, (cudaStream_t)stream);
  return pkcu_launch_status("pkcu_bias_swish_rows");
}

extern "C" int pkcu_residual_add(float *x, const float *y, const float *bias, float alpha,
                                 int n_rows, int D, pkcu_stream_t stream) {
  if (!x || !y || n_rows < 0 || D <= 0)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_residual_add: bad argument");
  if (n_rows == 0) return PKCU_OK;
  launch_rows<ROW_RESID>(x, bias, y, alpha, x, n_rows, D, (cudaStream_t)stream);
  return pkcu_launch_status("pkcu_residual_add");
}

extern "C" int pkcu_joint_add_act(const float *enc, const float *pred, float *out, int B, int T,
                                  int J, int act, pkcu_stream_t stream) {
  if (!enc || !pred || !out || B < 0 || T <= 0 || J <= 0 ||
      (act != PKCU_ACT_RELU && act != PKCU_ACT_TANH))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_joint_add_act: bad argument");
  if (B == 0) return PKCU_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const long long rows = (long long)B * T;
  const bool vec = (J % 4 == 0) && PK_ALIGNED16(enc) && PK_ALIGNED16(pred) && PK_ALIGNED16(out);
  if (vec) {
    const unsigned g = (unsigned)((rows + ROWS_PER_CTA - 1) / ROWS_PER_CTA);
    if (act == PKCU_ACT_RELU)
      joint_vec_kernel<PKCU_ACT_RELU><<<g, 32 * ROWS_PER_CTA, 0, s>>>(enc, pred, out, rows, T, J);
    else
      joint_vec_kernel<PKCU_ACT_TANH><<<g, 32 * ROWS_PER_CTA, 0, s>>>(enc, pred, out, rows, T, J);
  } else {
    const long long n = rows * J;
    if (act == PKCU_ACT_RELU)
      joint_scalar_kernel<PKCU_ACT_RELU><<<flat_grid(n, EW_THREADS * 4), EW_THREADS, 0, s>>>(
          enc, pred, out, n, T, J);
    else
      joint_scalar_kernel<PKCU_ACT_TANH><<<flat_grid(n, EW_THREADS * 4), EW_THREADS, 0, s>>>(
          enc, pred, out, n, T, J);
  }
  return pkcu_launch_status("pkcu_joint_add_act");
}
