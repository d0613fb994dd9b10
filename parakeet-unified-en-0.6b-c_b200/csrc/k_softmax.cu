// k_softmax.cu -- row softmax and the relative-position attention scores.
//
// Reference: pk_softmax (csrc/tensor_ops.c:284-344, AVX2 path :312-334):
// row max; e = exp(x - max) with the polynomial pk_exp_avx2 on the first
// 8*floor(len/8) entries and libm expf on the rest; sum; x *= 1/sum.
// Here the polynomial is restated bit-exactly (exp_poly) and applied to the
// same entries; the sum is reduced in a different order (tolerance 2e-6 abs /
// 1e-5 rel).
//
// The score path of self_attention (csrc/encoder.c:380-403):
//   bd' = relative_shift(bd)      [H,T,2T-1] -> [H,T,T]   (:230-254)
//   S   = (ac + bd') * (1/sqrt(128))                       (:383-400)
//   S   = softmax over each row                            (:403)
// relative_shift pads each row with a zero column and re-reads the buffer with
// stride 2T-1; the element it lands on is bd[h, i, T-1-i+j] (the pad column is
// never read), so the fused kernel gathers that diagonal band directly: it
// reads ac and the used half of bd once and writes S once (12*H*T^2 bytes per
// item instead of the reference's padded copy, result copy and three passes).
//
// One warp per row, the row in registers (ceil(len/32) values per lane), for
// len <= 1024; a CTA per row with the row in shared memory above that.
#include <math.h>

#include "pk_common.cuh"

namespace pk {

constexpr int SM_ROWS_PER_CTA = 8;
constexpr int SM_BIG_THREADS = 512;
constexpr int SM_MAX_SMEM_LEN = 48 * 1024;   // floats staged per row in the CTA path

// Softmax of one row held by a warp: lane owns entries j = lane + 32k.
template <int NPL>
__device__ __forceinline__ void softmax_regs(float (&v)[NPL], int len, int lane) {
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < NPL; k++)
    if (lane + 32 * k < len) mx = fmaxf(mx, v[k]);
  mx = warp_max(mx);
  const int len8 = len & ~7;
  float s = 0.0f;
  // Polynomial everywhere, then libm expf for the len % 8 tail entries only
  // (a warp-uniform branch: the tail lies in one or two register slots).
  if constexpr (NPL == 1) {
    if (lane < len) {
      float e = exp_poly_nonpos(v[0] - mx);
      if (lane >= len8) e = expf(v[0] - mx);
      v[0] = e;
      s = e;
    }
    s = warp_sum(s);
    v[0] *= 1.0f / s;
  } else {
    static_assert(NPL % 2 == 0, "register slots are processed in pairs");
    float2 s2 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < NPL; k += 2) {
      const int j0 = lane + 32 * k, j1 = j0 + 32;
      float2 d = sub2(make_float2(v[k], v[k + 1]), splat2(mx));
      d.x = fmaxf(d.x, -87.0f);   // exp_poly_nonpos: arguments are <= 0 or NaN
      d.y = fmaxf(d.y, -87.0f);
      float2 e = exp_poly2_clamped(d);
      if (32 * k + 63 < len8) {   // warp-uniform: both slots valid, both polynomial
        v[k] = e.x;
        v[k + 1] = e.y;
        s2 = add2(s2, e);
        continue;
      }
      {
        if (j0 >= len8 && j0 < len) e.x = expf(v[k] - mx);
        if (j1 >= len8 && j1 < len) e.y = expf(v[k + 1] - mx);
      }
      e.x = (j0 < len) ? e.x : 0.0f;
      e.y = (j1 < len) ? e.y : 0.0f;
      v[k] = e.x;
      v[k + 1] = e.y;
      s2 = add2(s2, e);
    }
    s = warp_sum(s2.x + s2.y);
    const float2 inv = splat2(1.0f / s);
#pragma unroll
    for (int k = 0; k < NPL; k += 2) {
      const float2 o = mul2(make_float2(v[k], v[k + 1]), inv);
      v[k] = o.x;
      v[k + 1] = o.y;
    }
  }
}

// In-place softmax of rows of len <= 32*NPL (pk_softmax_rows).
template <int NPL>
__global__ void __launch_bounds__(32 * SM_ROWS_PER_CTA)
softmax_rows_warp_kernel(float *x, long long n_rows, int len) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * SM_ROWS_PER_CTA + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  float *r = x + row * len;
  float v[NPL];
#pragma unroll
  for (int k = 0; k < NPL; k++) {
    const int j = lane + 32 * k;
    v[k] = (j < len) ? r[j] : 0.0f;
  }
  softmax_regs<NPL>(v, len, lane);
#pragma unroll
  for (int k = 0; k < NPL; k++) {
    const int j = lane + 32 * k;
    if (j < len) r[j] = v[k];
  }
}

// Long rows: one CTA per row, staged in shared memory (len <= SM_MAX_SMEM_LEN),
// or re-read from global memory (any len) when smem == 0.
__global__ void __launch_bounds__(SM_BIG_THREADS)
softmax_rows_cta_kernel(float *x, int len, int use_smem) {
  extern __shared__ float sm_row[];
  __shared__ float red[33];
  float *r = x + (long long)blockIdx.x * len;
  float *buf = use_smem ? sm_row : r;
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < len; j += blockDim.x) {
    const float t = r[j];
    if (use_smem) buf[j] = t;
    mx = fmaxf(mx, t);
  }
  mx = block_max(mx, red);
  const int len8 = len & ~7;
  float s = 0.0f;
  for (int j = threadIdx.x; j < len; j += blockDim.x) {
    const float d = buf[j] - mx;
    const float e = (j < len8) ? exp_poly_nonpos(d) : expf(d);
    buf[j] = e;
    s += e;
  }
  s = block_sum(s, red);
  const float inv = 1.0f / s;
  for (int j = threadIdx.x; j < len; j += blockDim.x) r[j] = buf[j] * inv;
}

// Per-item score rows: row r of item b is head h = r / T, query i = r % T.
struct ScoreRow {
  long long ac, bd, s;  // element offsets of the row's first entry
  int T, i;
};

__device__ __forceinline__ bool score_row(const SeqDev &seq, int item, int r, ScoreRow &o) {
  const int T = seq_T(seq, item);
  if (r >= PK_H * T) return false;
  const int i = r % T;
  const long long so = seq_score_off(seq, item) + (long long)r * T;
  o.ac = so;
  o.s = so;
  o.bd = seq_bd_off(seq, item) + (long long)r * (2 * T - 1) + (T - 1 - i);
  o.T = T;
  o.i = i;
  return true;
}

// S = (ac + bd_shift) * scale [+ softmax], one warp per score row.
template <int NPL, bool SOFTMAX>
__global__ void __launch_bounds__(32 * SM_ROWS_PER_CTA)
relpos_scores_warp_kernel(const float *ac, const float *__restrict__ bd, float *S, float scale,
                          SeqDev seq) {
  const int lane = threadIdx.x & 31;
  ScoreRow rw;
  if (!score_row(seq, blockIdx.y, blockIdx.x * SM_ROWS_PER_CTA + (threadIdx.x >> 5), rw)) return;
  const int len = rw.T;
  float v[NPL];
#pragma unroll
  for (int k = 0; k < NPL; k++) {
    const int j = lane + 32 * k;
    v[k] = (j < len) ? (__ldcs(ac + rw.ac + j) + __ldcs(bd + rw.bd + j)) * scale : 0.0f;
  }
  if (SOFTMAX) softmax_regs<NPL>(v, len, lane);
#pragma unroll
  for (int k = 0; k < NPL; k++) {
    const int j = lane + 32 * k;
    if (j < len) S[rw.s + j] = v[k];
  }
}

// Rows longer than 32*32: one CTA per score row, row staged in shared memory.
template <bool SOFTMAX>
__global__ void __launch_bounds__(SM_BIG_THREADS)
relpos_scores_cta_kernel(const float *ac, const float *__restrict__ bd, float *S, float scale,
                         SeqDev seq) {
  extern __shared__ float sm_row[];
  __shared__ float red[33];
  ScoreRow rw;
  if (!score_row(seq, blockIdx.y, blockIdx.x, rw)) return;
  const int len = rw.T;
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < len; j += blockDim.x) {
    const float t = (ac[rw.ac + j] + bd[rw.bd + j]) * scale;
    sm_row[j] = t;
    mx = fmaxf(mx, t);
  }
  if (!SOFTMAX) {
    __syncthreads();
    for (int j = threadIdx.x; j < len; j += blockDim.x) S[rw.s + j] = sm_row[j];
    return;
  }
  mx = block_max(mx, red);
  const int len8 = len & ~7;
  float s = 0.0f;
  for (int j = threadIdx.x; j < len; j += blockDim.x) {
    const float d = sm_row[j] - mx;
    const float e = (j < len8) ? exp_poly_nonpos(d) : expf(d);
    sm_row[j] = e;
    s += e;
  }
  s = block_sum(s, red);
  const float inv = 1.0f / s;
  for (int j = threadIdx.x; j < len; j += blockDim.x) S[rw.s + j] = sm_row[j] * inv;
}

// ── pipelined score rows ─────────────────────────────────────────────────────
// Persistent warps walk the flat list of score rows of every item. Each warp
// double-buffers in shared memory: while it computes row n (registers), the
// async copies of row n+1's ac row and bd band are in flight, so the HBM
// stream never waits on the softmax arithmetic. Rows of up to 32*NPL entries.
constexpr int PIPE_WARPS = 8;

struct RowLoc {
  long long ac, bd;   // first element of the ac row / of the used bd band
  int T, valid;
};

// Row indices fit in 32 bits (the launcher checks H * frames < 2^31), so the
// decomposition row -> (item, head-row r, query i) uses 32-bit unsigned
// division; only the element offsets are 64-bit.
__device__ __forceinline__ RowLoc locate_row(const SeqDev &seq, unsigned row, unsigned total_rows) {
  RowLoc o;
  o.valid = row < total_rows;
  if (!o.valid) { o.ac = o.bd = 0; o.T = 0; return o; }
  int item;
  unsigned r;
  if (seq.uniform_T > 0) {
    const unsigned per = (unsigned)(PK_H * seq.uniform_T);
    item = (int)(row / per);
    r = row - (unsigned)item * per;
  } else {   // rows of item b: [H*frame_off[b], H*frame_off[b+1])
    int lo = 0, hi = seq.n_items;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if ((unsigned)(PK_H * __ldg(seq.frame_off + mid)) <= row) lo = mid; else hi = mid;
    }
    item = lo;
    r = row - (unsigned)(PK_H * __ldg(seq.frame_off + lo));
  }
  const int T = seq_T(seq, item);
  const int i = (int)(r % (unsigned)T);
  o.ac = seq_score_off(seq, item) + (long long)r * T;
  o.bd = seq_bd_off(seq, item) + (long long)r * (2 * T - 1) + (T - 1 - i);
  o.T = T;
  return o;
}

template <int NPL, bool SOFTMAX>
__global__ void __launch_bounds__(32 * PIPE_WARPS)
relpos_scores_pipe_kernel(const float *ac, const float *__restrict__ bd, float *S, float scale,
                          SeqDev seq, unsigned total_rows, long long ac_total, long long bd_total,
                          int stage) {
  extern __shared__ float4 pipe_smem4[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // per warp: [buf0 ac | buf0 bd | buf1 ac | buf1 bd], `stage` floats each
  float *wb = reinterpret_cast<float *>(pipe_smem4) + (size_t)warp * 4 * stage;
  const unsigned nw = gridDim.x * PIPE_WARPS;
  unsigned row = blockIdx.x * PIPE_WARPS + warp;
  RowLoc cur = locate_row(seq, row, total_rows);
  int off_ac = 0, off_bd = 0;
  if (cur.valid) {
    off_ac = cp_async_span(wb, ac, cur.ac, cur.T, ac_total, lane);
    off_bd = cp_async_span(wb + stage, bd, cur.bd, cur.T, bd_total, lane);
  }
  cp_async_commit();
  int buf = 0;
  for (; cur.valid; row += nw) {
    // prefetch the next row into the other buffer
    const RowLoc nxt = locate_row(seq, row + nw, total_rows);
    int noff_ac = 0, noff_bd = 0;
    float *nb = wb + (buf ^ 1) * 2 * stage;
    if (nxt.valid) {
      noff_ac = cp_async_span(nb, ac, nxt.ac, nxt.T, ac_total, lane);
      noff_bd = cp_async_span(nb + stage, bd, nxt.bd, nxt.T, bd_total, lane);
    }
    cp_async_commit();
    cp_async_wait<1>();   // this lane's copies of the current row have landed
    __syncwarp();         // ... and every other lane's
    const float *sa = wb + buf * 2 * stage + off_ac;
    const float *sb = wb + buf * 2 * stage + stage + off_bd;
    const int len = cur.T;
    float v[NPL];
#pragma unroll
    for (int k = 0; k < NPL; k += 2) {
      const int j0 = lane + 32 * k, j1 = j0 + 32;
      if (32 * k + 63 < len) {   // warp-uniform: both slots inside the row
        const float2 c = mul2(add2(make_float2(sa[j0], sa[j1]), make_float2(sb[j0], sb[j1])),
                              splat2(scale));   // (ac + bd) * scale, each rounded
        v[k] = c.x;
        v[k + 1] = c.y;
        continue;
      }
      const float2 a = make_float2(j0 < len ? sa[j0] : 0.0f, j1 < len ? sa[j1] : 0.0f);
      const float2 b = make_float2(j0 < len ? sb[j0] : 0.0f, j1 < len ? sb[j1] : 0.0f);
      const float2 c = mul2(add2(a, b), splat2(scale));
      v[k] = j0 < len ? c.x : 0.0f;
      v[k + 1] = j1 < len ? c.y : 0.0f;
    }
    if (SOFTMAX) softmax_regs<NPL>(v, len, lane);
    float *dst = S + cur.ac;
#pragma unroll
    for (int k = 0; k < NPL; k++) {
      const int j = lane + 32 * k;
      if (32 * k + 31 < len || j < len) dst[j] = v[k];
    }
    __syncwarp();         // the buffer is refilled two rows from now
    cur = nxt;
    off_ac = noff_ac;
    off_bd = noff_bd;
    buf ^= 1;
  }
  cp_async_wait<0>();
}

// relative_shift alone: out[h,i,j] = bd[h,i,T-1-i+j] (exact gather).
__global__ void __launch_bounds__(256)
relative_shift_kernel(const float *__restrict__ bd, float *__restrict__ out, SeqDev seq) {
  const int item = blockIdx.y;
  const int T = seq_T(seq, item);
  const long long n = (long long)PK_H * T * T;
  const long long so = seq_score_off(seq, item), bo = seq_bd_off(seq, item);
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const long long r = e / T;
    const int j = (int)(e - r * T);
    const int i = (int)(r % T);
    out[so + e] = bd[bo + r * (2 * T - 1) + (T - 1 - i) + j];
  }
}

template <int NPL, bool SOFTMAX>
static void launch_scores_warp(const float *ac, const float *bd, float *S, float scale,
                               const pkcu_seq *seq, cudaStream_t s) {
  dim3 grid((unsigned)((PK_H * seq->dev.max_T + SM_ROWS_PER_CTA - 1) / SM_ROWS_PER_CTA),
            (unsigned)seq->dev.n_items);
  relpos_scores_warp_kernel<NPL, SOFTMAX><<<grid, 32 * SM_ROWS_PER_CTA, 0, s>>>(ac, bd, S, scale,
                                                                              seq->dev);
}

template <int NPL, bool SOFTMAX>
static void launch_scores_pipe(const float *ac, const float *bd, float *S, float scale,
                               const pkcu_seq *seq, cudaStream_t s) {
  const int stage = ((seq->dev.max_T + 8 + 3) / 4) * 4;
  const size_t smem = sizeof(float) * 4 * (size_t)stage * PIPE_WARPS;
  static int flags[64];
  smem_optin(relpos_scores_pipe_kernel<NPL, SOFTMAX>, smem, flags);
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, relpos_scores_pipe_kernel<NPL, SOFTMAX>,
                                                32 * PIPE_WARPS, smem);
  if (per_sm < 1) per_sm = 1;
  const long long rows = (long long)PK_H * seq->frames;
  long long grid = (rows + PIPE_WARPS - 1) / PIPE_WARPS;
  const long long cap = (long long)pkcu_sm_count() * per_sm;
  if (grid > cap) grid = cap;
  relpos_scores_pipe_kernel<NPL, SOFTMAX><<<(unsigned)grid, 32 * PIPE_WARPS, smem, s>>>(
      ac, bd, S, scale, seq->dev, (unsigned)rows, seq->score_elems, seq->bd_elems, stage);
}

// The pipelined kernel indexes rows in 32 bits (and nw + row must not wrap).
static bool pipe_rows_fit(const pkcu_seq *seq) {
  return (long long)PK_H * seq->frames < (1LL << 31);
}

template <bool SOFTMAX>
static int launch_scores(const float *ac, const float *bd, float *S, float scale,
                         const pkcu_seq *seq, cudaStream_t s) {
  const int T = seq->dev.max_T;
  const int npl = (T + 31) / 32;
  if (PK_ALIGNED16(ac) && PK_ALIGNED16(bd) && npl <= 16 && pipe_rows_fit(seq)) {
    if (npl <= 4) launch_scores_pipe<4, SOFTMAX>(ac, bd, S, scale, seq, s);
    else if (npl <= 8) launch_scores_pipe<8, SOFTMAX>(ac, bd, S, scale, seq, s);
    else if (npl <= 12) launch_scores_pipe<12, SOFTMAX>(ac, bd, S, scale, seq, s);
    else launch_scores_pipe<16, SOFTMAX>(ac, bd, S, scale, seq, s);
    return PKCU_OK;
  }
  if (npl <= 4) launch_scores_warp<4, SOFTMAX>(ac, bd, S, scale, seq, s);
  else if (npl <= 8) launch_scores_warp<8, SOFTMAX>(ac, bd, S, scale, seq, s);
  else if (npl <= 12) launch_scores_warp<12, SOFTMAX>(ac, bd, S, scale, seq, s);
  else if (npl <= 16) launch_scores_warp<16, SOFTMAX>(ac, bd, S, scale, seq, s);
  else if (npl <= 24) launch_scores_warp<24, SOFTMAX>(ac, bd, S, scale, seq, s);
  else if (npl <= 32) launch_scores_warp<32, SOFTMAX>(ac, bd, S, scale, seq, s);
  else {
    if (T > SM_MAX_SMEM_LEN)
      return pkcu_fail(PKCU_ERR_ARG, "relpos scores: T=%d above the %d-frame limit", T,
                       SM_MAX_SMEM_LEN);
    const size_t smem = sizeof(float) * (size_t)T;
    static int flags[64];
    smem_optin(relpos_scores_cta_kernel<SOFTMAX>, smem, flags);
    dim3 grid((unsigned)(PK_H * T), (unsigned)seq->dev.n_items);
    relpos_scores_cta_kernel<SOFTMAX><<<grid, SM_BIG_THREADS, smem, s>>>(ac, bd, S, scale,
                                                                        seq->dev);
  }
  return PKCU_OK;
}

template <int NPL>
static void launch_softmax_warp(float *x, long long n_rows, int len, cudaStream_t s) {
  const unsigned grid = (unsigned)((n_rows + SM_ROWS_PER_CTA - 1) / SM_ROWS_PER_CTA);
  softmax_rows_warp_kernel<NPL><<<grid, 32 * SM_ROWS_PER_CTA, 0, s>>>(x, n_rows, len);
}

static int check_scores(const float *ac, const float *bd, const float *S, const pkcu_seq *seq,
                        const char *what) {
  if (!ac || !bd || !S || !seq) return pkcu_fail(PKCU_ERR_ARG, "%s: NULL argument", what);
  if (seq->dev.n_items > 65535)
    return pkcu_fail(PKCU_ERR_ARG, "%s: at most 65535 items per call", what);
  return PKCU_OK;
}

}  // namespace pk

using namespace pk;

extern "C" int pkcu_softmax_rows(float *x, int n_rows, int len, pkcu_stream_t stream) {
  if (!x || n_rows < 0 || len <= 0) return pkcu_fail(PKCU_ERR_ARG, "pkcu_softmax_rows: bad argument");
  if (n_rows == 0) return PKCU_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int npl = (len + 31) / 32;
  if (npl <= 1) launch_softmax_warp<1>(x, n_rows, len, s);
  else if (npl <= 2) launch_softmax_warp<2>(x, n_rows, len, s);
  else if (npl <= 4) launch_softmax_warp<4>(x, n_rows, len, s);
  else if (npl <= 8) launch_softmax_warp<8>(x, n_rows, len, s);
  else if (npl <= 12) launch_softmax_warp<12>(x, n_rows, len, s);
  else if (npl <= 16) launch_softmax_warp<16>(x, n_rows, len, s);
  else if (npl <= 24) launch_softmax_warp<24>(x, n_rows, len, s);
  else if (npl <= 32) launch_softmax_warp<32>(x, n_rows, len, s);
  else {
    const int use_smem = len <= SM_MAX_SMEM_LEN;
    const size_t smem = use_smem ? sizeof(float) * (size_t)len : 0;
    static int flags[64];
    if (use_smem) smem_optin(softmax_rows_cta_kernel, smem, flags);
    softmax_rows_cta_kernel<<<n_rows, SM_BIG_THREADS, smem, s>>>(x, len, use_smem);
  }
  return pkcu_launch_status("pkcu_softmax_rows");
}

extern "C" int pkcu_relpos_combine(const float *ac, const float *bd, float *S, float scale,
                                   const pkcu_seq *seq, pkcu_stream_t stream) {
  int st = check_scores(ac, bd, S, seq, "pkcu_relpos_combine");
  if (st) return st;
  if (seq->frames == 0) return PKCU_OK;
  st = launch_scores<false>(ac, bd, S, scale, seq, (cudaStream_t)stream);
  if (st) return st;
  return pkcu_launch_status("pkcu_relpos_combine");
}

extern "C" int pkcu_relpos_combine_softmax(const float *ac, const float *bd, float *S,
                                           float scale, const pkcu_seq *seq,
                                           pkcu_stream_t stream) {
  int st = check_scores(ac, bd, S, seq, "pkcu_relpos_combine_softmax");
  if (st) return st;
  if (seq->frames == 0) return PKCU_OK;
  st = launch_scores<true>(ac, bd, S, scale, seq, (cudaStream_t)stream);
  if (st) return st;
  return pkcu_launch_status("pkcu_relpos_combine_softmax");
}

extern "C" int pkcu_relative_shift(const float *bd, float *out, const pkcu_seq *seq,
                                   pkcu_stream_t stream) {
  if (!bd || !out || !seq) return pkcu_fail(PKCU_ERR_ARG, "pkcu_relative_shift: NULL argument");
  if (seq->dev.n_items > 65535)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_relative_shift: at most 65535 items per call");
  if (seq->frames == 0) return PKCU_OK;
  const long long per = (long long)PK_H * seq->dev.max_T * seq->dev.max_T;
  long long bx = (per + 255) / 256;
  if (bx > 4096) bx = 4096;
  relative_shift_kernel<<<dim3((unsigned)bx, (unsigned)seq->dev.n_items), 256, 0,
                          (cudaStream_t)stream>>>(bd, out, seq->dev);
  return pkcu_launch_status("pkcu_relative_shift");
}
