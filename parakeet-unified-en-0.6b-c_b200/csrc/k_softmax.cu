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

// In-place softmax of rows of len <= 32*NPL (pk_softmax_rows): a warp takes
// ROWS consecutive rows and requests all of them before computing the first,
// so that more loads are in flight per warp.
template <int NPL, int ROWS>
__global__ void __launch_bounds__(32 * SM_ROWS_PER_CTA)
softmax_rows_warp_kernel(float *x, long long n_rows, int len) {
  const int lane = threadIdx.x & 31;
  const long long row0 = ((long long)blockIdx.x * SM_ROWS_PER_CTA + (threadIdx.x >> 5)) * ROWS;
  if (row0 >= n_rows) return;
  float v[ROWS][NPL];
#pragma unroll
  for (int q = 0; q < ROWS; q++) {
    const bool ok = row0 + q < n_rows;
    const float *r = x + (ok ? row0 + q : row0) * len;
#pragma unroll
    for (int k = 0; k < NPL; k++) {
      const int j = lane + 32 * k;
      v[q][k] = (ok && j < len) ? r[j] : 0.0f;
    }
  }
#pragma unroll
  for (int q = 0; q < ROWS; q++) {
    if (row0 + q >= n_rows) break;   // warp-uniform
    softmax_regs<NPL>(v[q], len, lane);
    float *r = x + (row0 + q) * len;
#pragma unroll
    for (int k = 0; k < NPL; k++) {
      const int j = lane + 32 * k;
      if (j < len) r[j] = v[q][k];
    }
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
// Persistent warps, each owning a contiguous range of score rows (all items'
// rows in flat order), ROWS rows at a time: lane group g = lane / LPR
// (LPR = 32 / ROWS lanes) computes row r + g, so the per-row bookkeeping, the
// copy issue and the reductions of ROWS rows share their instructions. Each
// warp keeps a ring of NBUF buffers in shared memory: while it computes one
// group of rows, the bulk copies of the next NBUF - 1 groups' ac rows and bd
// bands (issued by the group leaders, completion on each buffer's mbarrier)
// are in flight.
//
// S and ac have the same layout, so a score row starts at the same offset mod
// 4 floats (off) in both. The entries are processed in the 4-float chunks of
// that alignment: chunk q holds row entries j = 4q + e - off (e = 0..3). The
// main loop takes the chunks that lie wholly inside [0, len8) -- lane li of
// the group owns chunks q_lo + li + LPR k -- with one 16-byte shared load of
// ac and one 16-byte store of S each and the arithmetic as packed pairs. The
// leftover entries (at most 3 before the first such chunk and 10 after the
// last: the row's unaligned head, and its tail including the len % 8 entries
// that take libm expf) are taken one per lane in a separate step, so no lane
// runs an edge path inside the main loop. The bd band has an alignment of
// its own: it is staged 0 or 4 floats further in, so that the band entries
// of chunk q start `shift` (0..3) floats into chunk slot q and are cut out of
// slots q and q + 1.
constexpr int PIPE_WARPS = 2;   // warps per CTA
constexpr int NBUF = 4;         // ring slots per warp (3 row groups in flight)

struct RowLoc {
  long long ac, bd;   // first element of the ac row / of the used bd band
  int T, i, valid;
};

// Ragged batches: rows of item b are [H*frame_off[b], H*frame_off[b+1]).
__device__ __forceinline__ RowLoc locate_row(const SeqDev &seq, unsigned row, unsigned total_rows) {
  RowLoc o;
  o.valid = row < total_rows;
  if (!o.valid) { o.ac = o.bd = 0; o.T = 1; o.i = 0; return o; }
  int lo = 0, hi = seq.n_items;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if ((unsigned)(PK_H * __ldg(seq.frame_off + mid)) <= row) lo = mid; else hi = mid;
  }
  const unsigned r = row - (unsigned)(PK_H * __ldg(seq.frame_off + lo));
  const int T = seq_T(seq, lo);
  o.i = (int)(r % (unsigned)T);
  o.ac = seq_score_off(seq, lo) + (long long)r * T;
  o.bd = seq_bd_off(seq, lo) + (long long)r * (2 * T - 1) + (T - 1 - o.i);
  o.T = T;
  return o;
}

// Uniform batches: row n of the flat list has ac = n T and
// bd = n (2T - 1) + T - 1 - i = 2 ac - n + T - 1 - i with i = n mod T.
__device__ __forceinline__ RowLoc uniform_row(unsigned row, unsigned total_rows, int T, int i) {
  RowLoc o;
  o.valid = row < total_rows;
  o.T = T;
  o.i = i;
  o.ac = (long long)row * T;
  o.bd = 2 * o.ac - row + (T - 1 - i);
  return o;
}

// Lane li == 0 of each group posts its row's copies into (ac buffer, bd
// buffer) on mbarrier bar (one arrival per group); lanes of the group copy the
// row's tail floats. Returns off | shift << 8.
__device__ __forceinline__ int issue_row(float *abuf, float *bbuf, const RowLoc &loc,
                                         const float *ac, const float *bd, long long ac_total,
                                         long long bd_total, unsigned long long *bar, int li) {
  if (!loc.valid) {
    if (li == 0) mbar_arrive_tx(bar, 0);
    return 0;
  }
  const Span sa = span_of(loc.ac, loc.T, ac_total);
  const Span sb = span_of(loc.bd, loc.T, bd_total);
  const int d = sb.off - sa.off;   // -3 .. 3
  const int pad = d < 0 ? 4 : 0;
  if (li == 0) mbar_arrive_tx(bar, sa.bytes + sb.bytes);
  span_issue(abuf, ac, sa, bar, li);
  span_issue(bbuf + pad, bd, sb, bar, li);
  return sa.off | ((d + pad) << 8);
}

// v[k] = (ac + bd) * scale for the chunks q0 + LPR k, the band cut at shift SH.
template <int SH, int NCH, int LPR>
__device__ __forceinline__ void combine_chunks(float4 (&v)[NCH], const float *sa, const float *sbd,
                                               int q0, float scale) {
#pragma unroll
  for (int k = 0; k < NCH; k++) {
    const int q = q0 + LPR * k;
    const float4 a = ld4(sa + 4 * q);
    const float4 lo = ld4(sbd + 4 * q);
    float4 b = lo;
    if (SH != 0) {
      const float4 hi = ld4(sbd + 4 * q + 4);
      if (SH == 1) b = make_float4(lo.y, lo.z, lo.w, hi.x);
      if (SH == 2) b = make_float4(lo.z, lo.w, hi.x, hi.y);
      if (SH == 3) b = make_float4(lo.w, hi.x, hi.y, hi.z);
    }
    const float2 c01 = mul2(add2(make_float2(a.x, a.y), make_float2(b.x, b.y)), splat2(scale));
    const float2 c23 = mul2(add2(make_float2(a.z, a.w), make_float2(b.z, b.w)), splat2(scale));
    v[k] = make_float4(c01.x, c01.y, c23.x, c23.y);
  }
}

__device__ __forceinline__ float max4(float4 v) {
  return fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
}

template <int LPR>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(PK_FULL_MASK, v, o));
  return v;
}
template <int LPR>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(PK_FULL_MASK, v, o);
  return v;
}

// 1/s as the IEEE quotient: the fast reciprocal is exact on [1, 2^126), where
// every softmax sum lies unless the row holds +-inf or NaN.
__device__ __forceinline__ float recip_sum(float s) {
  return (s >= 1.0f && s < 0x1p126f) ? rcp_1_2e126(s) : __frcp_rn(s);
}

// A ring slot's row: ac offset, length and off | shift << 8 | valid << 16.
struct SlotRow {
  long long ac;
  int T, pk;
};

// Computes one group's rows from ring slot `slot` (see the kernel).
template <int NCH, int ROWS, bool SOFTMAX>
__device__ __forceinline__ void score_rows(const float *sa, const SlotRow &cur, float *S,
                                           float scale, int li);

// Shared memory per warp: NB (ring depth) buffers x ROWS rows x (ac, bd) x stg floats.
template <int NCH, int ROWS, bool SOFTMAX, int NB>
__global__ void __launch_bounds__(32 * PIPE_WARPS)
relpos_scores_pipe_kernel(const float *ac, const float *__restrict__ bd, float *S, float scale,
                          SeqDev seq, unsigned total_rows, long long ac_total, long long bd_total,
                          unsigned rows_per_warp) {
  constexpr int LPR = 32 / ROWS;
  constexpr int STG = 4 * LPR * NCH + 8;   // floats per staged ac row or bd band
  extern __shared__ float4 pipe_smem4[];
  __shared__ unsigned long long bars[PIPE_WARPS][NB];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR, li = lane % LPR;
  // buffer b, row g: ac at wb + ((b * ROWS + g) * 2) * STG, bd STG floats later
  float *wb = reinterpret_cast<float *>(pipe_smem4) + (size_t)warp * NB * ROWS * 2 * STG;
  unsigned long long *bar = bars[warp];
  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < NB; b++) mbar_init(bar + b, ROWS);
    mbar_init_fence();
  }
  __syncwarp();
  const unsigned wid = blockIdx.x * PIPE_WARPS + warp;
  const unsigned long long first = (unsigned long long)wid * rows_per_warp;
  if (first >= total_rows) return;
  const unsigned r_end = (unsigned)min((unsigned long long)total_rows, first + rows_per_warp);
  const bool uniform = seq.uniform_T > 0;
  const int uT = uniform ? seq.uniform_T : 1;
  // ring: slot n % NB holds group n; groups 0 .. NB-2 are issued up
  // front, group n + NB - 1 while group n is computed. The loop is unrolled
  // over the slots so that each slot's row record stays in registers.
  SlotRow slot[NB];
  unsigned irow = (unsigned)first + g;   // this group's row of the next group to issue
  int iu = uniform ? (int)(irow % (unsigned)uT) : 0;
  auto issue = [&](int b) -> SlotRow {
    const RowLoc loc = uniform ? uniform_row(irow, r_end, uT, iu) : locate_row(seq, irow, r_end);
    float *p = wb + ((b * ROWS + g) * 2) * STG;
    const int pk = issue_row(p, p + STG, loc, ac, bd, ac_total, bd_total, bar + b, li);
    irow += ROWS;
    if (uniform) {
      iu += ROWS;
      while (iu >= uT) iu -= uT;
    }
    SlotRow r;
    r.ac = loc.ac;
    r.T = loc.T;
    r.pk = pk | (loc.valid ? 1 << 16 : 0);
    return r;
  };
#pragma unroll
  for (int b = 0; b < NB - 1; b++) slot[b] = issue(b);
  unsigned parity = 0;   // bit b: phase parity of buffer b's next completion
  unsigned base = (unsigned)first;
  while (true) {
#pragma unroll
    for (int b = 0; b < NB; b++) {   // compile-time slot b computes group n
      if (base >= r_end) return;       // nothing in flight: later groups are past the range
      slot[(b + NB - 1) % NB] = issue((b + NB - 1) % NB);   // the slot freed last
      const bool ok = mbar_wait(bar + b, (parity >> b) & 1);
      if (__any_sync(PK_FULL_MASK, !ok)) {   // a copy never landed: give up this warp
        if (lane == 0) atomicAdd(&g_wait_timeouts, 1u);
#pragma unroll
        for (int o = 0; o < NB; o++)
          if (o != b) mbar_wait(bar + o, (parity >> o) & 1);
        return;
      }
      parity ^= 1u << b;
      __syncwarp();   // tail floats copied by other lanes are visible
      score_rows<NCH, ROWS, SOFTMAX>(wb + ((b * ROWS + g) * 2) * STG, slot[b], S, scale, li);
      __syncwarp();   // every lane is done with this buffer before it is refilled
      base += ROWS;
    }
  }
}

template <int NCH, int ROWS, bool SOFTMAX>
__device__ __forceinline__ void score_rows(const float *sa, const SlotRow &cur, float *S,
                                           float scale, int li) {
  constexpr int LPR = 32 / ROWS;
  constexpr int STG = 4 * LPR * NCH + 8;
  const bool valid = (cur.pk >> 16) & 1;
  {   // every lane runs the group reductions; stores only for a valid row
      const float *sbd = sa + STG;
      const int T = cur.T, off = cur.pk & 0xff, sh = (cur.pk >> 8) & 0xff;
      const int len8 = T & ~7;
      const int q_lo = off > 0 ? 1 : 0;
      const int q_hi = (len8 + off) >> 2;   // chunks [q_lo, q_hi) lie inside [0, len8)
      const int n_head = off > 0 ? min(4 - off, T) : 0;
      const int tail0 = q_hi > q_lo ? 4 * q_hi - off : n_head;
      const int n_left = n_head + (T - tail0);
      // leftover entry of this lane (li < n_left)
      const int jl = li < n_head ? li : tail0 + (li - n_head);
      const bool has_left = li < n_left;
      float vl = 0.0f;
      if (has_left) vl = (sa[off + jl] + sbd[off + sh + jl]) * scale;
      const int q0 = q_lo + li;
      float4 v[NCH];
      switch (sh) {
        case 0: combine_chunks<0, NCH, LPR>(v, sa, sbd, q0, scale); break;
        case 1: combine_chunks<1, NCH, LPR>(v, sa, sbd, q0, scale); break;
        case 2: combine_chunks<2, NCH, LPR>(v, sa, sbd, q0, scale); break;
        default: combine_chunks<3, NCH, LPR>(v, sa, sbd, q0, scale); break;
      }
      float el = vl;   // the leftover entry's output
      if (SOFTMAX) {
        float mx = has_left ? vl : -INFINITY;
#pragma unroll
        for (int k = 0; k < NCH; k++)
          if (q0 + LPR * k < q_hi) mx = fmaxf(mx, max4(v[k]));
        mx = group_max<LPR>(mx);
        float2 s2 = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < NCH; k++) {   // polynomial exp (every main entry is below len8)
          float2 d01 = sub2(make_float2(v[k].x, v[k].y), splat2(mx));
          float2 d23 = sub2(make_float2(v[k].z, v[k].w), splat2(mx));
          d01.x = fmaxf(d01.x, -87.0f);   // arguments are <= 0 or NaN
          d01.y = fmaxf(d01.y, -87.0f);
          d23.x = fmaxf(d23.x, -87.0f);
          d23.y = fmaxf(d23.y, -87.0f);
          const float2 e01 = exp_poly2_clamped(d01), e23 = exp_poly2_clamped(d23);
          if (q0 + LPR * k < q_hi) s2 = add2(s2, add2(e01, e23));
          v[k] = make_float4(e01.x, e01.y, e23.x, e23.y);
        }
        // leftovers: polynomial below len8, libm expf on the len % 8 tail
        el = 0.0f;
        if (has_left) {
          const float d = vl - mx;
          el = jl < len8 ? exp_poly_nonpos(d) : expf(d);
        }
        const float inv = recip_sum(group_sum<LPR>(s2.x + s2.y + el));
        const float2 inv2 = splat2(inv);
#pragma unroll
        for (int k = 0; k < NCH; k++) {
          const float2 o01 = mul2(make_float2(v[k].x, v[k].y), inv2);
          const float2 o23 = mul2(make_float2(v[k].z, v[k].w), inv2);
          v[k] = make_float4(o01.x, o01.y, o23.x, o23.y);
        }
        el = el * inv;
      }
      if (valid) {
        float *dst = S + cur.ac - off;   // 16-byte aligned
#pragma unroll
        for (int k = 0; k < NCH; k++)
          if (q0 + LPR * k < q_hi) st4(dst + 4 * (q0 + LPR * k), v[k]);
        if (has_left) S[cur.ac + jl] = el;
      }
  }
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

template <int NCH, int ROWS, bool SOFTMAX, int NB = NBUF>
static void launch_scores_pipe(const float *ac, const float *bd, float *S, float scale,
                               const pkcu_seq *seq, cudaStream_t s) {
  constexpr int STG = 4 * (32 / ROWS) * NCH + 8;
  const size_t smem = sizeof(float) * NB * ROWS * 2 * (size_t)STG * PIPE_WARPS;
  static int flags[64];
  smem_optin(relpos_scores_pipe_kernel<NCH, ROWS, SOFTMAX, NB>, smem, flags);
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, relpos_scores_pipe_kernel<NCH, ROWS, SOFTMAX, NB>,
                                                32 * PIPE_WARPS, smem);
  if (per_sm < 1) per_sm = 1;
  const long long rows = (long long)PK_H * seq->frames;
  long long grid = (rows + PIPE_WARPS * ROWS - 1) / (PIPE_WARPS * ROWS);
  const long long cap = (long long)pkcu_sm_count() * per_sm;
  if (grid > cap) grid = cap;
  // contiguous row ranges, a multiple of ROWS rows per warp
  const long long warps = grid * PIPE_WARPS;
  long long per_warp = (rows + warps - 1) / warps;
  per_warp = (per_warp + ROWS - 1) / ROWS * ROWS;
  relpos_scores_pipe_kernel<NCH, ROWS, SOFTMAX, NB><<<(unsigned)grid, 32 * PIPE_WARPS, smem, s>>>(
      ac, bd, S, scale, seq->dev, (unsigned)rows, seq->score_elems, seq->bd_elems,
      (unsigned)per_warp);
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
  // chunks per lane: a row of T entries at offset off <= 3 spans (T + 6) / 4
  // chunks; two rows per warp (16 lanes each) up to 8 chunks per lane, one
  // row per warp above that
  const int nq = (T + 6) / 4;
  // The pipelined kernel needs a few dozen rows per warp to cover its ring's
  // ramp; below about 32 rows per warp of a full wave (12 warps per SM) the
  // one-warp-per-row kernel is faster (8 chunks of 416 frames: 34.9 against
  // 38.4 us).
  const bool few_rows = (long long)PK_H * seq->frames < (long long)pkcu_sm_count() * 12 * 32;
  if (PK_ALIGNED16(ac) && PK_ALIGNED16(bd) && PK_ALIGNED16(S) && nq <= 32 * 8 && pipe_rows_fit(seq) &&
      !(few_rows && npl <= 32)) {
    // measured at 256 x 375 / 256 x 416: two rows per warp up to 6 chunks per
    // lane (<6, 2>: 0.59 ms); one row per warp above (<4, 1>: 0.72 ms at
    // T = 416, against 0.97 ms for <8, 2>, whose 90 registers and 66 KB per
    // CTA left six warps per SM)
    if (nq <= 16 * 1) launch_scores_pipe<1, 2, SOFTMAX>(ac, bd, S, scale, seq, s);
    else if (nq <= 16 * 2) launch_scores_pipe<2, 2, SOFTMAX>(ac, bd, S, scale, seq, s);
    else if (nq <= 16 * 4) launch_scores_pipe<4, 2, SOFTMAX>(ac, bd, S, scale, seq, s);
    else if (nq <= 16 * 6) launch_scores_pipe<6, 2, SOFTMAX>(ac, bd, S, scale, seq, s);
    else if (nq <= 32 * 4) launch_scores_pipe<4, 1, SOFTMAX>(ac, bd, S, scale, seq, s);
    else if (nq <= 32 * 6) launch_scores_pipe<6, 1, SOFTMAX>(ac, bd, S, scale, seq, s);
    else launch_scores_pipe<8, 1, SOFTMAX>(ac, bd, S, scale, seq, s);
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
  // two rows per warp for rows of 129..512 entries
  constexpr int ROWS = (NPL >= 8 && NPL <= 16) ? 2 : 1;
  const long long per_cta = (long long)SM_ROWS_PER_CTA * ROWS;
  const unsigned grid = (unsigned)((n_rows + per_cta - 1) / per_cta);
  softmax_rows_warp_kernel<NPL, ROWS><<<grid, 32 * SM_ROWS_PER_CTA, 0, s>>>(x, n_rows, len);
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

PK_WAIT_TIMEOUTS_ACCESSOR(pk_softmax_wait_timeouts)

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
