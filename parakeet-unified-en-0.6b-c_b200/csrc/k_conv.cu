// k_conv.cu -- convolution-module ops: GLU and the depthwise conv with its
// bias, optional BatchNorm and Swish.
//
// GLU (csrc/encoder.c:454-465): the pointwise-conv output pw1 [2C, T] gets its
// bias (csrc/tensor_ops.c:585-589), then out[c,t] = a * 1/(1 + expf(-g)) with
// a = pw1[c,t], g = pw1[C+c,t]. Per item the [C, T] halves are contiguous, so
// the kernel streams both halves as flat float4 arrays (12 bytes per output).
// The gate's exp is the library's own (glu_gate, pk_common.cuh); the
// reference's -ffast-math build uses glibc's vectorised expf, so GLU is
// compared within tolerance.
//
// Depthwise conv (csrc/tensor_ops.c:477-575): out[c,t] = b[c] + sum_k
// x[c, t-pad+k] * w[c,k], pad = (K-1)/2, taps outside [0, T) skipped, the sum
// accumulated in k order as a fused multiply-add chain from the bias (the
// reference's vectorised interior). Then optional inference BatchNorm
// ((y - mean)/sqrtf(var + eps))*gamma + beta and optional Swish (the pk_swish
// call of csrc/encoder.c:470, polynomial on the first 8*floor(C*T/8) entries of
// the item). One warp per channel row; 128-output chunks of the row plus the
// K-1 halo are staged in shared memory so every input element is read from HBM
// once (8 bytes per output).
#include <math.h>

#include "pk_common.cuh"

namespace pk {

constexpr int GLU_THREADS = 256;
constexpr int DW_WARPS = 8;
constexpr int DW_CHUNK = 128;
constexpr int DW_MAX_K = PK_DW_MAX_K;
constexpr int DW_SMEM_PER_WARP = DW_CHUNK + DW_MAX_K - 1;

__device__ __forceinline__ float glu1(float a, float g) { return glu_gate(a, g); }

// Channel-first GLU over each item's [2C, T] block.
__global__ void __launch_bounds__(GLU_THREADS)
glu_cf_kernel(const float *__restrict__ in, const float *__restrict__ bias, float *__restrict__ out,
              int C, SeqDev seq, int vec) {
  const int item = blockIdx.y;
  const int T = seq_T(seq, item);
  const long long f0 = seq_frame_off(seq, item);
  const long long n = (long long)C * T;
  const float *A = in + 2 * f0 * C;
  const float *G = A + n;
  float *O = out + f0 * C;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec) {
    for (; i < (n >> 2); i += stride) {
      const long long e = 4 * i;
      float4 a = ldg4_stream(A + e), g = ldg4_stream(G + e);
      if (bias) {
        int d = (int)(e / T), r = (int)(e - (long long)d * T);
        float av[4] = {a.x, a.y, a.z, a.w}, gv[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
          av[k] = av[k] + __ldg(bias + d);
          gv[k] = gv[k] + __ldg(bias + C + d);
          if (++r == T) { r = 0; d++; }
        }
        a = make_float4(av[0], av[1], av[2], av[3]);
        g = make_float4(gv[0], gv[1], gv[2], gv[3]);
      }
      st4(O + e, make_float4(glu1(a.x, g.x), glu1(a.y, g.y), glu1(a.z, g.z), glu1(a.w, g.w)));
    }
  } else {
    for (; i < n; i += stride) {
      float a = A[i], g = G[i];
      if (bias) {
        const int d = (int)(i / T);
        a = a + bias[d];
        g = g + bias[C + d];
      }
      O[i] = glu1(a, g);
    }
  }
}

// Time-first GLU: rows [2C] -> [C], split along the channel axis.
__global__ void __launch_bounds__(GLU_THREADS)
glu_tf_kernel(const float *__restrict__ in, const float *__restrict__ bias, float *__restrict__ out,
              int C, long long n) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / C;
    const int c = (int)(e - row * C);
    float a = in[row * 2 * C + c], g = in[row * 2 * C + C + c];
    if (bias) { a = a + bias[c]; g = g + bias[C + c]; }
    out[e] = glu1(a, g);
  }
}

// The depthwise conv's input row c of an item, read either plainly (x per
// item [C, T]) or, with the GLU folded in, from the pointwise-conv output
// pw1 per item [2C, T]: in[c, t] = a * sigmoid(g), a = pw1[c, t] (+ bias[c]),
// g = pw1[C + c, t] (+ bias[C + c]) -- the same operations as glu_cf_kernel,
// so the fused result is bit-identical to GLU followed by the conv.
struct DwIn {
  const float *src;
  long long base;      // element offset of row c (or of the a-row with GLU)
  long long gate;      // offset from the a-row to the g-row (C * T)
  float ba, bg;
  bool bias;
};

__device__ __forceinline__ DwIn dw_in_row(const float *src, const float *glu_bias, bool glu,
                                          const SeqDev &seq, int item, int c, int C, int T) {
  DwIn r;
  r.src = src;
  const long long f0 = seq_frame_off(seq, item);
  r.base = (glu ? 2 * f0 * C : f0 * C) + (long long)c * T;
  r.gate = (long long)C * T;
  r.bias = glu && glu_bias != nullptr;
  r.ba = r.bias ? __ldg(glu_bias + c) : 0.0f;
  r.bg = r.bias ? __ldg(glu_bias + C + c) : 0.0f;
  return r;
}

template <bool GLU>
__device__ __forceinline__ float dw_in(const DwIn &in, int tt) {
  if (!GLU) return __ldcs(in.src + in.base + tt);
  float a = __ldcs(in.src + in.base + tt), g = __ldcs(in.src + in.base + in.gate + tt);
  if (in.bias) {
    a = a + in.ba;
    g = g + in.bg;
  }
  return glu1(a, g);
}

// KC > 0: compile-time kernel width (taps in registers); KC == 0: runtime K.
template <int KC>
__global__ void __launch_bounds__(32 * DW_WARPS)
dwconv_kernel(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ b,
              const float *__restrict__ bn, float bn_eps, int apply_swish, float *__restrict__ out,
              int C, int Kr, SeqDev seq, int glu, const float *__restrict__ glu_bias) {
  __shared__ float stage[DW_WARPS][DW_SMEM_PER_WARP];
  const int K = KC > 0 ? KC : Kr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * DW_WARPS + warp;
  if (c >= C) return;
  const int item = blockIdx.y;
  const int T = seq_T(seq, item);
  const long long base = seq_frame_off(seq, item) * C + (long long)c * T;
  const DwIn in = dw_in_row(x, glu_bias, glu != 0, seq, item, c, C, T);
  const int pad = (K - 1) / 2;
  const long long n8 = ((long long)C * T) & ~7LL;
  float wk[KC > 0 ? KC : 1];
  if (KC > 0) {
#pragma unroll
    for (int k = 0; k < (KC > 0 ? KC : 1); k++) wk[k] = __ldg(w + (long long)c * K + k);
  }
  const float bias = b ? __ldg(b + c) : 0.0f;
  float mean = 0.0f, den = 1.0f, gam = 1.0f, bet = 0.0f;
  if (bn) {
    mean = __ldg(bn + c);
    den = sqrtf(__ldg(bn + C + c) + bn_eps);
    gam = __ldg(bn + 2 * C + c);
    bet = __ldg(bn + 3 * C + c);
  }
  float *s = stage[warp];
  for (int t0 = 0; t0 < T; t0 += DW_CHUNK) {
    for (int k = lane; k < DW_CHUNK + K - 1; k += 32) {
      const int tt = t0 - pad + k;
      s[k] = (tt >= 0 && tt < T) ? (glu ? dw_in<true>(in, tt) : dw_in<false>(in, tt)) : 0.0f;
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < DW_CHUNK / 32; j++) {
      const int o = lane + 32 * j;
      const int t = t0 + o;
      if (t >= T) break;
      float val = bias;
      if (KC > 0) {
#pragma unroll
        for (int k = 0; k < (KC > 0 ? KC : 1); k++) {
          const int tt = t - pad + k;
          if (tt >= 0 && tt < T) val = fmaf(s[o + k], wk[k], val);
        }
      } else {
        for (int k = 0; k < K; k++) {
          const int tt = t - pad + k;
          if (tt >= 0 && tt < T) val = fmaf(s[o + k], __ldg(w + (long long)c * K + k), val);
        }
      }
      if (bn) val = ((val - mean) / den) * gam + bet;
      if (apply_swish) {
        const long long flat = (long long)c * T + t;
        val = (flat < n8) ? swish_poly(val) : swish_tail(val);
      }
      out[base + t] = val;
    }
    __syncwarp();
  }
}

// K = 9 rows up to DW_ROW_MAX - 12 frames: the whole row plus its zero halo is
// staged in shared memory in one pass (every lane issues its loads back to
// back). Each lane then produces 4 consecutive outputs t = 4g..4g+3 from the 12
// staged values s[4g .. 4g+11] read as three 16-byte shared loads. Groups whose
// every tap lies inside [0, T) run without per-tap predicates; edge groups skip
// the out-of-range taps exactly as the reference does.
constexpr int DW_ROW_MAX = 640;

// Swish after the conv: none, polynomial only (C*T_b a multiple of 8, e.g.
// C = 1024), or with the scalar-tail rule for the last C*T_b % 8 entries.
enum { DW_SWISH_NONE = 0, DW_SWISH_POLY = 1, DW_SWISH_TAIL = 2 };

template <int SW, bool BN>
__device__ __forceinline__ float dw_finish(float val, float mean, float den, float gam, float bet,
                                           long long flat, long long n8) {
  if (BN) val = ((val - mean) / den) * gam + bet;
  if (SW == DW_SWISH_POLY) val = swish_poly(val);
  if (SW == DW_SWISH_TAIL) val = (flat < n8) ? swish_poly(val) : swish_tail(val);
  return val;
}

template <int KC, int SW, bool BN, bool GLU>
__global__ void __launch_bounds__(32 * DW_WARPS)
dwconv_row_kernel(const float *__restrict__ x, const float *__restrict__ w,
                  const float *__restrict__ b, const float *__restrict__ bn, float bn_eps,
                  float *__restrict__ out, int C, SeqDev seq, const float *__restrict__ glu_bias) {
  static_assert(KC == 9, "the 4-output register window assumes K = 9");
  __shared__ __align__(16) float stage[DW_WARPS][DW_ROW_MAX];
  constexpr int K = KC;
  constexpr int pad = (K - 1) / 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * DW_WARPS + warp;
  if (c >= C) return;
  const int item = blockIdx.y;
  const int T = seq_T(seq, item);
  const long long base = seq_frame_off(seq, item) * C + (long long)c * T;
  const DwIn in = dw_in_row(x, glu_bias, GLU, seq, item, c, C, T);
  float *s = stage[warp];
  const int n_groups = (T + 3) >> 2;
  const int n_stage = 4 * n_groups + 8;   // s[0 .. 4*n_groups + 7] are read
  // s[k] = in[k - pad], zero outside [0, T)
  if constexpr (GLU) {
    // Both GLU halves land in shared memory through async copies (every load
    // of the row in flight at once), then the gate is applied in place.
    __shared__ float stage_g[DW_WARPS][DW_ROW_MAX];
    float *sg = stage_g[warp];
    for (int k = lane; k < n_stage; k += 32) {
      const int tt = k - pad;
      if (tt >= 0 && tt < T) {
        cp_async4(s + k, in.src + in.base + tt);
        cp_async4(sg + k, in.src + in.base + in.gate + tt);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    for (int k = lane; k < n_stage; k += 32) {   // the same k as this lane copied
      const int tt = k - pad;
      float val = 0.0f;
      if (tt >= 0 && tt < T) {
        float a = s[k], g = sg[k];
        if (in.bias) {
          a = a + in.ba;
          g = g + in.bg;
        }
        val = glu1(a, g);
      }
      s[k] = val;
    }
  } else {
#pragma unroll 4
    for (int k = lane; k < n_stage; k += 32) {
      const int tt = k - pad;
      s[k] = (tt >= 0 && tt < T) ? dw_in<false>(in, tt) : 0.0f;
    }
  }
  float wk[K];
#pragma unroll
  for (int k = 0; k < K; k++) wk[k] = __ldg(w + (long long)c * K + k);
  const float bias = b ? __ldg(b + c) : 0.0f;
  float mean = 0.0f, den = 1.0f, gam = 1.0f, bet = 0.0f;
  if (BN) {
    mean = __ldg(bn + c);
    den = sqrtf(__ldg(bn + C + c) + bn_eps);
    gam = __ldg(bn + 2 * C + c);
    bet = __ldg(bn + 3 * C + c);
  }
  const long long n8 = ((long long)C * T) & ~7LL;
  const long long flat0 = (long long)c * T;
  __syncwarp();
  for (int g = lane; g < n_groups; g += 32) {
    const int t0 = 4 * g;
    const float4 a0 = *reinterpret_cast<const float4 *>(s + t0);
    const float4 a1 = *reinterpret_cast<const float4 *>(s + t0 + 4);
    const float4 a2 = *reinterpret_cast<const float4 *>(s + t0 + 8);
    const float win[12] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w,
                           a2.x, a2.y, a2.z, a2.w};
    float v[4];
    if (t0 >= pad && t0 + 3 + pad < T) {
      // outputs (t0, t0+1) and (t0+2, t0+3) as packed pairs; each output's
      // multiply-add chain runs in the same k order as the scalar form
      float2 v01 = splat2(bias), v23 = splat2(bias);
#pragma unroll
      for (int k = 0; k < K; k++) {
        v01 = fma2(make_float2(win[k], win[k + 1]), splat2(wk[k]), v01);
        v23 = fma2(make_float2(win[k + 2], win[k + 3]), splat2(wk[k]), v23);
      }
      v[0] = v01.x;
      v[1] = v01.y;
      v[2] = v23.x;
      v[3] = v23.y;
    } else {
#pragma unroll
      for (int q = 0; q < 4; q++) {
        float val = bias;
#pragma unroll
        for (int k = 0; k < K; k++) {
          const int tt = t0 + q - pad + k;
          if (tt >= 0 && tt < T) val = fmaf(win[q + k], wk[k], val);
        }
        v[q] = val;
      }
    }
    if (SW == DW_SWISH_POLY) {
#pragma unroll
      for (int q = 0; q < 4; q += 2) {
        float2 p = make_float2(v[q], v[q + 1]);
        if (BN) {
          p.x = ((p.x - mean) / den) * gam + bet;
          p.y = ((p.y - mean) / den) * gam + bet;
        }
        p = swish_poly2(p);
        v[q] = p.x;
        v[q + 1] = p.y;
      }
#pragma unroll
      for (int q = 0; q < 4; q++)
        if (t0 + q < T) out[base + t0 + q] = v[q];
    } else {
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const int t = t0 + q;
        if (t < T) out[base + t] = dw_finish<SW, BN>(v[q], mean, den, gam, bet, flat0 + t, n8);
      }
    }
  }
}

// ── aligned-chunk form (K = 9, C % 8 == 0, 16-byte aligned arrays) ──────────
// With C a multiple of 4 an item's input row c (x or either GLU half) and its
// output row start at the same offset mod 4 floats (off), so the work is cut
// into the 4-float chunks of that common alignment. Lane 0 of each warp copies
// the row (both GLU halves) into shared memory as the 16-byte aligned superset
// with one bulk copy per half, completion on the warp's mbarrier:
// s[4 + k] = row[(start & ~3) + k], so row entry t sits at s[4 + off + t] and
// chunk q (entries t = 4q + e - off) at s[4 + 4q + e].
//
// The GLU gate runs 4 entries at a time on the chunks wholly inside the row
// and one entry per lane on the at most 6 entries outside them (16 lanes per
// row, two rows per warp). The conv runs
// 4 outputs at a time on the chunks whose 9-tap windows s[4q .. 4q + 11] lie
// wholly inside the row -- packed tap chains, packed Swish, one 16-byte store
// -- and one output per lane, with the out-of-row taps skipped, on the at most
// 15 outputs near the row's ends. No lane runs an edge path inside the loops.
constexpr int DWA_ROW = 656;

__host__ __device__ constexpr int dwa_row_need(int T) { return 4 * ((T + 6) / 4) + 8; }

// GLU of 4 values as two packed pairs (bit-identical to glu1 on each value).
template <class F = F2Ptx>
__device__ __forceinline__ float4 glu4(float4 a, float4 g, float ba, float bg, bool bias) {
  if (bias) {
    const float2 a01 = F::add(make_float2(a.x, a.y), splat2(ba));
    const float2 a23 = F::add(make_float2(a.z, a.w), splat2(ba));
    a = make_float4(a01.x, a01.y, a23.x, a23.y);
  }
  // the gate's bias enters the gate's own first FMA, -(g + bg) = g * -1 - bg
  const float2 nbg = splat2(bias ? -bg : -0.0f);
  const float2 o01 = glu_gate2<F>(make_float2(a.x, a.y), make_float2(g.x, g.y), nbg);
  const float2 o23 = glu_gate2<F>(make_float2(a.z, a.w), make_float2(g.z, g.w), nbg);
  return make_float4(o01.x, o01.y, o23.x, o23.y);
}

template <int SW, bool BN>
__device__ __forceinline__ float dwa_finish(float val, float mean, float den, float gam, float bet) {
  if (BN) val = ((val - mean) / den) * gam + bet;
  if (SW == DW_SWISH_POLY) val = swish_poly(val);
  return val;
}

// Two channel rows per warp (lane group g = lane / 16 takes row 2w + g), so
// the copy issue, the parameter loads and the one-output-per-lane edge steps
// of both rows share their instructions (packed arithmetic in the F2Cu form,
// measured faster here); DWA_WARPS warps = 8 channels per CTA
// (C % 8 == 0 on this path, so every row of a CTA exists). Staging sized to the
// batch keeps nine such CTAs (36 warps) on an SM at T = 375; a persistent form
// with a two-buffer copy pipeline per warp (16 warps per SM) measured 0.64-0.67
// of the copy bandwidth against 0.82-0.88 for this one.
constexpr int DWA_WARPS = 4, DWA_RPW = 2, DWA_LPR = 32 / DWA_RPW;
constexpr int DWA_CH = DWA_WARPS * DWA_RPW;

template <int SW, bool BN, bool GLU>
__global__ void __launch_bounds__(32 * DWA_WARPS)
dwconv_al_kernel(const float *__restrict__ x, const float *__restrict__ w,
                 const float *__restrict__ b, const float *__restrict__ bn, float bn_eps,
                 float *__restrict__ out, int C, SeqDev seq, const float *__restrict__ glu_bias,
                 long long x_total, int rs) {
  static_assert(SW == DW_SWISH_NONE || SW == DW_SWISH_POLY, "no scalar Swish tail here");
  constexpr int K = 9;
  constexpr int LPR = DWA_LPR;
  // DWA_CH staging rows of rs floats (then DWA_CH more for the GLU gate half)
  extern __shared__ float4 dwa_smem4[];
  float *stage = reinterpret_cast<float *>(dwa_smem4);
  __shared__ unsigned long long bars[DWA_WARPS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane / LPR, li = lane % LPR;
  const int slot = warp * DWA_RPW + g;
  const int c = blockIdx.x * DWA_CH + slot;
  if (blockIdx.x * DWA_CH + warp * DWA_RPW >= C) return;   // whole warp
  const int item = blockIdx.y;
  const int T = seq_T(seq, item);
  const long long f0 = seq_frame_off(seq, item);
  const long long row = (GLU ? 2 * f0 * C : f0 * C) + (long long)c * T;
  float *s = stage + slot * rs;
  float *sg = stage + (GLU ? DWA_CH + slot : slot) * rs;
  unsigned long long *bar = bars + warp;
  if (lane == 0) {
    mbar_init(bar, DWA_RPW);   // one arrival per row
    mbar_init_fence();
  }
  __syncwarp();
  const Span sa = span_of(row, T, x_total);
  Span sgs = sa;
  if (GLU) sgs = span_of(row + (long long)C * T, T, x_total);
  if (li == 0) mbar_arrive_tx(bar, sa.bytes + (GLU ? sgs.bytes : 0u));
  span_issue(s + 4, x, sa, bar, li);
  if (GLU) span_issue(sg + 4, x, sgs, bar, li);
  // per-channel parameters while the copies are in flight
  float wk[K];
#pragma unroll
  for (int k = 0; k < K; k++) wk[k] = __ldg(w + (long long)c * K + k);
  const float bias = b ? __ldg(b + c) : 0.0f;
  const bool gbias = GLU && glu_bias != nullptr;
  const float ba = gbias ? __ldg(glu_bias + c) : 0.0f;
  const float bg = gbias ? __ldg(glu_bias + C + c) : 0.0f;
  float mean = 0.0f, den = 1.0f, gam = 1.0f, bet = 0.0f;
  if (BN) {
    mean = __ldg(bn + c);
    den = sqrtf(__ldg(bn + C + c) + bn_eps);
    gam = __ldg(bn + 2 * C + c);
    bet = __ldg(bn + 3 * C + c);
  }
  const int off = sa.off;
  const bool ok = mbar_wait(bar, 0);
  if (__any_sync(PK_FULL_MASK, !ok)) {   // the copy never landed: give up this row
    if (lane == 0) atomicAdd(&g_wait_timeouts, 1u);
    mbar_wait(bar, 0);
    return;
  }
  __syncwarp();   // tail floats copied by other lanes are visible
  if (GLU) {
    // chunks [g_lo, g_hi) lie wholly inside the row (entries 4q - off .. 4q - off + 3)
    const int g_lo = off > 0 ? 1 : 0;
    const int g_hi = (T + off) >> 2;
    const int n_head = off > 0 ? (4 - off < T ? 4 - off : T) : 0;
    const int tail0 = g_hi > g_lo ? 4 * g_hi - off : n_head;
    const int n_left = n_head + (T - tail0);
    for (int q = g_lo + li; q < g_hi; q += LPR)
      st4(s + 4 + 4 * q, glu4<F2Cu>(ld4(s + 4 + 4 * q), ld4(sg + 4 + 4 * q), ba, bg, gbias));
    if (li < n_left) {
      const int t = li < n_head ? li : tail0 + (li - n_head);
      float aa = s[4 + off + t], gg = sg[4 + off + t];
      if (gbias) {
        aa = aa + ba;
        gg = gg + bg;
      }
      s[4 + off + t] = glu1(aa, gg);
    }
    __syncwarp();
  }
  float *orow = out + f0 * C + (long long)c * T;   // orow - off is 16-byte aligned
  // output chunks [c_lo, c_hi] have every tap inside the row: 4q - off >= 4 and
  // 4q - off + 7 <= T - 1
  const int c_lo = 1 + ((off + 3) >> 2);
  const int c_hi = (T - 8 + off) >= 0 ? (T - 8 + off) >> 2 : -1;
  for (int q = c_lo + li; q <= c_hi; q += LPR) {
    const int t0 = 4 * q - off;
    const float4 a0 = ld4(s + 4 * q), a1 = ld4(s + 4 * q + 4), a2 = ld4(s + 4 * q + 8);
    const float win[12] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w,
                           a2.x, a2.y, a2.z, a2.w};
    // outputs (t0, t0+1) and (t0+2, t0+3) as packed pairs; each output's
    // multiply-add chain runs in the same k order as the scalar form
    float2 v01 = splat2(bias), v23 = splat2(bias);
#pragma unroll
    for (int k = 0; k < K; k++) {
      v01 = F2Cu::fma(make_float2(win[k], win[k + 1]), splat2(wk[k]), v01);
      v23 = F2Cu::fma(make_float2(win[k + 2], win[k + 3]), splat2(wk[k]), v23);
    }
    if (BN) {
      v01 = make_float2(((v01.x - mean) / den) * gam + bet, ((v01.y - mean) / den) * gam + bet);
      v23 = make_float2(((v23.x - mean) / den) * gam + bet, ((v23.y - mean) / den) * gam + bet);
    }
    if (SW == DW_SWISH_POLY) {
      v01 = swish_poly2<F2Cu>(v01);
      v23 = swish_poly2<F2Cu>(v23);
    }
    st4(orow + t0, make_float4(v01.x, v01.y, v23.x, v23.y));
  }
  // leftover outputs: [0, h_end) and [t_beg, T), one per lane
  const int h_end = c_hi >= c_lo ? 4 * c_lo - off : T;
  const int t_beg = c_hi >= c_lo ? 4 * c_hi - off + 4 : T;
  const int n_out = h_end + (T - t_beg);
  if (li < n_out) {
    const int t = li < h_end ? li : t_beg + (li - h_end);
    float val = bias;
#pragma unroll
    for (int k = 0; k < K; k++) {
      const int tt = t - 4 + k;
      if (tt >= 0 && tt < T) val = fmaf(s[4 + off + tt], wk[k], val);
    }
    orow[t] = dwa_finish<SW, BN>(val, mean, den, gam, bet);
  }
}

static unsigned per_item_grid(long long work, int n_items) {
  long long g = (work + GLU_THREADS - 1) / GLU_THREADS;
  long long cap = ((long long)pkcu_sm_count() * 16 + n_items - 1) / n_items;
  if (cap < 1) cap = 1;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

// glu != 0: x is the pointwise-conv output per item [2C, T] and the GLU (with
// glu_bias, may be NULL) is applied while staging.
static int launch_dwconv(const float *x, const float *w, const float *b, const float *bn,
                         float bn_eps, int apply_swish, float *out, int C, int K, SeqDev sd,
                         long long frames, cudaStream_t s, int glu = 0,
                         const float *glu_bias = nullptr) {
  dim3 grid((unsigned)((C + DW_WARPS - 1) / DW_WARPS), (unsigned)sd.n_items);
  if (K == 9 && C % DWA_CH == 0 && PK_ALIGNED16(x) && PK_ALIGNED16(out) &&
      dwa_row_need(sd.max_T) <= DWA_ROW) {
    const dim3 grid_al((unsigned)(C / DWA_CH), (unsigned)sd.n_items);
    const long long x_total = (glu ? 2 : 1) * frames * C;
    // staging sized for the batch's longest item (at most 42 KB), so shorter
    // batches keep more CTAs resident per SM
    const int rs = dwa_row_need(sd.max_T);
    const size_t smem = sizeof(float) * (size_t)(glu ? 2 : 1) * DWA_CH * rs;
#define PK_DW_AL(SWV, BNV, GLUV)                                                         \
  dwconv_al_kernel<SWV, BNV, GLUV><<<grid_al, 32 * DWA_WARPS, smem, s>>>(                \
      x, w, b, bn, bn_eps, out, C, sd, glu_bias, x_total, rs)
#define PK_DW_AL_SW(BNV, GLUV)                                  \
  do {                                                          \
    if (apply_swish) PK_DW_AL(DW_SWISH_POLY, BNV, GLUV);        \
    else PK_DW_AL(DW_SWISH_NONE, BNV, GLUV);                    \
  } while (0)
    if (bn) {
      if (glu) PK_DW_AL_SW(true, true); else PK_DW_AL_SW(true, false);
    } else {
      if (glu) PK_DW_AL_SW(false, true); else PK_DW_AL_SW(false, false);
    }
#undef PK_DW_AL_SW
#undef PK_DW_AL
  } else if (K == 9 && 4 * ((sd.max_T + 3) / 4) + 8 <= DW_ROW_MAX) {
    // every item's C*T_b is a multiple of 8 when C is: no scalar Swish tail
    const int sw = !apply_swish ? DW_SWISH_NONE : (C % 8 == 0 ? DW_SWISH_POLY : DW_SWISH_TAIL);
#define PK_DW_ROW(SWV, BNV, GLUV)                                                        \
  dwconv_row_kernel<9, SWV, BNV, GLUV><<<grid, 32 * DW_WARPS, 0, s>>>(x, w, b, bn, bn_eps, \
                                                                      out, C, sd, glu_bias)
#define PK_DW_ROW_SW(BNV, GLUV)                               \
  do {                                                        \
    if (sw == DW_SWISH_NONE) PK_DW_ROW(DW_SWISH_NONE, BNV, GLUV); \
    else if (sw == DW_SWISH_POLY) PK_DW_ROW(DW_SWISH_POLY, BNV, GLUV); \
    else PK_DW_ROW(DW_SWISH_TAIL, BNV, GLUV);                 \
  } while (0)
    if (bn) {
      if (glu) PK_DW_ROW_SW(true, true); else PK_DW_ROW_SW(true, false);
    } else {
      if (glu) PK_DW_ROW_SW(false, true); else PK_DW_ROW_SW(false, false);
    }
#undef PK_DW_ROW_SW
#undef PK_DW_ROW
  } else if (K == 9) {
    dwconv_kernel<9><<<grid, 32 * DW_WARPS, 0, s>>>(x, w, b, bn, bn_eps, apply_swish, out, C, K, sd,
                                                     glu, glu_bias);
  } else {
    dwconv_kernel<0><<<grid, 32 * DW_WARPS, 0, s>>>(x, w, b, bn, bn_eps, apply_swish, out, C, K, sd,
                                                     glu, glu_bias);
  }
  return PKCU_OK;
}

}  // namespace pk

using namespace pk;

PK_WAIT_TIMEOUTS_ACCESSOR(pk_conv_wait_timeouts)

extern "C" int pkcu_glu(const float *in, const float *bias, float *out, int C, int layout,
                        const pkcu_seq *seq, pkcu_stream_t stream) {
  if (!in || !out || !seq || C <= 0 ||
      (layout != PKCU_CHANNEL_FIRST && layout != PKCU_TIME_FIRST))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_glu: bad argument");
  if (seq->dev.n_items > 65535)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_glu: at most 65535 items per call");
  if (seq->frames == 0) return PKCU_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (layout == PKCU_CHANNEL_FIRST) {
    const int vec = (C % 4 == 0) && PK_ALIGNED16(in) && PK_ALIGNED16(out);
    const long long per = (long long)C * seq->dev.max_T;
    dim3 grid(per_item_grid(vec ? per / 4 : per, seq->dev.n_items), (unsigned)seq->dev.n_items);
    glu_cf_kernel<<<grid, GLU_THREADS, 0, s>>>(in, bias, out, C, seq->dev, vec);
  } else {
    const long long n = seq->frames * C;
    long long g = (n + GLU_THREADS * 4 - 1) / (GLU_THREADS * 4);
    if (g > (long long)pkcu_sm_count() * 32) g = (long long)pkcu_sm_count() * 32;
    glu_tf_kernel<<<(unsigned)g, GLU_THREADS, 0, s>>>(in, bias, out, C, n);
  }
  return pkcu_launch_status("pkcu_glu");
}

extern "C" int pkcu_dwconv_bn_swish(const float *x, const float *w, const float *b,
                                    const float *bn, float bn_eps, int apply_swish, float *out,
                                    int C, int K, const pkcu_seq *seq, pkcu_stream_t stream) {
  if (!x || !w || !out || !seq || C <= 0 || K <= 0 || K > DW_MAX_K)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_dwconv_bn_swish: bad argument (K must be 1..%d)",
                     DW_MAX_K);
  if (seq->dev.n_items > 65535)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_dwconv_bn_swish: at most 65535 items per call");
  if (seq->frames == 0) return PKCU_OK;
  launch_dwconv(x, w, b, bn, bn_eps, apply_swish, out, C, K, seq->dev, seq->frames,
                (cudaStream_t)stream);
  return pkcu_launch_status("pkcu_dwconv_bn_swish");
}

extern "C" int pkcu_glu_dwconv_bn_swish(const float *pw1, const float *pw1_bias, const float *w,
                                        const float *b, const float *bn, float bn_eps,
                                        int apply_swish, float *out, int C, int K,
                                        const pkcu_seq *seq, pkcu_stream_t stream) {
  if (!pw1 || !w || !out || !seq || C <= 0 || K <= 0 || K > DW_MAX_K)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_glu_dwconv_bn_swish: bad argument (K must be 1..%d)",
                     DW_MAX_K);
  if (seq->dev.n_items > 65535)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_glu_dwconv_bn_swish: at most 65535 items per call");
  if (seq->frames == 0) return PKCU_OK;
  launch_dwconv(pw1, w, b, bn, bn_eps, apply_swish, out, C, K, seq->dev, seq->frames,
                (cudaStream_t)stream, 1, pw1_bias);
  return pkcu_launch_status("pkcu_glu_dwconv_bn_swish");
}

extern "C" int pkcu_depthwise_conv1d(const float *x, const float *w, const float *b, float *out,
                                     int C, int T, int K, pkcu_stream_t stream) {
  if (!x || !w || !out || C < 0 || T < 0 || K <= 0 || K > DW_MAX_K)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_depthwise_conv1d: bad argument (K must be 1..%d)",
                     DW_MAX_K);
  if (C == 0 || T == 0) return PKCU_OK;
  pkcu_seq_dev sd = {1, T, T, nullptr, nullptr, nullptr, nullptr, nullptr};
  launch_dwconv(x, w, b, nullptr, 0.0f, 0, out, C, K, sd, T, (cudaStream_t)stream);
  return pkcu_launch_status("pkcu_depthwise_conv1d");
}
