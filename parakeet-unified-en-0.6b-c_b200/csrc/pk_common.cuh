// pk_common.cuh -- device helpers shared by the sm_100a kernels of the
// non-GEMM encoder ops (LayerNorm, softmax, rel-pos scores, Swish, GLU,
// depthwise conv, residuals, dequant, joint, argmax).
//
// All kernel translation units are compiled with --fmad=false: a multiply and
// an add round separately unless the code calls fmaf(), which is where the
// reference's AVX2 path (csrc/tensor_ops.c, csrc/encoder.c) fuses them.
#pragma once

#include <cuda_runtime.h>
#include <mutex>
#include <stdint.h>

#include "pkcuda_internal.h"

#define PK_FULL_MASK 0xffffffffu

namespace pk {

// ── reductions ───────────────────────────────────────────────────────────────

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(PK_FULL_MASK, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(PK_FULL_MASK, v, o));
  return v;
}

// Sum over a CTA whose size is a multiple of 32; every thread gets the result.
// red must hold 33 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < nw ? red[lane] : 0.0f;
    t = warp_sum(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ float block_max(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < nw ? red[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// ── the reference's polynomial exp ───────────────────────────────────────────
//
// Restates pk_exp_avx2 (csrc/tensor_ops.c:97-121) operation by operation so the
// GPU result is bit-identical to it: clamp to [-87, 87] (max first, so NaN
// becomes -87 as with _mm256_max_ps), k = round-half-even(x * log2 e),
// r = x - k ln2 as one fused multiply-add (the reference build contracts it),
// Horner evaluation of the degree-5 Taylor polynomial with FMAs, and 2^k built
// directly in the exponent field.
//
// The rounding uses the 1.5 * 2^23 shifter: for |t| < 2^22, t + 1.5*2^23 lands
// in [2^23, 2^24), where the float spacing is 1, so the add itself rounds t to
// the nearest integer, ties to even (the reference's _MM_FROUND_TO_NEAREST_INT),
// and the subtraction back is exact. The integer k sits in the low mantissa
// bits of the shifted value, so no float-to-int conversion is needed either:
// the whole function runs on the FMA/ALU pipes.
__device__ __forceinline__ float exp_poly_clamped(float x) {   // x in [-87, 87]
  constexpr float kShift = 12582912.0f;   // 1.5 * 2^23, bit pattern 0x4B400000
  const float shifted = __fadd_rn(__fmul_rn(x, 1.44269504088896341f), kShift);
  const float kf = __fsub_rn(shifted, kShift);
  const float r = fmaf(-kf, 0.69314718055994529f, x);
  float y = 1.0f / 120.0f;
  y = fmaf(y, r, 1.0f / 24.0f);
  y = fmaf(y, r, 1.0f / 6.0f);
  y = fmaf(y, r, 0.5f);
  y = fmaf(y, r, 1.0f);
  y = fmaf(y, r, 1.0f);
  // (k + 127) << 23 with k = bits(shifted) - 0x4B400000
  const int pow2k = (__float_as_int(shifted) - (0x4B400000 - 127)) << 23;
  return __fmul_rn(y, __int_as_float(pow2k));
}

__device__ __forceinline__ float exp_poly(float x) {
  // fmaxf returns -87 for a NaN x, like _mm256_max_ps(x, -87); the result is
  // then never NaN, so fminf is the plain upper clamp.
  return exp_poly_clamped(fminf(fmaxf(x, -87.0f), 87.0f));
}

// exp_poly for arguments that are <= 0 or NaN (softmax's x - max): the upper
// clamp cannot change them.
__device__ __forceinline__ float exp_poly_nonpos(float x) {
  return exp_poly_clamped(fmaxf(x, -87.0f));
}

// ── packed fp32 pairs (sm_100 f32x2 arithmetic) ──────────────────────────────
// add/sub/mul/fma.rn.f32x2 apply one IEEE fp32 operation, round to nearest,
// to each half of a register pair: the results are those of the scalar
// instructions, at half the issue slots. Used where the kernels are bound by
// instruction issue (polynomial exp, Swish, depthwise taps, score combine).
//
// Two forms of the same operations, chosen per kernel by measurement:
//   F2Ptx  inline PTX (the default: add2 / sub2 / mul2 / fma2 below). Faster in
//          the Swish and int4 dequant kernels (0.87 / 0.73 of the copy
//          bandwidth against 0.80 / 0.64 with the other form).
//   F2Cu   CUDA's __fadd2_rn / __fmul2_rn / __ffma2_rn, which the compiler can
//          schedule and allocate as pairs: faster in the GLU + depthwise conv
//          kernel (204 against 219 us at 256 x 375, same box).
// Both give the same results. Either way a packed multiply feeding a packed add
// may be fused into one multiply-add by the assembler: where the separately
// rounded product matters (the exp's k), it is formed with scalar __fmul_rn.

struct F2Ptx {
  static __device__ __forceinline__ unsigned long long pk(float2 v) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
    return r;
  }
  static __device__ __forceinline__ float2 unpk(unsigned long long r) {
    float2 v;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
    return v;
  }
  static __device__ __forceinline__ float2 add(float2 a, float2 b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)));
    return unpk(r);
  }
  static __device__ __forceinline__ float2 sub(float2 a, float2 b) {
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)));
    return unpk(r);
  }
  static __device__ __forceinline__ float2 mul(float2 a, float2 b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)));
    return unpk(r);
  }
  static __device__ __forceinline__ float2 fma(float2 a, float2 b, float2 c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)), "l"(pk(c)));
    return unpk(r);
  }
};

struct F2Cu {   // a - b as a + (-b): the same IEEE result
  static __device__ __forceinline__ float2 add(float2 a, float2 b) { return __fadd2_rn(a, b); }
  static __device__ __forceinline__ float2 sub(float2 a, float2 b) {
    return __fadd2_rn(a, make_float2(-b.x, -b.y));
  }
  static __device__ __forceinline__ float2 mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
  static __device__ __forceinline__ float2 fma(float2 a, float2 b, float2 c) {
    return __ffma2_rn(a, b, c);
  }
};

__device__ __forceinline__ float2 add2(float2 a, float2 b) { return F2Ptx::add(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) { return F2Ptx::sub(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return F2Ptx::mul(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return F2Ptx::fma(a, b, c); }
__device__ __forceinline__ float2 splat2(float s) { return make_float2(s, s); }

// exp_poly_clamped on a pair (inputs already in [-87, 87]); per element the
// same operations as the scalar form. -kf*ln2 + x == kf*(-ln2) + x exactly.
// The product x * log2(e) is formed by two scalar __fmul_rn, which are never
// contracted: a packed multiply followed by the packed shifter add was fused
// into one multiply-add in the generated code (measured), and then k rounds
// differently from the reference wherever the rounded product is a tie k + 1/2
// (x = 1.03972077: the reference's k is 2, the fused form's 1).
template <class F = F2Ptx>
__device__ __forceinline__ float2 exp_poly2_clamped(float2 x) {
  constexpr float kShift = 12582912.0f;
  const float2 shifted = F::add(make_float2(__fmul_rn(x.x, 1.44269504088896341f),
                                            __fmul_rn(x.y, 1.44269504088896341f)),
                                splat2(kShift));
  const float2 kf = F::sub(shifted, splat2(kShift));
  const float2 r = F::fma(kf, splat2(-0.69314718055994529f), x);
  float2 y = splat2(1.0f / 120.0f);
  y = F::fma(y, r, splat2(1.0f / 24.0f));
  y = F::fma(y, r, splat2(1.0f / 6.0f));
  y = F::fma(y, r, splat2(0.5f));
  y = F::fma(y, r, splat2(1.0f));
  y = F::fma(y, r, splat2(1.0f));
  const int px = (__float_as_int(shifted.x) - (0x4B400000 - 127)) << 23;
  const int py = (__float_as_int(shifted.y) - (0x4B400000 - 127)) << 23;
  return F::mul(y, make_float2(__int_as_float(px), __int_as_float(py)));
}

// Correctly rounded 1/d for d in [1, 2^126): the hardware approximation
// followed by one fused Newton step, r = r0 + r0*(1 - d*r0). Over that range
// it equals the IEEE quotient (__frcp_rn) for every float: the library's
// self-test pkcu_selftest() checks all 1,056,964,608 inputs on the device.
// Swish's denominators 1 + exp_poly(-v) lie in [1, 6.1e37].
__device__ __forceinline__ float rcp_approx(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  return r;
}
__device__ __forceinline__ float rcp_1_2e126(float d) {
  const float r0 = rcp_approx(d);
  return fmaf(fmaf(-d, r0, 1.0f), r0, r0);
}
template <class F = F2Ptx>
__device__ __forceinline__ float2 rcp2_1_2e126(float2 d) {
  const float2 r0 = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  const float2 e = F::fma(make_float2(-d.x, -d.y), r0, splat2(1.0f));
  return F::fma(e, r0, r0);
}

template <class F = F2Ptx>
__device__ __forceinline__ float2 swish_poly2(float2 v) {
  float2 m = F::sub(splat2(0.0f), v);
  m.x = fminf(fmaxf(m.x, -87.0f), 87.0f);
  m.y = fminf(fmaxf(m.y, -87.0f), 87.0f);
  const float2 d = F::add(splat2(1.0f), exp_poly2_clamped<F>(m));
  return F::mul(v, rcp2_1_2e126<F>(d));
}

// Swish of the vector body of pk_swish (csrc/tensor_ops.c:383-388):
// v * (1 / (1 + exp(0 - v))). __frcp_rn is the correctly rounded reciprocal,
// i.e. the IEEE quotient 1/d.
__device__ __forceinline__ float swish_poly(float v) {
  const float e = exp_poly(__fsub_rn(0.0f, v));
  return __fmul_rn(v, rcp_1_2e126(__fadd_rn(1.0f, e)));
}

// Swish of the scalar tail of pk_swish (csrc/tensor_ops.c:389): x / (1 + expf(-x)).
__device__ __forceinline__ float swish_tail(float v) {
  return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
}

// Sigmoid gate of the GLU (csrc/encoder.c:462): 1 / (1 + expf(-b)).
__device__ __forceinline__ float sigmoid_libm(float b) {
  const float d = __fadd_rn(1.0f, expf(-b));   // in [1, inf]
  return d < 0x1p126f ? rcp_1_2e126(d) : __frcp_rn(d);
}

// ── the GLU gate (csrc/encoder.c:460-463: a * 1/(1 + expf(-b))) ───────────────
// The reference's build evaluates expf with glibc's vector exp; the gate here
// computes e^x from the hardware base-2 exponential instead, for |x| <= 86:
// k = round(x log2 e) with the 1.5 * 2^23 shifter (one FMA: the rounding to an
// integer happens in the add), f = x log2 e - k with log2 e split into its
// float value and the float of the remainder (two FMAs; |f| <= 0.5 + 2^-20),
// 2^f by ex2.approx.ftz on f in [-0.5, 0.5], times 2^k built in the exponent
// field (the shifted value's low bits are k, so bits(t) << 23 is k << 23 mod
// 2^32; the product is exact). Then 1 + e and its hardware reciprocal
// (rcp.approx, 1 ulp: the denominator lies in [1, 2.2e37], so the result is a
// normal float). The argument x = -(b + bias) is one FMA, b * -1 - bias, and is
// clamped to [-86, 86] first: past it the sigmoid is 1 or below 4.5e-38, where
// the reference gives 1 or below that (0 once expf overflows). The clamp keeps
// a NaN (max.NaN / min.NaN), which then runs through ex2 and the products: a
// NaN gate gives NaN as in the reference, with no select. Error against the
// correctly rounded sigmoid: a few units in the last place (checked on the
// device against glibc by a dense sweep), inside the GLU's tolerance.
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float clamp86_nan(float x) {
  float r;
  asm("{\n .reg .f32 t;\n max.NaN.f32 t, %1, 0fC2AC0000;\n min.NaN.f32 %0, t, 0f42AC0000;\n}"
      : "=f"(r) : "f"(x));
  return r;
}
// 2^k for the shifter value t = 1.5 * 2^23 + k
__device__ __forceinline__ float gate_pow2k(float t) {
  return __uint_as_float((__float_as_uint(t) << 23) + 0x3F800000u);
}
constexpr float GATE_L2E_HI = 1.44269502162933349609375f;   // float(log2 e)
constexpr float GATE_L2E_LO = 1.925963033500011e-08f;       // float(log2 e - GATE_L2E_HI)
constexpr float GATE_SHIFT = 12582912.0f;                   // 1.5 * 2^23

// a * sigmoid(g + bias) on a pair, nbg = -bias (-0 without one)
template <class F = F2Ptx>
__device__ __forceinline__ float2 glu_gate2(float2 a, float2 g, float2 nbg) {
  float2 m = F::fma(g, splat2(-1.0f), nbg);
  m.x = clamp86_nan(m.x);
  m.y = clamp86_nan(m.y);
  const float2 t = F::fma(m, splat2(GATE_L2E_HI), splat2(GATE_SHIFT));
  float2 f = F::fma(m, splat2(GATE_L2E_HI), F::sub(splat2(GATE_SHIFT), t));
  f = F::fma(m, splat2(GATE_L2E_LO), f);
  const float2 e = F::mul(make_float2(ex2_approx(f.x), ex2_approx(f.y)),
                          make_float2(gate_pow2k(t.x), gate_pow2k(t.y)));
  const float2 d = F::add(splat2(1.0f), e);
  return F::mul(a, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}
// The same operations on one value (bit-identical to either half of glu_gate2).
__device__ __forceinline__ float glu_gate(float a, float g, float nbg = -0.0f) {
  const float m = clamp86_nan(fmaf(g, -1.0f, nbg));
  const float t = fmaf(m, GATE_L2E_HI, GATE_SHIFT);
  float f = fmaf(m, GATE_L2E_HI, __fsub_rn(GATE_SHIFT, t));
  f = fmaf(m, GATE_L2E_LO, f);
  const float e = __fmul_rn(ex2_approx(f), gate_pow2k(t));
  return __fmul_rn(a, rcp_approx(__fadd_rn(1.0f, e)));
}

// ── exact division by a run-time divisor ─────────────────────────────────────
// n / d for n < 2^32 and 1 <= d < 2^32 as a 64-bit multiply-high with
// m = floor(2^64 / d) + 1: n*m/2^64 = n/d + err with 0 < err < 2^-32 <= 1/d,
// and the fractional part of n/d is at most 1 - 1/d, so the floor is exact.
// m = 0 stands for d = 1. Computed on the host once per launch.
struct FastDiv {
  unsigned long long m;
};
static inline FastDiv make_fastdiv(unsigned d) {
  FastDiv f;
  if (d <= 1) {
    f.m = 0;
  } else {
    const unsigned long long all = ~0ULL;   // 2^64 - 1
    f.m = all / d + (all % d == d - 1 ? 1 : 0) + 1;   // floor(2^64 / d) + 1
  }
  return f;
}
__device__ __forceinline__ unsigned fast_div(unsigned n, FastDiv f) {
  return f.m ? (unsigned)__umul64hi((unsigned long long)n, f.m) : n;
}

// ── ragged batches ───────────────────────────────────────────────────────────
//
// A batch of independent utterances / chunks with per-item frame counts T_b.
// Per-item tensors are concatenated item after item. Uniform batches carry
// no device arrays: every offset is computed from uniform_T.
using SeqDev = pkcu_seq_dev;

__device__ __forceinline__ int seq_T(const SeqDev &s, int b) {
  return s.uniform_T > 0 ? s.uniform_T : __ldg(s.T + b);
}
__device__ __forceinline__ long long seq_frame_off(const SeqDev &s, int b) {
  return s.uniform_T > 0 ? (long long)b * s.uniform_T : __ldg(s.frame_off + b);
}
__device__ __forceinline__ long long seq_score_off(const SeqDev &s, int b) {
  return s.uniform_T > 0 ? (long long)b * PK_H * s.uniform_T * s.uniform_T
                         : __ldg(s.score_off + b);
}
__device__ __forceinline__ long long seq_bd_off(const SeqDev &s, int b) {
  return s.uniform_T > 0 ? (long long)b * PK_H * s.uniform_T * (2LL * s.uniform_T - 1)
                         : __ldg(s.bd_off + b);
}
__device__ __forceinline__ long long seq_pos_off(const SeqDev &s, int b) {
  return s.uniform_T > 0 ? (long long)b * (2LL * s.uniform_T - 1) : __ldg(s.pos_off + b);
}

// ── memory helpers ───────────────────────────────────────────────────────────

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
// Read once: cache-streaming load (evict-first).
__device__ __forceinline__ float4 ldg4_stream(const float *p) {
  return __ldcs(reinterpret_cast<const float4 *>(p));
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                     __fadd_rn(a.w, b.w));
}

// ── asynchronous global -> shared copies (cp.async) ─────────────────────────
// Completion is tracked per thread by commit groups; a warp that reads data
// copied by other lanes waits for its own groups and then __syncwarp()s.

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Copies floats [start, start + n) of a 16-byte aligned array of `total`
// floats into dst (16-byte aligned) as 16-byte chunks of the aligned superset
// [start & ~3, ...): dst[k] holds src[(start & ~3) + k]. Chunks that would run
// past the end of the array fall back to 4-byte copies. Returns start & 3,
// the offset of src[start] in dst. Warp-cooperative.
__device__ __forceinline__ int cp_async_span(float *dst, const float *src, long long start, int n,
                                             long long total, int lane) {
  const long long a0 = start & ~3LL;
  long long a1 = (start + n + 3) & ~3LL;
  const long long lim = total & ~3LL;
  if (a1 > lim) a1 = lim > a0 ? lim : a0;
  const int n16 = (int)((a1 - a0) >> 2);
  for (int q = lane; q < n16; q += 32) cp_async16(dst + 4 * q, src + a0 + 4 * q);
  for (long long e = a1 + lane; e < start + n; e += 32) cp_async4(dst + (e - a0), src + e);
  return (int)(start - a0);
}

// ── bulk asynchronous copies (TMA engine) with mbarrier completion ──────────
// One thread issues cp.async.bulk (no multicast) for a whole 16-byte aligned
// span; the copy engine signals the bytes it wrote on a shared-memory mbarrier
// that the consumers wait on. Waits are bounded by the global nanosecond
// timer: a wait that runs out counts a timeout in the translation unit's
// g_wait_timeouts (read by the host through pkcu_wait_timeouts()) and the
// kernel abandons its work instead of spinning forever.

__device__ __forceinline__ unsigned smem_u32(const void *p) {
  return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(unsigned long long *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes initialised mbarriers visible to the copy engine.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(unsigned long long *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes,
                                         unsigned long long *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long *bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr unsigned long long PK_WAIT_NS = 1000000000ULL;   // 1 s per wait

// Waits that ran out in this translation unit's kernels since the last reset.
static __device__ unsigned g_wait_timeouts;

// Host accessor of g_wait_timeouts for one translation unit (current device).
#define PK_WAIT_TIMEOUTS_ACCESSOR(fn)                                              \
  extern "C" int fn(unsigned *count, int reset) {                                  \
    unsigned v = 0;                                                                \
    if (cudaMemcpyFromSymbol(&v, pk::g_wait_timeouts, sizeof v) != cudaSuccess)    \
      return PKCU_ERR_CUDA;                                                        \
    if (reset) {                                                                   \
      const unsigned zero = 0;                                                     \
      if (cudaMemcpyToSymbol(pk::g_wait_timeouts, &zero, sizeof zero) != cudaSuccess) \
        return PKCU_ERR_CUDA;                                                      \
    }                                                                              \
    *count = v;                                                                    \
    return PKCU_OK;                                                                \
  }

// Waits until phase `parity` of bar has completed, at most `limit_ns`.
__device__ __forceinline__ bool mbar_wait(unsigned long long *bar, unsigned parity,
                                          unsigned long long limit_ns = PK_WAIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > limit_ns) return false;
  return true;
}

// Geometry of one row of n floats starting at element `start` of a 16-byte
// aligned array of `total` floats, copied as its 16-byte aligned superset:
// dst[k] = src[a0 + k] for k < bytes / 4 (bulk), then the n_tail floats that
// a 16-byte chunk would have read past the array's end as plain loads, at
// dst[bytes / 4 ...]. off = start - a0 is the row's offset in dst.
struct Span {
  long long a0;
  unsigned bytes;
  int n_tail, off;
};
__device__ __forceinline__ Span span_of(long long start, int n, long long total) {
  Span s;
  s.a0 = start & ~3LL;
  long long a1 = (start + n + 3) & ~3LL;
  const long long lim = total & ~3LL;
  if (a1 > lim) a1 = lim > s.a0 ? lim : s.a0;
  s.bytes = (unsigned)(a1 - s.a0) * 4u;
  const long long tail = start + n - a1;
  s.n_tail = tail > 0 ? (int)tail : 0;
  s.off = (int)(start - s.a0);
  return s;
}
// Asks the copy engine to bring a span into L2 (no completion to wait for).
__device__ __forceinline__ void prefetch_l2(const float *src, const Span &s) {
  if (s.bytes)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src + s.a0), "r"(s.bytes)
                 : "memory");
}

// Lane 0 issues the bulk copy of a span (its bytes are part of an
// expect-tx already posted on bar); lanes < n_tail copy the tail floats.
__device__ __forceinline__ void span_issue(float *dst, const float *src, const Span &s,
                                           unsigned long long *bar, int lane) {
  if (lane == 0 && s.bytes) bulk_g2s(dst, src + s.a0, s.bytes, bar);
  if (lane < s.n_tail) dst[s.bytes / 4 + lane] = src[s.a0 + s.bytes / 4 + lane];
}

// Raises a kernel's dynamic shared-memory limit once per device (the first
// launch on each device; later launches, including ones under stream
// capture, make no attribute call). `flags` is a per-kernel static array of
// the size raised so far per device: read atomically on the fast path, raised
// under one process-wide lock so that concurrent first calls from several
// host threads never leave a smaller limit recorded than set.
inline std::mutex &smem_optin_lock() {
  static std::mutex m;
  return m;
}
template <typename K>
inline void smem_optin(K kernel, size_t bytes, int *flags) {
  const int dev = pkcu_device();
  if (dev < 64 && __atomic_load_n(&flags[dev], __ATOMIC_ACQUIRE) >= (int)bytes) return;
  std::lock_guard<std::mutex> lock(smem_optin_lock());
  if (dev < 64 && flags[dev] >= (int)bytes) return;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
      cudaSuccess)
    return;   // the launch that follows reports the error
  if (dev < 64) __atomic_store_n(&flags[dev], (int)bytes, __ATOMIC_RELEASE);
}

}  // namespace pk
