// k_tcgemm.cu -- the library's own tcgen05 GEMM for weight products:
// C[M, N] = epilogue(A[M, K] W[K, N]) at fp32 accuracy on the bf16 tensor
// cores, for the reference's three weight storages (csrc/parakeet.h:52-57,
// dispatched by pk_wmatmul, csrc/tensor_ops.c:50-61): float32, int8 with one
// per-tensor scale (csrc/blas.c:759, dequantised while packing :526-558) and
// GPTQ int4 with group scales (csrc/blas.c:950, :780-843).
//
// Operands. The activation A is split into three bf16 parts a0 + a1 + a2
// (k_split.cu, one memory-bound pass; row m = [a0 | a1 | a2]). The weight is
// prepared once, K-major ([N, K] rows, so both operands are K-major for the
// MMA): an int8 weight as its q, exact in bf16 (one plane; the scale s
// becomes the epilogue's alpha, so W = s q is used as stored), a float32 or
// int4 weight as the three bf16 parts of its fp32 values (the int4 ones
// dequantised first, (float)q * scale bit for bit as the reference packs
// them). The products kept are a_i w_j with i + j <= 2: three MMAs per k-step
// for one weight plane (a0 q, a1 q, a2 q), six for three planes.
//
// Accuracy. The tensor cores align the products of a step to the largest and
// truncate what falls below, so a long run of accumulations into one TMEM
// accumulator loses more than fp32 rounding would. The accumulator is
// therefore drained into fp32 registers of the epilogue warps every 24 MMAs
// (128 of K with one plane, 64 with three) and restarted; the drains are
// summed with ordinary fp32 adds. Two accumulators alternate, so the MMAs of
// the next run overlap the drain of the last.
//
// Kernel. Persistent, one CTA per SM taking 128 x 256 output tiles in turn,
// 320 threads: warp 0 issues the
// TMA loads (cp.async.bulk.tensor, no multicast) of each 32-wide K block --
// the three A parts (128 x 32 each) and the weight planes (256 x 32 each),
// 64-byte swizzled -- into a ring of stages, completion on the stage's
// mbarrier; warp 1 allocates the 512 TMEM columns and one of its threads
// issues the tcgen05.mma (kind::f16, bf16 x bf16 -> fp32, M 128, N 256, K 16)
// of each stage, then tcgen05.commit frees the stage; warps 2..9 drain the
// accumulators (tcgen05.ld, one TMEM lane quadrant and 128 columns per warp)
// and run the epilogue from registers: alpha, bias, then store / Swish /
// scaled residual / the QKV head split with pos_bias_u/v / channel-first
// store with or without the GLU. A tile's epilogue math and stores run while
// the MMAs of the CTA's next tile fill the freed accumulators. Every wait is
// bounded by the global timer; a wait that runs out records an error and the
// CTA skips the rest of its work.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "pk_common.cuh"

namespace pk {
namespace tc {

constexpr int BM = 128, BK = 32;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 32 * (2 + EPI_WARPS);
constexpr int A_TILE = BM * BK * 2;   // one A part of a stage: 8 KB

// Tile width BN: 256 for large products, 64 when 256-wide tiles would leave
// most SMs idle (the decoder's products over a batch of a few hundred rows).
template <int NPB, int BN_>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int B_TILE = BN * BK * 2;      // one weight plane of a stage
  static constexpr int STAGE = 3 * A_TILE + NPB * B_TILE;
  static constexpr int STAGES = (220 * 1024) / STAGE < 6 ? (220 * 1024) / STAGE : 6;
  static constexpr int PRODUCTS = NPB == 1 ? 3 : 6;
  static constexpr int DRAIN_KB = NPB == 1 ? 4 : 2;   // K blocks per accumulator run (24 MMAs)
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
  static constexpr int TMEM_COLS = 2 * BN;            // two accumulators
  static constexpr int CW = BN / 2;                   // columns per epilogue warp
};

// Part pairs (A part, weight plane) with i + j <= 2, in issue order.
__device__ __forceinline__ void product_parts(int npb, int p, int &ia, int &ib) {
  if (npb == 1) {
    ia = p;
    ib = 0;
  } else {
    constexpr int PA[6] = {0, 0, 1, 0, 1, 2};
    constexpr int PB[6] = {0, 1, 0, 2, 1, 0};
    ia = PA[p];
    ib = PB[p];
  }
}

// ── PTX wrappers ──────────────────────────────────────────────────────────────

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            unsigned long long *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<unsigned long long>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 64-byte swizzle, rows of 64 bytes
// (32 bf16), 8-row groups 512 bytes apart (stride-dimension offset); the
// leading-dimension offset is unused for a swizzled K-major operand whose K
// extent fits one swizzle row. Bits 46-48 hold the fixed value 0b001.
__device__ __forceinline__ unsigned long long sdesc_k64(unsigned saddr) {
  unsigned long long d = 0;
  d |= (unsigned long long)((saddr & 0x3FFFFu) >> 4);
  d |= (unsigned long long)(16u >> 4) << 16;
  d |= (unsigned long long)(512u >> 4) << 32;
  d |= 1ull << 46;
  d |= 4ull << 61;   // 64-byte swizzle
  return d;
}

// Instruction descriptor, kind::f16: fp32 D, bf16 A and B, both K-major, M x N.
__host__ __device__ constexpr unsigned idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((unsigned)(N >> 3) << 17) | ((unsigned)(M >> 4) << 24);
}

__device__ __forceinline__ void umma(unsigned tmem_d, unsigned long long a, unsigned long long b,
                                     unsigned idesc, unsigned accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(unsigned long long *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes: v[j] = column col + j.
__device__ __forceinline__ void tmem_ld32(unsigned taddr, float (&v)[32]) {
  unsigned r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
}

// ── epilogue ────────────────────────────────────────────────────────────────

struct Epi {
  int mode;              // PK_TC_* (STORE, SWISH, RESID, QKV, CF, GLU, STORE_T, SWISH_SPLIT)
  float alpha;           // applied to the product first (an int8 weight's scale)
  float beta;            // STORE: C = alpha AW + beta C (the reference's pk_wmatmul)
  float rscale;          // RESID: X += rscale (alpha AW + bias)
  const float *bias;     // [N] or NULL, added after alpha
  float *C;              // output / residual stream, row pitch ldc floats
  long long ldc;
  // QKV: Q/K/V of frame r to [8, T, 128] per item; Qu = Q + u, Qv = Q + v
  const float *u, *v;
  float *Qu, *Qv, *Kh, *Vh;
  SeqDev seq;
  int channels;          // CF / GLU: output channels per frame (GLU: C, half of N)
  int vec;               // row-major output rows 16-byte aligned (ldc % 4 == 0)
  // Z products of the same shape in one launch (the per-head products): entry
  // z reads A rows from z * a_z and B rows from z * b_z, and writes from C + z * c_z
  int Z;
  long long a_z, b_z, c_z;
  __nv_bfloat16 *Cb;     // SWISH_SPLIT: the parts [M, 3N]
};

// Item of frame r: a division for a uniform batch, else a binary search of
// the batch's frame offsets (frame_off[i] <= r < frame_off[i + 1]).
__device__ __forceinline__ int item_of_row(const Epi &e, long long r) {
  if (e.seq.uniform_T) return (int)(r / e.seq.uniform_T);
  int lo = 0, hi = e.seq.n_items;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(e.seq.frame_off + mid) <= r) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Channel-first store of 32 channels c0 .. c0 + 31 of frame r: each item's
// output is [channels, T] (the pointwise convolutions' layout,
// csrc/tensor_ops.c:579-590), at element f0 * channels; the lanes of a warp
// hold consecutive frames, so each channel's 32 stores are contiguous.
__device__ __forceinline__ void store_cf32(const Epi &e, long long r, int c0, int channels, const float (&v)[32]) {
  const int item = item_of_row(e, r);
  const long long f0 = seq_frame_off(e.seq, item);
  const int T = seq_T(e.seq, item);
  float *o = e.C + f0 * channels + (long long)c0 * T + (r - f0);
#pragma unroll
  for (int j = 0; j < 32; j++) o[(long long)j * T] = v[j];
}

// The GLU of the first pointwise convolution (csrc/encoder.c:454-465) on 32
// channel pairs: a = the 32 "value" channels d0 .. d0 + 31, g = their gates
// d0 + C .. (the weight's rows are interleaved in groups of 32 at
// preparation, so both halves of a pair sit in one thread's columns);
// bias as pk_pointwise_conv1d adds it, then a * 1/(1 + exp(-g)) as the GLU
// kernels compute it (glu_gate).
__device__ __forceinline__ void epi_glu32(const Epi &e, long long r, int d0, int C, float (&a)[32],
                                          const float (&g)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j++) {
    const float va = e.bias ? a[j] + __ldg(e.bias + d0 + j) : a[j];
    const float vb = e.bias ? g[j] + __ldg(e.bias + C + d0 + j) : g[j];
    a[j] = glu_gate(va, vb);
  }
  store_cf32(e, r, d0, C, a);
}

// Finishes 32 columns n0 .. n0 + 31 of row r (all < N when the row exists).
__device__ __forceinline__ void epi_store32(const Epi &e, long long r, int n0, float (&v)[32]) {
  if (e.mode == PK_TC_CF) {
    if (e.bias) {
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] = v[j] + __ldg(e.bias + n0 + j);
    }
    store_cf32(e, r, n0, e.channels, v);
    return;
  }
  if (e.mode == PK_TC_QKV) {
    // n0 .. n0+31 lie in one head of one of Q, K, V (32 | 128)
    const int part = n0 >> 10, h = (n0 & 1023) >> 7, d0 = n0 & 127;
    const int item = item_of_row(e, r);
    const long long f0 = seq_frame_off(e.seq, item);
    const int T = seq_T(e.seq, item);
    const long long t = r - f0;
    const long long o = f0 * 1024 + ((long long)h * T + t) * 128 + d0;
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = v[j] + __ldg(e.bias + n0 + j);   // the fused [Bq | Bk | Bv]
    if (part == 0) {
      const float *u = e.u + h * 128 + d0, *w = e.v + h * 128 + d0;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        st4(e.Qu + o + j, make_float4(v[j] + __ldg(u + j), v[j + 1] + __ldg(u + j + 1),
                                      v[j + 2] + __ldg(u + j + 2), v[j + 3] + __ldg(u + j + 3)));
        st4(e.Qv + o + j, make_float4(v[j] + __ldg(w + j), v[j + 1] + __ldg(w + j + 1),
                                      v[j + 2] + __ldg(w + j + 2), v[j + 3] + __ldg(w + j + 3)));
      }
    } else {
      float *dst = part == 1 ? e.Kh : e.Vh;
#pragma unroll
      for (int j = 0; j < 32; j += 4) st4(dst + o + j, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
    }
    return;
  }
  if (e.mode == PK_TC_SWISH_SPLIT) {
    // Swish, then the three bf16 parts of each value as the activation split
    // makes them (x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1)):
    // 64-byte runs into the [h0 | h1 | h2] row of the next product's operand
    const long long N = e.channels;
    __nv_bfloat16 *o = e.Cb + r * 3 * N + n0;
#pragma unroll
    for (int j0 = 0; j0 < 32; j0 += 8) {
      __align__(16) __nv_bfloat16 p[3][8];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        float2 h = make_float2(v[j0 + j], v[j0 + j + 1]);
        if (e.bias) {
          h.x = h.x + __ldg(e.bias + n0 + j0 + j);
          h.y = h.y + __ldg(e.bias + n0 + j0 + j + 1);
        }
        h = swish_poly2(h);
        const float hv[2] = {h.x, h.y};
#pragma unroll
        for (int u = 0; u < 2; u++) {
          p[0][j + u] = __float2bfloat16_rn(hv[u]);
          const float r1 = hv[u] - __bfloat162float(p[0][j + u]);
          p[1][j + u] = __float2bfloat16_rn(r1);
          p[2][j + u] = __float2bfloat16_rn(r1 - __bfloat162float(p[1][j + u]));
        }
      }
#pragma unroll
      for (int k = 0; k < 3; k++)
        *reinterpret_cast<uint4 *>(o + k * N + j0) = *reinterpret_cast<const uint4 *>(p[k]);
    }
    return;
  }
  float *c = e.C + r * e.ldc + n0;
  if (e.bias) {
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = v[j] + __ldg(e.bias + n0 + j);
  }
  if (e.mode == PK_TC_SWISH) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const float2 s = swish_poly2(make_float2(v[j], v[j + 1]));
      v[j] = s.x;
      v[j + 1] = s.y;
    }
  } else if (e.mode == PK_TC_RESID) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 x = ld4(c + j);
      // x + s * out as one fused multiply-add (the reference's macaron residual
      // body is fma(out, 0.5, x); s = 1 gives x + out exactly)
      v[j] = fmaf(v[j], e.rscale, x.x);
      v[j + 1] = fmaf(v[j + 1], e.rscale, x.y);
      v[j + 2] = fmaf(v[j + 2], e.rscale, x.z);
      v[j + 3] = fmaf(v[j + 3], e.rscale, x.w);
    }
  } else if (e.beta != 0.0f) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 x = ld4(c + j);
      v[j] = fmaf(e.beta, x.x, v[j]);
      v[j + 1] = fmaf(e.beta, x.y, v[j + 1]);
      v[j + 2] = fmaf(e.beta, x.z, v[j + 2]);
      v[j + 3] = fmaf(e.beta, x.w, v[j + 3]);
    }
  }
#pragma unroll
  for (int j = 0; j < 32; j += 4) st4(c + j, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
}

// STORE_T: C[n, m] = alpha (A W)[m, n] -- the product written transposed, so
// the lanes of a warp (consecutive m) store consecutive addresses.
__device__ __forceinline__ void epi_store_t(float *cz, long long ldc, long long r, int n, int ncols,
                                            const float (&v)[32]) {
  float *o = cz + (long long)n * ldc + r;
#pragma unroll
  for (int j = 0; j < 32; j++)
    if (j < ncols) o[(long long)j * ldc] = v[j];
}

// Row-major STORE / SWISH / RESID of the columns n .. n + ncols - 1 (ncols <=
// 32) one at a time: a ragged last column group (N not a multiple of 32) or
// rows that are not 16-byte aligned (ldc not a multiple of 4).
__device__ __forceinline__ void epi_store_tail(const Epi &e, long long r, int n, int ncols, const float (&v)[32]) {
  float *c = e.C + r * e.ldc + n;
#pragma unroll
  for (int j = 0; j < 32; j++) {
    if (j < ncols) {
      float o = e.bias ? v[j] + __ldg(e.bias + n + j) : v[j];
      if (e.mode == PK_TC_SWISH) o = swish_poly(o);
      else if (e.mode == PK_TC_RESID) o = fmaf(o, e.rscale, c[j]);
      else if (e.beta != 0.0f) o = fmaf(e.beta, c[j], o);
      c[j] = o;
    }
  }
}

template <int NPB, int BN_>
__global__ void __launch_bounds__(THREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               int M, int N, int K, Epi epi) {
  using C = Cfg<NPB, BN_>;
  constexpr int BN = C::BN, B_TILE = C::B_TILE, TMEM_COLS = C::TMEM_COLS, CW = C::CW;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned long long *full = reinterpret_cast<unsigned long long *>(smem + C::STAGES * C::STAGE);
  unsigned long long *empty = full + C::STAGES;
  unsigned long long *acc_full = empty + C::STAGES;    // [2]
  unsigned long long *acc_empty = acc_full + 2;        // [2]
  unsigned long long *done = acc_empty + 2;            // the MMA thread's last commit
  unsigned *tmem_slot = reinterpret_cast<unsigned *>(done + 1);
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = K / BK;
  const int n_runs = (nkb + C::DRAIN_KB - 1) / C::DRAIN_KB;
  // persistent: this CTA takes tiles blockIdx.x, + gridDim.x, ...; n-blocks
  // vary fastest, so the CTAs of a wave share the rows of A they read
  const int tiles_n = (N + BN - 1) / BN;
  const int per_z = tiles_n * ((M + BM - 1) / BM);
  const int n_tiles = per_z * epi.Z;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; s++) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, EPI_WARPS);
    }
    mbar_init(done, 1);
    mbar_init_fence();
    s_abort = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = *tmem_slot;

  if (warp == 0) {
    // ── producer: TMA loads of each K block into the stage ring ──
    if (lane == 0) {
      int it = 0;   // K blocks issued by this CTA, over all its tiles
      bool stop = false;
      for (int tile = blockIdx.x; tile < n_tiles && !stop; tile += gridDim.x) {
        const int z = tile / per_z, t = tile - z * per_z;
        const int m0 = (t / tiles_n) * BM, n0 = (t % tiles_n) * BN;
        const int ya = (int)(z * epi.a_z) + m0, yb = (int)(z * epi.b_z) + n0;
        for (int kb = 0; kb < nkb; kb++) {
          const int s = it % C::STAGES;
          if (it >= C::STAGES && !mbar_wait(empty + s, ((it / C::STAGES) - 1) & 1)) {
            atomicAdd(&g_wait_timeouts, 1u);
            s_abort = 1;
          }
          if (*(volatile int *)&s_abort) {
            stop = true;
            break;
          }
          unsigned char *st = smem + s * C::STAGE;
          mbar_arrive_tx(full + s, C::STAGE);
          for (int p = 0; p < 3; p++) tma_load_2d(st + p * A_TILE, &map_a, p * K + kb * BK, ya, full + s);
          for (int p = 0; p < NPB; p++)
            tma_load_2d(st + 3 * A_TILE + p * B_TILE, &map_b, p * K + kb * BK, yb, full + s);
          it++;
        }
      }
      if (*(volatile int *)&s_abort) {
        // a wait ran out somewhere: let this CTA's copies still in flight land
        // (bounded) before its shared memory is released
        for (int j = it > C::STAGES ? it - C::STAGES : 0; j < it; j++)
          mbar_wait(full + j % C::STAGES, (j / C::STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ── MMA issue: one thread ──
    if (lane == 0) {
      constexpr unsigned IDESC = idesc_bf16(BM, BN);
      int it = 0, gr = 0;   // K blocks consumed and accumulator runs, over all tiles
      for (int tile = blockIdx.x; tile < n_tiles && !*(volatile int *)&s_abort; tile += gridDim.x) {
        int kb = 0;
        for (int run = 0; run < n_runs && !*(volatile int *)&s_abort; run++, gr++) {
          const int buf = gr & 1;
          if (gr >= 2 && !mbar_wait(acc_empty + buf, ((gr >> 1) - 1) & 1)) {
            atomicAdd(&g_wait_timeouts, 1u);
            s_abort = 1;
            break;
          }
          tc_fence_after();
          const unsigned d = tmem + buf * BN;
          const int kb_end = kb + C::DRAIN_KB < nkb ? kb + C::DRAIN_KB : nkb;
          bool first = true;
          for (; kb < kb_end; kb++, it++) {
            const int s = it % C::STAGES;
            if (!mbar_wait(full + s, (it / C::STAGES) & 1)) {
              atomicAdd(&g_wait_timeouts, 1u);
              s_abort = 1;
              break;
            }
            tc_fence_after();
            const unsigned st = smem_u32(smem + s * C::STAGE);
#pragma unroll
            for (int k = 0; k < BK / 16; k++) {
#pragma unroll
              for (int p = 0; p < C::PRODUCTS; p++) {
                int ia, ib;
                product_parts(NPB, p, ia, ib);
                const unsigned long long da = sdesc_k64(st + ia * A_TILE + k * 32);
                const unsigned long long db = sdesc_k64(st + 3 * A_TILE + ib * B_TILE + k * 32);
                umma(d, da, db, IDESC, first ? 0u : 1u);
                first = false;
              }
            }
            umma_commit(empty + s);   // the stage is free once these MMAs are done
          }
          if (*(volatile int *)&s_abort) break;
          umma_commit(acc_full + buf);   // this run's sum is ready to drain
        }
      }
      // every MMA issued here has finished before the TMEM is released
      umma_commit(done);
      mbar_wait(done, 0);
    }
  } else {
    // ── drain and epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31; the
    // MMAs of the next tile run into the free accumulators meanwhile ──
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const unsigned lane_addr = ((unsigned)(q * 32) << 16) + half * CW;
    int gr = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
      const int z = tile / per_z, t = tile - z * per_z;
      const int m0 = (t / tiles_n) * BM, n0 = (t % tiles_n) * BN;
      float sum[CW];
#pragma unroll
      for (int j = 0; j < CW; j++) sum[j] = 0.0f;
      for (int run = 0; run < n_runs; run++, gr++) {
        const int buf = gr & 1;
        // the outcome is made warp-uniform: tcgen05.ld needs every lane
        if (!__all_sync(PK_FULL_MASK, mbar_wait(acc_full + buf, (gr >> 1) & 1))) {
          if (lane == 0) atomicAdd(&g_wait_timeouts, 1u);
          s_abort = 1;
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < CW / 32; c++) {
          float v[32];
          tmem_ld32(tmem + lane_addr + buf * BN + c * 32, v);
#pragma unroll
          for (int j = 0; j < 32; j++) sum[c * 32 + j] += v[j];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + buf);
      }
      const long long r = (long long)m0 + row;
      if (CW >= 64 && ok && r < M && epi.mode == PK_TC_GLU) {
        // columns 64k .. 64k + 31 hold value channels 32k .., the next 32 their gates
#pragma unroll
        for (int c = 0; c + 1 < CW / 32; c += 2) {
          const int n = n0 + half * CW + c * 32;
          if (n < N) {
            float a[32], g[32];
#pragma unroll
            for (int j = 0; j < 32; j++) {
              a[j] = sum[c * 32 + j] * epi.alpha;
              g[j] = sum[(c + 1) * 32 + j] * epi.alpha;
            }
            epi_glu32(epi, r, n / 2, epi.channels, a, g);
          }
        }
      } else if (ok && r < M && epi.mode == PK_TC_STORE_T) {
#pragma unroll
        for (int c = 0; c < CW / 32; c++) {
          const int n = n0 + half * CW + c * 32;
          if (n < N) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = sum[c * 32 + j] * epi.alpha;
            epi_store_t(epi.C + z * epi.c_z, epi.ldc, r, n, N - n < 32 ? N - n : 32, v);
          }
        }
      } else if (ok && r < M) {
        Epi ez = epi;
        ez.C = epi.C + z * epi.c_z;
#pragma unroll
        for (int c = 0; c < CW / 32; c++) {
          const int n = n0 + half * CW + c * 32;
          if (n < N) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] = sum[c * 32 + j] * epi.alpha;
            if (n + 32 <= N && ez.vec) epi_store32(ez, r, n, v);
            else epi_store_tail(ez, r, n, N - n < 32 ? N - n : 32, v);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ── weight preparation (once per weight) ─────────────────────────────────────

// W [K, N] fp32 -> out [N, 3K] bf16, row n = [w0 | w1 | w2] of column n.
// 32 x 32 tiles through shared memory: coalesced reads along N, writes along K.
__global__ void prep_split_t_kernel(const float *__restrict__ W, __nv_bfloat16 *__restrict__ out, int K,
                                    int N) {
  __shared__ float tile[32][33];
  const int k0 = blockIdx.y * 32, nb = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8 threads
  for (int i = ty; i < 32; i += 8) {
    const int k = k0 + i, n = nb + tx;
    tile[i][tx] = (k < K && n < N) ? __ldg(W + (long long)k * N + n) : 0.0f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int n = nb + i, k = k0 + tx;
    if (n < N && k < K) {
      const float x = tile[tx][i];
      const __nv_bfloat16 p0 = __float2bfloat16_rn(x);
      const float r1 = x - __bfloat162float(p0);
      const __nv_bfloat16 p1 = __float2bfloat16_rn(r1);
      const __nv_bfloat16 p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
      __nv_bfloat16 *o = out + (long long)n * 3 * K + k;
      o[0] = p0;
      o[K] = p1;
      o[2 * K] = p2;
    }
  }
}

// q [K, N] int8 -> out [N, K] bf16 (exact: |q| <= 127).
__global__ void prep_q8_t_kernel(const int8_t *__restrict__ q, __nv_bfloat16 *__restrict__ out, int K, int N) {
  __shared__ float tile[32][33];
  const int k0 = blockIdx.y * 32, nb = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int i = ty; i < 32; i += 8) {
    const int k = k0 + i, n = nb + tx;
    tile[i][tx] = (k < K && n < N) ? (float)q[(long long)k * N + n] : 0.0f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int n = nb + i, k = k0 + tx;
    if (n < N && k < K) out[(long long)n * K + k] = __float2bfloat16_rn(tile[tx][i]);
  }
}

// A pointwise-convolution weight W [N, K] (out channels x in channels, already
// K-major) -> planes [N, 3K], row n' = [w0 | w1 | w2] of source row src(n').
// With glu (N = 2C) the rows are interleaved in groups of 32: rows 64k .. 64k+31
// are value channels 32k .., rows 64k+32 .. 64k+63 their gates C + 32k ..
__global__ void prep_split_rows_kernel(const float *__restrict__ W, __nv_bfloat16 *__restrict__ out, int N, int K,
                                       int glu) {
  const long long total = (long long)N * K;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(e / K), k = (int)(e - (long long)n * K);
    int src = n;
    if (glu) {
      const int blk = n >> 6, w = n & 63;
      src = w < 32 ? blk * 32 + w : (N >> 1) + blk * 32 + (w - 32);
    }
    const float x = __ldg(W + (long long)src * K + k);
    const __nv_bfloat16 p0 = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(p0);
    const __nv_bfloat16 p1 = __float2bfloat16_rn(r1);
    const __nv_bfloat16 p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
    __nv_bfloat16 *o = out + (long long)n * 3 * K + k;
    o[0] = p0;
    o[K] = p1;
    o[2 * K] = p2;
  }
}

// Two row sets side by side as one K-major operand: row m of the output is the
// parts of [X1[m] (K1) | X2[m] (K2)], each part K1 + K2 wide (the decoder's
// [x | h] against [W_i | W_r]: one product per LSTM layer instead of two).
__global__ void split_rows_cat_kernel(const float *__restrict__ X1, const float *__restrict__ X2,
                                      __nv_bfloat16 *__restrict__ out, long long M, int K1, int K2) {
  const int K = K1 + K2;
  const long long total = M * K;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long m = e / K;
    const int k = (int)(e - m * K);
    const float x = k < K1 ? __ldg(X1 + m * K1 + k) : __ldg(X2 + m * K2 + (k - K1));
    const __nv_bfloat16 p0 = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(p0);
    const __nv_bfloat16 p1 = __float2bfloat16_rn(r1);
    const __nv_bfloat16 p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
    __nv_bfloat16 *o = out + m * 3 * K + k;
    o[0] = p0;
    o[K] = p1;
    o[2 * K] = p2;
  }
}

// Channel-first items X [C, T_b] (item after item) -> time-first parts
// [frames, 3C], row f0_b + t = [x0 | x1 | x2] of column t: the operand of a
// pointwise convolution as a K-major matrix. 32 x 32 tiles through shared
// memory; blockIdx.z = item.
__global__ void split_cf_t_kernel(const float *__restrict__ X, __nv_bfloat16 *__restrict__ out, int C,
                                  SeqDev seq) {
  __shared__ float tile[32][33];
  const int item = blockIdx.z;
  const int T = seq_T(seq, item);
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  if (t0 >= T) return;
  const long long f0 = seq_frame_off(seq, item);
  const float *x = X + f0 * C;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8 threads
  for (int i = ty; i < 32; i += 8) {
    const int c = c0 + i, t = t0 + tx;
    tile[i][tx] = (c < C && t < T) ? __ldg(x + (long long)c * T + t) : 0.0f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int t = t0 + i, c = c0 + tx;
    if (t < T && c < C) {
      const float v = tile[tx][i];
      const __nv_bfloat16 p0 = __float2bfloat16_rn(v);
      const float r1 = v - __bfloat162float(p0);
      const __nv_bfloat16 p1 = __float2bfloat16_rn(r1);
      const __nv_bfloat16 p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
      __nv_bfloat16 *o = out + (f0 + t) * 3 * C + c;
      o[0] = p0;
      o[C] = p1;
      o[2 * C] = p2;
    }
  }
}

// Rows A [M, K] (any K) -> parts [M, 3 Kp], row m = [a0 | a1 | a2] each Kp wide
// with zeros from column K on: a K-major operand whose K is padded to the
// GEMM's 32-wide K blocks (the score rows S of the context product, K = T).
__global__ void split_rows_pad_kernel(const float *__restrict__ A, __nv_bfloat16 *__restrict__ out, long long M,
                                      int K, int Kp) {
  // a thread takes 8 consecutive columns of a row (Kp % 8 == 0): 8 coalesced
  // scalar loads (rows of odd K are not 16-byte aligned) and one 16-byte
  // store per part
  const int K8 = Kp / 8;
  const long long total = M * K8;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long m = e / K8;
    const int k0 = (int)(e - m * K8) * 8;
    const float *a = A + m * K;
    __align__(16) __nv_bfloat16 p[3][8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float x = k0 + j < K ? __ldg(a + k0 + j) : 0.0f;
      p[0][j] = __float2bfloat16_rn(x);
      const float r1 = x - __bfloat162float(p[0][j]);
      p[1][j] = __float2bfloat16_rn(r1);
      p[2][j] = __float2bfloat16_rn(r1 - __bfloat162float(p[1][j]));
    }
    __nv_bfloat16 *o = out + m * 3 * Kp + k0;
#pragma unroll
    for (int q = 0; q < 3; q++) *reinterpret_cast<uint4 *>(o + (long long)q * Kp) = *reinterpret_cast<const uint4 *>(p[q]);
  }
}

// Z matrices X [R, Cc] (one after another) -> their transposes as parts: out
// rows z Cc + c = [x0 | x1 | x2] of column c, each Kp wide, zeros from R on
// (the value heads V [T, 128] as the context product's K-major operand).
__global__ void split_t_pad_kernel(const float *__restrict__ X, __nv_bfloat16 *__restrict__ out, int R, int Cc,
                                   int Kp) {
  __shared__ float tile[32][33];
  const int z = blockIdx.z;
  const int r0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const float *x = X + (long long)z * R * Cc;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8 threads
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + tx;
    tile[i][tx] = (r < R && c < Cc) ? __ldg(x + (long long)r * Cc + c) : 0.0f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + tx;
    if (c < Cc && r < Kp) {
      const float v = tile[tx][i];   // 0 past R
      const __nv_bfloat16 p0 = __float2bfloat16_rn(v);
      const float r1 = v - __bfloat162float(p0);
      const __nv_bfloat16 p1 = __float2bfloat16_rn(r1);
      const __nv_bfloat16 p2 = __float2bfloat16_rn(r1 - __bfloat162float(p1));
      __nv_bfloat16 *o = out + ((long long)z * Cc + c) * 3 * Kp + r;
      o[0] = p0;
      o[Kp] = p1;
      o[2 * Kp] = p2;
    }
  }
}

PK_WAIT_TIMEOUTS_ACCESSOR(pk_tc_wait_timeouts_acc)

}  // namespace tc
}  // namespace pk

using namespace pk;

// ── host side ─────────────────────────────────────────────────────────────────

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_encode_lock;

int encoder_fn(PFN_cuTensorMapEncodeTiled_v12000 *fn) {
  std::lock_guard<std::mutex> lock(g_encode_lock);
  if (!g_encode) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p) {
      cudaGetLastError();
      return pkcu_fail(PKCU_ERR_CUDA, "tcgen05 GEMM: cuTensorMapEncodeTiled is not available");
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  *fn = g_encode;
  return PKCU_OK;
}

// 2-D bf16 tensor map over rows x cols (row pitch `pitch` elements), boxes of
// box_rows x 32 columns, 64-byte swizzle, zero fill out of bounds.
int tmap_bf16(CUtensorMap *map, const void *base, long long rows, long long cols, long long pitch,
              int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  int st = encoder_fn(&fn);
  if (st) return st;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)pitch * 2};
  const cuuint32_t box[2] = {(cuuint32_t)tc::BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return pkcu_fail(PKCU_ERR_ARG, "tcgen05 GEMM: tensor map rejected (%d) for %lld x %lld", (int)r, rows,
                     cols);
  return PKCU_OK;
}

template <int NPB, int BN>
int *optin_flags() {
  static int flags[64];
  return flags;
}

template <int NPB, int BN>
int launch(const CUtensorMap &ma, const CUtensorMap &mb, int M, int N, int K, const tc::Epi &e,
           cudaStream_t s) {
  using C = tc::Cfg<NPB, BN>;
  smem_optin(tc::tc_gemm_kernel<NPB, BN>, C::SMEM, optin_flags<NPB, BN>());
  // persistent: one CTA per SM (the stage ring fills most of its shared memory)
  const long long tiles = (long long)((N + BN - 1) / BN) * ((M + tc::BM - 1) / tc::BM) * e.Z;
  const unsigned grid = (unsigned)(tiles < pkcu_sm_count() ? tiles : pkcu_sm_count());
  tc::tc_gemm_kernel<NPB, BN><<<grid, tc::THREADS, C::SMEM, s>>>(ma, mb, M, N, K, e);
  return pkcu_launch_status("tcgen05 GEMM");
}
}  // namespace

extern "C" void pk_tc_warm(void) {
  smem_optin(tc::tc_gemm_kernel<1, 256>, tc::Cfg<1, 256>::SMEM, optin_flags<1, 256>());
  smem_optin(tc::tc_gemm_kernel<3, 256>, tc::Cfg<3, 256>::SMEM, optin_flags<3, 256>());
  smem_optin(tc::tc_gemm_kernel<1, 64>, tc::Cfg<1, 64>::SMEM, optin_flags<1, 64>());
  smem_optin(tc::tc_gemm_kernel<3, 64>, tc::Cfg<3, 64>::SMEM, optin_flags<3, 64>());
  smem_optin(tc::tc_gemm_kernel<1, 128>, tc::Cfg<1, 128>::SMEM, optin_flags<1, 128>());
  smem_optin(tc::tc_gemm_kernel<3, 128>, tc::Cfg<3, 128>::SMEM, optin_flags<3, 128>());
}

extern "C" int pk_tc_wait_timeouts(unsigned *count, int reset) {
  return tc::pk_tc_wait_timeouts_acc(count, reset);
}

extern "C" int pk_tc_prepare(const void *data, int bits, float scale, int K, int N, void *planes,
                             float *alpha, pkcu_stream_t stream) {
  const dim3 grid((unsigned)((N + 31) / 32), (unsigned)((K + 31) / 32));
  cudaStream_t s = (cudaStream_t)stream;
  if (bits == 8) {
    tc::prep_q8_t_kernel<<<grid, 256, 0, s>>>(static_cast<const int8_t *>(data),
                                             static_cast<__nv_bfloat16 *>(planes), K, N);
    *alpha = scale;
  } else {
    tc::prep_split_t_kernel<<<grid, 256, 0, s>>>(static_cast<const float *>(data),
                                                static_cast<__nv_bfloat16 *>(planes), K, N);
    *alpha = 1.0f;
  }
  return pkcu_launch_status("tcgen05 GEMM weight preparation");
}

extern "C" int pk_tc_prepare_rows(const float *W, int N, int K, int glu, void *planes, pkcu_stream_t stream) {
  const long long total = (long long)N * K;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  tc::prep_split_rows_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(W, static_cast<__nv_bfloat16 *>(planes), N,
                                                                       K, glu);
  return pkcu_launch_status("tcgen05 GEMM pointwise weight preparation");
}

extern "C" int pk_split_rows_pad(const float *A, void *parts, long long M, int K, int Kp, pkcu_stream_t stream) {
  if (!A || !parts || M <= 0 || K <= 0 || Kp < K || Kp % 8 || !PK_ALIGNED16(parts))
    return pkcu_fail(PKCU_ERR_ARG, "pk_split_rows_pad: bad argument (Kp %% 8 == 0, parts 16-byte aligned)");
  long long blocks = (M * (Kp / 8) + 255) / 256;
  if (blocks > 16LL * pkcu_sm_count()) blocks = 16LL * pkcu_sm_count();
  tc::split_rows_pad_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      A, static_cast<__nv_bfloat16 *>(parts), M, K, Kp);
  return pkcu_launch_status("pk_split_rows_pad");
}

extern "C" int pk_split_t_pad(const float *X, void *parts, int Z, int R, int Cc, int Kp, pkcu_stream_t stream) {
  if (!X || !parts || Z <= 0 || Z > 65535 || R <= 0 || Cc <= 0 || Kp < R)
    return pkcu_fail(PKCU_ERR_ARG, "pk_split_t_pad: bad argument");
  const dim3 grid((unsigned)((Kp + 31) / 32), (unsigned)((Cc + 31) / 32), (unsigned)Z);
  tc::split_t_pad_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(X, static_cast<__nv_bfloat16 *>(parts), R, Cc,
                                                                  Kp);
  return pkcu_launch_status("pk_split_t_pad");
}

extern "C" int pk_split_rows_cat(const float *X1, const float *X2, void *parts, long long M, int K1, int K2,
                                 pkcu_stream_t stream) {
  if (!X1 || !X2 || !parts || M <= 0 || K1 <= 0 || K2 <= 0)
    return pkcu_fail(PKCU_ERR_ARG, "pk_split_rows_cat: bad argument");
  long long blocks = (M * (K1 + K2) + 255) / 256;
  if (blocks > 16LL * pkcu_sm_count()) blocks = 16LL * pkcu_sm_count();
  tc::split_rows_cat_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      X1, X2, static_cast<__nv_bfloat16 *>(parts), M, K1, K2);
  return pkcu_launch_status("pk_split_rows_cat");
}

extern "C" int pk_split_cf_t(const float *X, void *parts, int C, const pkcu_seq *seq, pkcu_stream_t stream) {
  if (!X || !parts || !seq || C <= 0) return pkcu_fail(PKCU_ERR_ARG, "pk_split_cf_t: bad argument");
  const dim3 grid((unsigned)((seq->dev.max_T + 31) / 32), (unsigned)((C + 31) / 32), (unsigned)seq->dev.n_items);
  tc::split_cf_t_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(X, static_cast<__nv_bfloat16 *>(parts), C,
                                                                seq->dev);
  return pkcu_launch_status("pk_split_cf_t");
}

namespace {
int tc_gemm_run(const void *a_parts, long long a_rows, const void *planes, long long b_rows, int npb, int M,
                int N, int K, const pk_tc_epi *ep, int Z, long long a_z, long long b_z, long long c_z,
                pkcu_stream_t stream);
}

extern "C" int pk_tc_gemm(const void *a_parts, const void *planes, int npb, int M, int N, int K,
                          const pk_tc_epi *ep, pkcu_stream_t stream) {
  return tc_gemm_run(a_parts, M, planes, N, npb, M, N, K, ep, 1, 0, 0, 0, stream);
}

extern "C" int pk_tc_gemm_batched(const void *a_parts, long long a_rows, const void *b_parts, long long b_rows,
                                  int M, int N, int K, const pk_tc_epi *ep, int Z, long long a_z,
                                  long long b_z, long long c_z, pkcu_stream_t stream) {
  // TMA row coordinates are 32-bit; rows past a_rows / b_rows read as zeros
  if (Z <= 0 || a_z < 0 || b_z < 0 || (long long)(Z - 1) * a_z + M > 0x7fffff00LL ||
      (long long)(Z - 1) * b_z + N > 0x7fffff00LL)
    return pkcu_fail(PKCU_ERR_ARG, "tcgen05 GEMM: bad batch (%d entries)", Z);
  return tc_gemm_run(a_parts, a_rows, b_parts, b_rows, 3, M, N, K, ep, Z, a_z, b_z, c_z, stream);
}

namespace {
int tc_gemm_run(const void *a_parts, long long a_rows, const void *planes, long long b_rows, int npb, int M,
                int N, int K, const pk_tc_epi *ep, int Z, long long a_z, long long b_z, long long c_z,
                pkcu_stream_t stream) {
  if (!a_parts || !planes || !ep || (npb != 1 && npb != 3) || M <= 0 || N <= 0 || K <= 0 ||
      K % tc::BK || (N % 32 && ep->mode != PK_TC_STORE && ep->mode != PK_TC_SWISH &&
                     ep->mode != PK_TC_RESID && ep->mode != PK_TC_STORE_T) ||
      !PK_ALIGNED16(a_parts) || !PK_ALIGNED16(planes))
    return pkcu_fail(PKCU_ERR_ARG, "tcgen05 GEMM: bad arguments (M %d, N %d, K %d)", M, N, K);
  // 256-wide tiles unless N <= 128 (half padding) or they would occupy fewer
  // than half the SMs; the GLU epilogue always takes them (a value group and
  // its gates in one warp's columns)
  const int narrow = ep->mode != PK_TC_GLU &&
                     (N <= 128 || Z * (long long)((N + 255) / 256) * ((M + tc::BM - 1) / tc::BM) * 2 <
                                      pkcu_sm_count());
  // otherwise 128-wide tiles where they pad N less than 256-wide ones (the
  // per-head products, N = T = 375: 384 against 512 columns of MMA work)
  const int bn = narrow ? 64
                        : (ep->mode != PK_TC_GLU && (N + 127) / 128 * 128 < (N + 255) / 256 * 256 ? 128 : 256);
  CUtensorMap ma, mb;
  int st = tmap_bf16(&ma, a_parts, a_rows, 3LL * K, 3LL * K, tc::BM);
  if (!st) st = tmap_bf16(&mb, planes, b_rows, (long long)npb * K, (long long)npb * K, bn);
  if (st) return st;
  tc::Epi e;
  e.mode = ep->mode;
  e.alpha = ep->alpha;
  e.beta = ep->beta;
  e.rscale = ep->rscale;
  e.bias = ep->bias;
  e.C = ep->C;
  e.ldc = ep->ldc ? ep->ldc : N;
  e.u = ep->u;
  e.v = ep->v;
  e.Qu = ep->Qu;
  e.Qv = ep->Qv;
  e.Kh = ep->K;
  e.Vh = ep->V;
  if (ep->seq) e.seq = ep->seq->dev;
  else memset(&e.seq, 0, sizeof(e.seq));
  e.channels = e.mode == PK_TC_GLU ? N / 2 : N;
  e.Cb = static_cast<__nv_bfloat16 *>(ep->Cb);
  if (e.mode == PK_TC_SWISH_SPLIT && (!e.Cb || !PK_ALIGNED16(e.Cb) || N % 32 || Z != 1))
    return pkcu_fail(PKCU_ERR_ARG, "tcgen05 GEMM: the split Swish epilogue needs aligned parts and N %% 32 == 0");
  if ((e.mode == PK_TC_CF || e.mode == PK_TC_GLU) &&
      (!ep->seq || !e.C || M != ep->seq->frames || (e.mode == PK_TC_GLU && N % 64)))
    return pkcu_fail(PKCU_ERR_ARG, "tcgen05 GEMM: a channel-first epilogue needs the batch and its output");
  if (e.mode == PK_TC_QKV &&
      (!ep->seq || !e.bias || !e.u || !e.v || !e.Qu || !e.Qv || !e.Kh || !e.Vh || N != 3 * PK_D ||
       M != ep->seq->frames))
    return pkcu_fail(PKCU_ERR_ARG, "tcgen05 GEMM: the QKV epilogue needs the batch and its outputs");
  if ((e.mode == PK_TC_STORE || e.mode == PK_TC_SWISH || e.mode == PK_TC_RESID) && (!e.C || e.ldc < N))
    return pkcu_fail(PKCU_ERR_ARG, "tcgen05 GEMM: no output, or rows shorter than N");
  e.vec = (PK_ALIGNED16(e.C) && e.ldc % 4 == 0 && (c_z % 4) == 0) || e.mode == PK_TC_SWISH_SPLIT;
  e.Z = Z;
  e.a_z = a_z;
  e.b_z = b_z;
  e.c_z = c_z;
  if (e.mode == PK_TC_STORE_T && (!e.C || !ep->ldc || ep->ldc < M))
    return pkcu_fail(PKCU_ERR_ARG, "tcgen05 GEMM: the transposed store needs rows of at least M");
  cudaStream_t s = (cudaStream_t)stream;
  if (bn == 64)
    return npb == 1 ? launch<1, 64>(ma, mb, M, N, K, e, s) : launch<3, 64>(ma, mb, M, N, K, e, s);
  if (bn == 128)
    return npb == 1 ? launch<1, 128>(ma, mb, M, N, K, e, s) : launch<3, 128>(ma, mb, M, N, K, e, s);
  return npb == 1 ? launch<1, 256>(ma, mb, M, N, K, e, s) : launch<3, 256>(ma, mb, M, N, K, e, s);
}
}  // namespace

// ── public entry points: weight products (csrc/tensor_ops.c:50-61) ──────────

struct pkcu_weight {
  int K, N, bits, npb;
  float alpha;      // the int8 scale (1 for the three-part planes)
  void *planes;     // [N, npb K] bf16
  int conv;         // a pointwise-convolution weight (N = out channels, K = in channels)
  int glu;          // its rows interleaved value / gate for the GLU epilogue
};

extern "C" void pkcu_weight_destroy(pkcu_weight *w) {
  if (!w) return;
  if (w->planes) cudaFree(w->planes);
  free(w);
}

extern "C" int pkcu_weight_create(const void *data, int bits, float scale, const float *scales, int group,
                                  int axis, int K, int N, pkcu_stream_t stream, pkcu_weight **out) {
  if (!out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weight_create: NULL out");
  *out = nullptr;
  if (!data || K <= 0 || N <= 0 || K % tc::BK || N % 32)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_weight_create: K %d must be a multiple of 32 and N %d of 32", K, N);
  if (bits != 32 && bits != 8 && bits != 4)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_weight_create: bits %d (32, 8 or 4)", bits);
  if (bits == 8 && !(scale > 0.0f)) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weight_create: int8 scale %g", scale);
  if (bits == 4 && !scales) return pkcu_fail(PKCU_ERR_ARG, "pkcu_weight_create: int4 without scales");
  pkcu_weight *w = (pkcu_weight *)calloc(1, sizeof(*w));
  if (!w) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_weight_create: host allocation");
  w->K = K;
  w->N = N;
  w->bits = bits;
  w->npb = bits == 8 ? 1 : 3;
  const size_t bytes = (size_t)w->npb * K * N * 2;
  if (cudaMalloc(&w->planes, bytes) != cudaSuccess) {
    cudaGetLastError();
    w->planes = nullptr;
    pkcu_weight_destroy(w);
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_weight_create: %zu bytes", bytes);
  }
  cudaStream_t s = (cudaStream_t)stream;
  int st = PKCU_OK;
  float *tmp = nullptr;
  const void *src = data;
  if (bits == 4) {   // (float)q * group scale, bit for bit as the reference packs it, then split
    if (cudaMalloc((void **)&tmp, sizeof(float) * (size_t)K * N) != cudaSuccess) {
      cudaGetLastError();
      tmp = nullptr;
      st = pkcu_fail(PKCU_ERR_NOMEM, "pkcu_weight_create: int4 staging");
    }
    if (!st) st = pkcu_dequant_i4(static_cast<const uint8_t *>(data), scales, tmp, K, N, group, axis, stream);
    src = tmp;
  }
  if (!st) st = pk_tc_prepare(src, bits == 8 ? 8 : 32, scale, K, N, w->planes, &w->alpha, stream);
  if (cudaStreamSynchronize(s) != cudaSuccess && !st)
    st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_weight_create: %s", cudaGetErrorString(cudaGetLastError()));
  if (tmp) cudaFree(tmp);
  if (st) {
    pkcu_weight_destroy(w);
    return st;
  }
  *out = w;
  return PKCU_OK;
}

extern "C" long long pkcu_wmatmul_work_bytes(int M, int K) {
  if (M <= 0 || K <= 0) return 0;
  return ((long long)M * K * 6 + 255) & ~255LL;
}

namespace {

int wm_run(const char *what, const float *A, const pkcu_weight *W, int M, void *work, pk_tc_epi &e,
           pkcu_stream_t stream) {
  if (!A || !W || !work || M <= 0) return pkcu_fail(PKCU_ERR_ARG, "%s: bad argument", what);
  if (!PK_ALIGNED16(A) || !PK_ALIGNED16(work))
    return pkcu_fail(PKCU_ERR_ARG, "%s: A and work must be 16-byte aligned", what);
  int st = pk_split_rows_bf16x3(A, work, M, W->K, stream);
  if (st) return st;
  e.alpha *= W->alpha;
  return pk_tc_gemm(work, W->planes, W->npb, M, W->N, W->K, &e, stream);
}

}  // namespace

extern "C" int pkcu_wmatmul(const float *A, const pkcu_weight *W, float *C, int M, float alpha, float beta,
                            void *work, pkcu_stream_t stream) {
  pk_tc_epi e = {};
  e.mode = PK_TC_STORE;
  e.alpha = alpha;
  e.beta = beta;
  e.C = C;
  return wm_run("pkcu_wmatmul", A, W, M, work, e, stream);
}

extern "C" int pkcu_wmatmul_bias_swish(const float *A, const pkcu_weight *W, const float *bias, float *D,
                                       int M, void *work, pkcu_stream_t stream) {
  if (!bias) return pkcu_fail(PKCU_ERR_ARG, "pkcu_wmatmul_bias_swish: NULL bias");
  pk_tc_epi e = {};
  e.mode = PK_TC_SWISH;
  e.alpha = 1.0f;
  e.bias = bias;
  e.C = D;
  return wm_run("pkcu_wmatmul_bias_swish", A, W, M, work, e, stream);
}

extern "C" int pkcu_wmatmul_bias_residual(const float *A, const pkcu_weight *W, const float *bias, float *X,
                                          float scale, int M, void *work, pkcu_stream_t stream) {
  if (!bias) return pkcu_fail(PKCU_ERR_ARG, "pkcu_wmatmul_bias_residual: NULL bias");
  pk_tc_epi e = {};
  e.mode = PK_TC_RESID;
  e.alpha = 1.0f;
  e.rscale = scale;
  e.bias = bias;
  e.C = X;
  return wm_run("pkcu_wmatmul_bias_residual", A, W, M, work, e, stream);
}

extern "C" int pkcu_wmatmul_qkv(const float *A, const pkcu_weight *W, const float *bqkv, const float *u,
                                const float *v, float *Qu, float *Qv, float *K, float *V, const pkcu_seq *seq,
                                void *work, pkcu_stream_t stream) {
  if (!seq || !bqkv || !u || !v || !Qu || !Qv || !K || !V)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_wmatmul_qkv: NULL argument");
  if (!W || W->N != 3 * PK_D || W->K != PK_D)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_wmatmul_qkv: the weight must be the fused [1024, 3072] QKV");
  if (seq->frames > 0x7fffffffLL) return pkcu_fail(PKCU_ERR_ARG, "pkcu_wmatmul_qkv: batch too large");
  pk_tc_epi e = {};
  e.mode = PK_TC_QKV;
  e.alpha = 1.0f;
  e.bias = bqkv;
  e.u = u;
  e.v = v;
  e.Qu = Qu;
  e.Qv = Qv;
  e.K = K;
  e.V = V;
  e.seq = seq;
  return wm_run("pkcu_wmatmul_qkv", A, W, (int)seq->frames, work, e, stream);
}

// ── public entry points: pointwise convolutions (csrc/tensor_ops.c:579-590) ──

extern "C" int pkcu_conv_weight_create(const float *w, int Cout, int Cin, int glu, pkcu_stream_t stream,
                                       pkcu_weight **out) {
  if (!out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_conv_weight_create: NULL out");
  *out = nullptr;
  if (!w || Cout <= 0 || Cin <= 0 || Cin % tc::BK || Cout % (glu ? 64 : 32))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_conv_weight_create: Cin %d must be a multiple of 32, Cout %d of %d",
                     Cin, Cout, glu ? 64 : 32);
  pkcu_weight *p = (pkcu_weight *)calloc(1, sizeof(*p));
  if (!p) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_conv_weight_create: host allocation");
  p->K = Cin;
  p->N = Cout;
  p->bits = 32;
  p->npb = 3;
  p->alpha = 1.0f;
  p->conv = 1;
  p->glu = glu != 0;
  const size_t bytes = (size_t)3 * Cin * Cout * 2;
  if (cudaMalloc(&p->planes, bytes) != cudaSuccess) {
    cudaGetLastError();
    p->planes = nullptr;
    pkcu_weight_destroy(p);
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_conv_weight_create: %zu bytes", bytes);
  }
  int st = pk_tc_prepare_rows(w, Cout, Cin, p->glu, p->planes, stream);
  if (!st && cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess)
    st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_conv_weight_create: %s", cudaGetErrorString(cudaGetLastError()));
  if (st) {
    pkcu_weight_destroy(p);
    return st;
  }
  *out = p;
  return PKCU_OK;
}

namespace {

// One utterance of T frames as a batch descriptor (uniform: no device arrays).
pkcu_seq one_item(int T) {
  pkcu_seq q;
  memset(&q, 0, sizeof(q));
  q.dev.n_items = 1;
  q.dev.uniform_T = T;
  q.dev.max_T = T;
  q.frames = T;
  return q;
}

int pw_run(const char *what, const float *x, const pkcu_weight *W, const float *b, float *out, int T,
           int glu, void *work, pkcu_stream_t stream) {
  if (!x || !W || !out || !work || T <= 0 || !W->conv)
    return pkcu_fail(PKCU_ERR_ARG, "%s: bad argument (a pkcu_conv_weight_create weight)", what);
  if (glu != W->glu)
    return pkcu_fail(PKCU_ERR_ARG, "%s: the weight was prepared %s the GLU interleave", what,
                     glu ? "without" : "with");
  if (!PK_ALIGNED16(work)) return pkcu_fail(PKCU_ERR_ARG, "%s: work must be 16-byte aligned", what);
  pkcu_seq q = one_item(T);
  int st = pk_split_cf_t(x, work, W->K, &q, stream);
  if (st) return st;
  pk_tc_epi e = {};
  e.mode = glu ? PK_TC_GLU : PK_TC_CF;
  e.alpha = 1.0f;
  e.bias = b;
  e.C = out;
  e.seq = &q;
  return pk_tc_gemm(work, W->planes, 3, T, W->N, W->K, &e, stream);
}

}  // namespace

extern "C" int pkcu_pointwise_conv1d(const float *x, const pkcu_weight *W, const float *b, float *out, int T,
                                     void *work, pkcu_stream_t stream) {
  return pw_run("pkcu_pointwise_conv1d", x, W, b, out, T, 0, work, stream);
}

extern "C" int pkcu_pointwise_conv1d_glu(const float *x, const pkcu_weight *W, const float *b, float *gated,
                                         int T, void *work, pkcu_stream_t stream) {
  return pw_run("pkcu_pointwise_conv1d_glu", x, W, b, gated, T, 1, work, stream);
}
