// k_layout.cu -- attention head gathers and concat (pure data movement, plus
// the QKV bias and pos_bias_u/v adds).
//
//   QKV split  (csrc/encoder.c:313-356): qkv [T, 3D] + bqkv -> Qu = Q + u[h],
//              Qv = Q + v[h], K, V as [H, T, 128]; 12 bytes read, 16 written
//              per frame-channel (28 T D bytes per item).
//   pos split  (csrc/encoder.c:362-368): P [2T-1, D] -> P_h [H, 2T-1, 128].
//   head concat(csrc/encoder.c:410-415): [H, T, 128] -> [T, D].
//
// One CTA = 8 warps = the 8 heads of FRAMES consecutive frames; a warp moves
// one 512-byte head slice per frame with one float4 per lane, so every load
// and store is a fully coalesced 512-byte run. Values are copied or added
// once (q + bq, then + u), exactly as the reference rounds them.
#include "pk_common.cuh"

namespace pk {

constexpr int LY_FRAMES = 4;
constexpr int LY_THREADS = 32 * PK_H;

__global__ void __launch_bounds__(LY_THREADS)
qkv_split_kernel(const float *__restrict__ qkv, const float *__restrict__ bqkv,
                 const float *__restrict__ u, const float *__restrict__ v,
                 float *__restrict__ Qu, float *__restrict__ Qv, float *__restrict__ K,
                 float *__restrict__ V, SeqDev seq) {
  const int item = blockIdx.y;
  const int T = seq_T(seq, item);
  const int t0 = blockIdx.x * LY_FRAMES;
  if (t0 >= T) return;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = h * PK_DH + 4 * lane;
  const float4 bq = bqkv ? __ldg(reinterpret_cast<const float4 *>(bqkv + c)) : make_float4(0, 0, 0, 0);
  const float4 bk = bqkv ? __ldg(reinterpret_cast<const float4 *>(bqkv + PK_D + c)) : make_float4(0, 0, 0, 0);
  const float4 bv = bqkv ? __ldg(reinterpret_cast<const float4 *>(bqkv + 2 * PK_D + c)) : make_float4(0, 0, 0, 0);
  const float4 uu = __ldg(reinterpret_cast<const float4 *>(u + c));
  const float4 vv = __ldg(reinterpret_cast<const float4 *>(v + c));
  const long long f0 = seq_frame_off(seq, item);
  const long long ob = f0 * PK_D + (long long)h * T * PK_DH + 4 * lane;
  const int n = min(LY_FRAMES, T - t0);
  float4 q[LY_FRAMES], k[LY_FRAMES], w[LY_FRAMES];
#pragma unroll
  for (int f = 0; f < LY_FRAMES; f++) {
    if (f < n) {
      const float *row = qkv + (f0 + t0 + f) * (3 * PK_D);
      q[f] = ldg4_stream(row + c);
      k[f] = ldg4_stream(row + PK_D + c);
      w[f] = ldg4_stream(row + 2 * PK_D + c);
    }
  }
#pragma unroll
  for (int f = 0; f < LY_FRAMES; f++) {
    if (f < n) {
      const long long o = ob + (long long)(t0 + f) * PK_DH;
      const float4 qb = add4(q[f], bq);
      st4(Qu + o, add4(qb, uu));
      st4(Qv + o, add4(qb, vv));
      st4(K + o, add4(k[f], bk));
      st4(V + o, add4(w[f], bv));
    }
  }
}

__global__ void __launch_bounds__(LY_THREADS)
pos_split_kernel(const float *__restrict__ P, float *__restrict__ Ph, SeqDev seq) {
  const int item = blockIdx.y;
  const int L = 2 * seq_T(seq, item) - 1;
  const int p0 = blockIdx.x * LY_FRAMES;
  if (p0 >= L) return;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long r0 = seq_pos_off(seq, item);
  const int n = min(LY_FRAMES, L - p0);
  float4 a[LY_FRAMES];
#pragma unroll
  for (int f = 0; f < LY_FRAMES; f++)
    if (f < n) a[f] = ldg4_stream(P + (r0 + p0 + f) * PK_D + h * PK_DH + 4 * lane);
#pragma unroll
  for (int f = 0; f < LY_FRAMES; f++)
    if (f < n) st4(Ph + r0 * PK_D + ((long long)h * L + p0 + f) * PK_DH + 4 * lane, a[f]);
}

__global__ void __launch_bounds__(LY_THREADS)
head_concat_kernel(const float *__restrict__ ah, float *__restrict__ attn, SeqDev seq) {
  const int item = blockIdx.y;
  const int T = seq_T(seq, item);
  const int t0 = blockIdx.x * LY_FRAMES;
  if (t0 >= T) return;
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long f0 = seq_frame_off(seq, item);
  const int n = min(LY_FRAMES, T - t0);
  float4 a[LY_FRAMES];
#pragma unroll
  for (int f = 0; f < LY_FRAMES; f++)
    if (f < n) a[f] = ldg4_stream(ah + f0 * PK_D + ((long long)h * T + t0 + f) * PK_DH + 4 * lane);
#pragma unroll
  for (int f = 0; f < LY_FRAMES; f++)
    if (f < n) st4(attn + (f0 + t0 + f) * PK_D + h * PK_DH + 4 * lane, a[f]);
}

static int check(const pkcu_seq *seq, const char *what) {
  if (!seq) return pkcu_fail(PKCU_ERR_ARG, "%s: NULL seq", what);
  if (seq->dev.n_items > 65535)
    return pkcu_fail(PKCU_ERR_ARG, "%s: at most 65535 items per call", what);
  return PKCU_OK;
}

}  // namespace pk

using namespace pk;

extern "C" int pkcu_qkv_split_uv(const float *qkv, const float *bqkv, const float *u,
                                 const float *v, float *Qu, float *Qv, float *K, float *V,
                                 const pkcu_seq *seq, pkcu_stream_t stream) {
  int st = check(seq, "pkcu_qkv_split_uv");
  if (st) return st;
  if (!qkv || !u || !v || !Qu || !Qv || !K || !V)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_qkv_split_uv: NULL pointer");
  if (!PK_ALIGNED16(qkv) || !PK_ALIGNED16(u) || !PK_ALIGNED16(v) || !PK_ALIGNED16(Qu) ||
      !PK_ALIGNED16(Qv) || !PK_ALIGNED16(K) || !PK_ALIGNED16(V) || (bqkv && !PK_ALIGNED16(bqkv)))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_qkv_split_uv: pointers must be 16-byte aligned");
  if (seq->frames == 0) return PKCU_OK;
  dim3 grid((unsigned)((seq->dev.max_T + LY_FRAMES - 1) / LY_FRAMES), (unsigned)seq->dev.n_items);
  qkv_split_kernel<<<grid, LY_THREADS, 0, (cudaStream_t)stream>>>(qkv, bqkv, u, v, Qu, Qv, K, V,
                                                                  seq->dev);
  return pkcu_launch_status("pkcu_qkv_split_uv");
}

extern "C" int pkcu_pos_head_split(const float *P, float *P_h, const pkcu_seq *seq,
                                   pkcu_stream_t stream) {
  int st = check(seq, "pkcu_pos_head_split");
  if (st) return st;
  if (!P || !P_h || !PK_ALIGNED16(P) || !PK_ALIGNED16(P_h))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_pos_head_split: bad or misaligned pointer");
  if (seq->frames == 0) return PKCU_OK;
  dim3 grid((unsigned)((2 * seq->dev.max_T - 1 + LY_FRAMES - 1) / LY_FRAMES),
            (unsigned)seq->dev.n_items);
  pos_split_kernel<<<grid, LY_THREADS, 0, (cudaStream_t)stream>>>(P, P_h, seq->dev);
  return pkcu_launch_status("pkcu_pos_head_split");
}

extern "C" int pkcu_head_concat(const float *attn_h, float *attn, const pkcu_seq *seq,
                                pkcu_stream_t stream) {
  int st = check(seq, "pkcu_head_concat");
  if (st) return st;
  if (!attn_h || !attn || !PK_ALIGNED16(attn_h) || !PK_ALIGNED16(attn))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_head_concat: bad or misaligned pointer");
  if (seq->frames == 0) return PKCU_OK;
  dim3 grid((unsigned)((seq->dev.max_T + LY_FRAMES - 1) / LY_FRAMES), (unsigned)seq->dev.n_items);
  head_concat_kernel<<<grid, LY_THREADS, 0, (cudaStream_t)stream>>>(attn_h, attn, seq->dev);
  return pkcu_launch_status("pkcu_head_concat");
}
