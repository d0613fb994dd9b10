// k_decode.cu -- batched greedy RNN-T decode (csrc/decoder.c:80-132) for a
// batch of utterances: the non-GEMM steps as kernels, every matrix-vector
// product of the reference (LSTM W_i x / W_r h, joint.enc / .pred / .out) as a
// batched GEMM at a hook.
//
// The reference decodes one utterance at a time: from a decoder step on the
// blank token, per frame t up to 10 times { joint(enc_t, pred); argmax; blank
// -> next frame; else emit and run a decoder step }. Here every utterance of
// the batch advances by one joint evaluation per iteration:
//      (x0 holds the embedding row of each pending row's token)
//      -> hooks L0_WI (x0 W_i0^T), L0_WR (h0 W_r0^T)
//   1. LSTM layer 0 cell on the pending rows                         (h0, c0)
//      -> hooks L1_WI (h0 W_i1^T), L1_WR (h1 W_r1^T)
//   2. LSTM layer 1 cell on the pending rows                         (h1, c1)
//      -> hook PRED (h1 joint.pred)
//   3. joint hidden of the active rows: relu((enc_t + b_enc) + (pred + b_pred))
//      -> hook OUT (hidden joint.out)
//   4. logits + b_out, first-maximum argmax, state update: blank -> next
//      frame; else emit, copy the token's embedding row into x0 (the next
//      iteration's pending decoder step), next frame after the 10th symbol.
// Each utterance thus goes through exactly the reference's sequence of
// operations (its k-th joint evaluation is iteration k; the decoder step that
// precedes it runs in the same iteration), interleaved with the others.
// Rows that are not pending / not active ignore the products of their row.
//
// The fused form (pkcu_greedy_decode_fused) runs the same iteration with the
// decoder's own product kernels: each LSTM layer is one kernel (both gate
// products + the cell) over the list of pending rows that the previous select
// built, writing the new h into separate buffers that the select commits;
// pred + joint hidden and out follow, then the same select.
#include "pk_common.cuh"

namespace pk {

constexpr int DEC_H = 640, DEC_V = 1025, DEC_BLANK = 1024, DEC_MAX_SYM = 10;
constexpr int DEC_H4 = DEC_H / 4;

struct DecState {      // one entry per utterance
  int *t, *s, *ntok, *last, *pending, *evals;
  int *live;           // rows still active or pending after the last select
  int *plist, *pcount; // the pending rows, in any order (fused decode)
};

__global__ void dec_init_kernel(DecState st, float *__restrict__ lstm, float *__restrict__ x0,
                                const float *__restrict__ embed, int B) {
  // lstm: h0, h1, c0, c1, each [B, 640]; x0 = the blank token's embedding row
  const long long n4 = 4LL * B * DEC_H4;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n4;
       e += (long long)gridDim.x * blockDim.x) {
    st4(lstm + 4 * e, make_float4(0.f, 0.f, 0.f, 0.f));
    if (e < (long long)B * DEC_H4)
      st4(x0 + 4 * e, __ldg(reinterpret_cast<const float4 *>(embed + (long long)DEC_BLANK * DEC_H) +
                            e % DEC_H4));
  }
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < B; b += gridDim.x * blockDim.x) {
    st.t[b] = 0;
    st.s[b] = 0;
    st.ntok[b] = 0;
    st.last[b] = DEC_BLANK;   // the first decoder step runs on blank (csrc/decoder.c:95-97)
    st.pending[b] = 1;
    st.evals[b] = 0;
    st.plist[b] = b;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *st.pcount = B;
}

__device__ __forceinline__ float dec_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

// pk_lstm_step's cell (csrc/tensor_ops.c:608-626) on the pending rows: gates =
// (W_r h + W_i x) + (B[i] + B[4H + i]) in the ONNX order i, o, f, c;
// c = f c + i g; h = o tanh(c). h and c are updated in place.
__global__ void dec_cell_kernel(const float *__restrict__ gi, const float *__restrict__ gr,
                                const float *__restrict__ bias, float *__restrict__ h,
                                float *__restrict__ c, const int *__restrict__ pending, int B) {
  const long long n = (long long)B * DEC_H;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(e / DEC_H), j = (int)(e - (long long)b * DEC_H);
    if (!pending[b]) continue;
    const long long r = (long long)b * 4 * DEC_H;
    float g[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int i = q * DEC_H + j;
      g[q] = (__ldg(gr + r + i) + __ldg(gi + r + i)) + (__ldg(bias + i) + __ldg(bias + 4 * DEC_H + i));
    }
    const float ig = dec_sigmoid(g[0]), og = dec_sigmoid(g[1]), fg = dec_sigmoid(g[2]);
    const float cg = tanhf(g[3]);
    const float cn = fg * c[e] + ig * cg;
    c[e] = cn;
    h[e] = og * tanhf(cn);
  }
}

// pk_joint's hidden (csrc/decoder.c:44-67) for the active rows: enc_proj + bias,
// pred_proj + bias, their sum, ReLU; inactive rows get zeros. Resets the live
// count that this iteration's select accumulates.
__global__ void dec_joint_kernel(const float *__restrict__ encp, const float *__restrict__ enc_b,
                                 const float *__restrict__ pred, const float *__restrict__ pred_b,
                                 float *__restrict__ hidden, const int *__restrict__ t, SeqDev seq,
                                 int B, int *live) {
  if (blockIdx.x == 0 && threadIdx.x == 0) *live = 0;
  const long long n4 = (long long)B * DEC_H4;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n4;
       e += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(e / DEC_H4), j4 = (int)(e - (long long)b * DEC_H4);
    const int tb = t[b];
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tb < seq_T(seq, b)) {
      const float4 ev = __ldg(reinterpret_cast<const float4 *>(encp + (seq_frame_off(seq, b) + tb) * DEC_H) + j4);
      const float4 eb = __ldg(reinterpret_cast<const float4 *>(enc_b) + j4);
      const float4 pv = ld4(pred + 4 * e);
      const float4 pb = __ldg(reinterpret_cast<const float4 *>(pred_b) + j4);
      const float hx = (ev.x + eb.x) + (pv.x + pb.x), hy = (ev.y + eb.y) + (pv.y + pb.y);
      const float hz = (ev.z + eb.z) + (pv.z + pb.z), hw = (ev.w + eb.w) + (pv.w + pb.w);
      o = make_float4(hx < 0.f ? 0.f : hx, hy < 0.f ? 0.f : hy, hz < 0.f ? 0.f : hz,
                      hw < 0.f ? 0.f : hw);
    }
    st4(hidden + 4 * e, o);
  }
}

constexpr int SEL_ROWS = 8;   // rows (warps) per CTA

// Where the fused decode keeps the new LSTM states of the pending rows until
// the select of the same iteration commits them (null for the hook forms,
// whose cell kernel updates h in place).
struct DecCommit {
  const float *h0n, *h1n;
  float *h0, *h1;
};

// Logits = joint.out product + bias, first-maximum argmax (strict '>' in index
// order, csrc/decoder.c:106-114; a NaN never wins, a NaN first logit keeps 0),
// then the greedy state machine of csrc/decoder.c:99-129 for one row. With a
// commit, a row that was pending first takes its new LSTM states, and a row
// left pending is appended to the pending list.
__global__ void __launch_bounds__(32 * SEL_ROWS)
dec_select_kernel(const float *__restrict__ out, const float *__restrict__ out_b, DecState st,
                  int *__restrict__ tokens, const float *__restrict__ embed, float *__restrict__ x0,
                  SeqDev seq, int B, DecCommit cm) {
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * SEL_ROWS + (threadIdx.x >> 5);
  if (b >= B) return;
  // every load this row needs before its argmax is issued here, together: the
  // row state, this lane's logits and, for a commit, the new LSTM states
  const int T = seq_T(seq, b);
  const int tb = st.t[b];
  const bool active = tb < T;
  const bool commit = cm.h0 && st.pending[b];
  int s_in = 0, ntok_in = 0, evals_in = 0;
  if (lane == 0 && active) {
    s_in = st.s[b];
    ntok_in = st.ntok[b];
    evals_in = st.evals[b];
  }
  const float *l = out + (long long)b * DEC_V;
  constexpr int NV = (DEC_V + 31) / 32;
  float xv[NV];
  if (active) {
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const int v = lane + 32 * i;
      xv[i] = v < DEC_V ? l[v] + __ldg(out_b + v) : 0.f;
    }
  }
  if (commit) {
    const long long r = (long long)b * DEC_H;
    float4 n0[DEC_H4 / 32], n1[DEC_H4 / 32];
#pragma unroll
    for (int k = 0; k < DEC_H4 / 32; k++) {
      n0[k] = ld4(cm.h0n + r + 4 * (lane + 32 * k));
      n1[k] = ld4(cm.h1n + r + 4 * (lane + 32 * k));
    }
#pragma unroll
    for (int k = 0; k < DEC_H4 / 32; k++) {
      st4(cm.h0 + r + 4 * (lane + 32 * k), n0[k]);
      st4(cm.h1 + r + 4 * (lane + 32 * k), n1[k]);
    }
  }
  if (!active) {                       // finished: its last decoder step (if any) has run
    if (lane == 0) st.pending[b] = 0;
    return;
  }
  // the comparisons in index order
  float bv = -INFINITY;
  int bi = INT_MAX;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int v = lane + 32 * i;
    if (v < DEC_V && xv[i] > bv) { bv = xv[i]; bi = v; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(PK_FULL_MASK, bv, o);
    const int oi = __shfl_xor_sync(PK_FULL_MASK, bi, o);
    if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
  }
  const float first = __shfl_sync(PK_FULL_MASK, xv[0], 0);   // logit 0 + its bias (lane 0's v = 0)
  const int best = (isnan(first) || bi == INT_MAX) ? 0 : bi;
  if (best != DEC_BLANK) {             // the next decoder step's input (csrc/decoder.c:19)
    const float4 *src = reinterpret_cast<const float4 *>(embed + (long long)best * DEC_H);
    float4 *dst = reinterpret_cast<float4 *>(x0 + (long long)b * DEC_H);
    for (int j = lane; j < DEC_H4; j += 32) dst[j] = __ldg(src + j);
  }
  if (lane != 0) return;
  st.evals[b] = evals_in + 1;
  int t = tb, s = s_in, pend = 0;
  if (best == DEC_BLANK) {
    t += 1;
    s = 0;
  } else {
    const int n = ntok_in;
    tokens[DEC_MAX_SYM * seq_frame_off(seq, b) + n] = best;
    st.ntok[b] = n + 1;
    st.last[b] = best;
    pend = 1;
    if (++s == DEC_MAX_SYM) {          // the symbol loop ends after 10 emissions
      t += 1;
      s = 0;
    }
  }
  st.t[b] = t;
  st.s[b] = s;
  st.pending[b] = pend;
  if (pend && cm.h0) st.plist[atomicAdd(st.pcount, 1)] = b;
  if (t < T || pend) atomicAdd(st.live, 1);
}

// ── the decode's own products (pkcu_greedy_decode_fused) ─────────────────
// Every product of an iteration has M = batch rows and K = 640: a skinny
// fp32 GEMM whose weights (31 MB for all six) stay in L2 from one iteration
// to the next. Each warp holds DEC_RW weight rows (of K contiguous floats) in
// registers -- lane l owns k in [20 l, 20 l + 20) -- and streams the input
// rows of its CTA's batch slice: per row 5 float4 loads, 40 packed f32x2
// FMAs and a 6-shuffle reduce-scatter that leaves row r's dot product in
// lanes 8 r .. 8 r + 7. The LSTM kernel applies the cell to its own gate
// products, the pred kernel the joint bias + add + ReLU, so an iteration is
// five kernels: lstm 0, lstm 1, pred + joint, out, select.

constexpr int DEC_RK = DEC_H / 32;   // consecutive k per lane
constexpr int DEC_RW = 4;            // weight rows per warp
constexpr int LSTM_UNITS = 4;        // hidden units per CTA: 8 warps = unit x {W_i, W_r}

// Rows rows[0..3] of W [nrows, 640] (rows past nrows read as 0), this lane's
// k range, kept as float4 so that every packed FMA takes an aligned pair.
__device__ __forceinline__ void dec_load_rows(float4 (&w)[DEC_RW][DEC_RK / 4], const float *__restrict__ W,
                                              const int (&rows)[DEC_RW], int nrows, int lane) {
#pragma unroll
  for (int r = 0; r < DEC_RW; r++) {
#pragma unroll
    for (int i = 0; i < DEC_RK / 4; i++)
      w[r][i] = rows[r] < nrows
                    ? __ldg(reinterpret_cast<const float4 *>(W + (long long)rows[r] * DEC_H + DEC_RK * lane) + i)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// This lane's partial dot products (its 20 k) of the warp's 4 rows with the
// input row x [640] (shared memory).
__device__ __forceinline__ void dec_dot_partial(const float4 (&w)[DEC_RW][DEC_RK / 4], const float *x, int lane,
                                                float *v) {
  float4 xv[DEC_RK / 4];
#pragma unroll
  for (int i = 0; i < DEC_RK / 4; i++) xv[i] = *reinterpret_cast<const float4 *>(x + DEC_RK * lane + 4 * i);
#pragma unroll
  for (int r = 0; r < DEC_RW; r++) {
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < DEC_RK / 4; i++) {
      acc = fma2(make_float2(w[r][i].x, w[r][i].y), make_float2(xv[i].x, xv[i].y), acc);
      acc = fma2(make_float2(w[r][i].z, w[r][i].w), make_float2(xv[i].z, xv[i].w), acc);
    }
    v[r] = acc.x + acc.y;
  }
}

// Reduce-scatter of 16 per-lane values v[j] over the warp: returns, in lanes
// 2 j' and 2 j' + 1, the warp-wide sum of value j' (bit-identical in both).
// Lane bit 4 keeps values 0..7 or 8..15, bit 3 half of those, then bits 2 and
// 1; bit 0 sums the pair.
__device__ __forceinline__ float dec_reduce16(float (&v)[16], int lane) {
#pragma unroll
  for (int half = 8, bit = 16; half >= 1; half >>= 1, bit >>= 1) {
    const bool hi = lane & bit;
#pragma unroll
    for (int i = 0; i < half; i++) {
      const float send = hi ? v[i] : v[i + half];
      const float keep = hi ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(PK_FULL_MASK, send, bit);
    }
  }
  return v[0] + __shfl_xor_sync(PK_FULL_MASK, v[0], 1);
}

// Input rows are staged through shared memory in groups of DEC_G batch rows,
// double-buffered with cp.async so that the next group's loads overlap this
// group's FMAs, together with what the epilogue needs per row.
constexpr int DEC_G = 8;
constexpr int DEC_H4Q = DEC_H / 4;

struct LstmStage {
  float x[DEC_G][2][DEC_H];   // x and h_in rows
  float4 c[DEC_G];            // c[b][j0 .. j0 + 3] (this CTA's units)
  int row[DEC_G];             // batch row b of the slot
  int use[DEC_G];             // slot within the segment
};
struct RowStage {
  float x[DEC_G][DEC_H];
  int use[DEC_G];             // active (t < T) and in range
  long long enc_row[DEC_G];   // frame index of the row's current frame
};
constexpr size_t DEC_LSTM_SMEM = 2 * sizeof(LstmStage);
static_assert(DEC_G == 8, "one staging warp per row slot of a 256-thread CTA");
constexpr size_t DEC_ROW_SMEM = 2 * sizeof(RowStage);

// Warp w of the 8 stages row slot w: its NSRC source rows (when `use`) as
// 5 x 32 16-byte copies each, at offsets fixed at compile time.
template <int NSRC>
__device__ __forceinline__ void dec_stage_row(float *x, const float *s0, const float *s1, long long b, bool use,
                                              int lane) {
  if (!use) return;
#pragma unroll
  for (int which = 0; which < NSRC; which++) {
    const float *src = (which ? s1 : s0) + b * DEC_H + 4 * lane;
    float *dst = x + which * DEC_H + 4 * lane;
#pragma unroll
    for (int k = 0; k < DEC_H4Q / 32; k++) cp_async16(dst + 128 * k, src + 128 * k);
  }
}

// Slot w of the group starting at list index i0: the pending row plist[i0 + w]
// (when below i_hi), its x and h_in rows and this CTA's slice of c.
__device__ __forceinline__ void lstm_stage(LstmStage *st, const float *x, const float *h_in, const float *c,
                                           const int *plist, int j0, int i0, int i_hi) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool use = i0 + w < i_hi;
  const int b = use ? plist[i0 + w] : 0;
  dec_stage_row<2>(&st->x[w][0][0], x, h_in, b, use, lane);
  if (lane == 0) {
    st->use[w] = use;
    st->row[w] = b;
    if (use) cp_async16(&st->c[w], c + (long long)b * DEC_H + j0);
  }
}

// Work split of the product kernels: the flattened space f = group * B + b
// (group = the CTA-sized set of weight rows, b = batch row) is cut into equal
// shares of `per` rows, one per CTA (the grid is about two CTAs per SM). A
// share covers one or more segments (group, rows [b_lo, b_hi)); the macro
// opens the loop over them -- every thread of the CTA runs the same segments
// -- and the kernel body closes it.
#define DEC_SEGMENTS(n_groups)                                                         \
  const long long f_end = min((long long)(n_groups) * B, (long long)(blockIdx.x + 1) * per); \
  for (long long f = (long long)blockIdx.x * per; f < f_end;) {                       \
    const int grp = (int)(f / B);                                                      \
    const int b_lo = (int)(f - (long long)grp * B);                                    \
    const int b_hi = (int)min((long long)B, b_lo + (f_end - f));                        \
    f += b_hi - b_lo;

// One LSTM layer (pk_lstm_step, csrc/tensor_ops.c:596-629) for the pending
// rows plist[0 .. *pcount): the flattened space f = group * n + i (group = 4
// hidden units j0 .. j0 + 3, i = list index) is shared out as above. Warp
// 2u + m of a segment computes gate rows {q 640 + j0 + u} of W_i with x
// (m = 0) or of W_r with h_in (m = 1); the gates (W_r h + W_i x) +
// (B[i] + B[4H + i]) then go through the cell (warp 0, one lane per row and
// unit): c in place, the new h into h_out (other CTAs still read h_in).
__global__ void __launch_bounds__(256, 2) dec_lstm_kernel(const float *__restrict__ Wi, const float *__restrict__ Wr,
                                                          const float *__restrict__ bias, const float *__restrict__ x,
                                                          const float *__restrict__ h_in, float *__restrict__ h_out,
                                                          float *__restrict__ c, const int *__restrict__ plist,
                                                          const int *__restrict__ pcount) {
  extern __shared__ __align__(16) unsigned char dec_smem[];
  LstmStage *stage = reinterpret_cast<LstmStage *>(dec_smem);
  __shared__ float g[2][DEC_G][LSTM_UNITS][2][4];   // [group parity][row slot][unit][W_i, W_r][gate]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u = warp >> 1, m = warp & 1;
  const int B = *pcount;   // the segments' "batch": the list
  if (B == 0) return;
  const long long total = (long long)(DEC_H / LSTM_UNITS) * B;
  const int per = (int)max((long long)DEC_G, (total + gridDim.x - 1) / gridDim.x);
  DEC_SEGMENTS(DEC_H / LSTM_UNITS)
  const int j0 = grp * LSTM_UNITS;
  float4 w[DEC_RW][DEC_RK / 4];
  const int rows[DEC_RW] = {j0 + u, DEC_H + j0 + u, 2 * DEC_H + j0 + u, 3 * DEC_H + j0 + u};
  dec_load_rows(w, m ? Wr : Wi, rows, 4 * DEC_H, lane);
  // the epilogue lane (warp 0): row slot eb, unit eu; bias sums B[i] + B[4H + i]
  const int eb = lane / LSTM_UNITS, eu = lane % LSTM_UNITS, ej = j0 + eu;
  float bs[4];
#pragma unroll
  for (int q = 0; q < 4; q++) bs[q] = __ldg(bias + q * DEC_H + ej) + __ldg(bias + 4 * DEC_H + q * DEC_H + ej);
  lstm_stage(stage, x, h_in, c, plist, j0, b_lo, b_hi);
  cp_async_commit();
  for (int g0 = b_lo, it = 0; g0 < b_hi; g0 += DEC_G, it++) {
    const int par = it & 1;
    const LstmStage *cur = stage + par;
    if (g0 + DEC_G < b_hi) lstm_stage(stage + (par ^ 1), x, h_in, c, plist, j0, g0 + DEC_G, b_hi);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    // the epilogue lane's inputs, read before the buffer can be restaged
    const int euse = warp == 0 ? cur->use[eb] : 0;
    const int erow = warp == 0 ? cur->row[eb] : 0;
    const float ec = warp == 0 ? reinterpret_cast<const float *>(&cur->c[eb])[eu] : 0.f;
#pragma unroll
    for (int h = 0; h < DEC_G / 4; h++) {   // 4 rows x 4 gates per reduction
      float v[16];
#pragma unroll
      for (int k = 0; k < 4; k++) {
        if (cur->use[4 * h + k]) {   // warp-uniform
          dec_dot_partial(w, cur->x[4 * h + k][m], lane, v + 4 * k);
        } else {
          v[4 * k] = v[4 * k + 1] = v[4 * k + 2] = v[4 * k + 3] = 0.f;
        }
      }
      const float t = dec_reduce16(v, lane);
      if ((lane & 1) == 0) g[par][4 * h + (lane >> 3)][u][m][(lane >> 1) & 3] = t;
    }
    __syncthreads();
    if (warp == 0 && euse) {
      const long long e = (long long)erow * DEC_H + ej;
      float gt[4];
#pragma unroll
      for (int q = 0; q < 4; q++) gt[q] = (g[par][eb][eu][1][q] + g[par][eb][eu][0][q]) + bs[q];
      const float ig = dec_sigmoid(gt[0]), og = dec_sigmoid(gt[1]), fg = dec_sigmoid(gt[2]);
      const float cg = tanhf(gt[3]);
      const float cn = fg * ec + ig * cg;
      c[e] = cn;
      h_out[e] = og * tanhf(cn);
    }
  }
  cp_async_wait<0>();
  }
}

// Slot w: batch row g0 + w when active, its input row taken from src_new for
// the rows with pending set (src_new non-null) and from src otherwise.
__device__ __forceinline__ void row_stage(RowStage *st, const float *src, const float *src_new,
                                          const int *pending, const int *t, SeqDev seq, int g0, int b_hi) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = g0 + w;
  const int tb = b < b_hi ? t[b] : 0;
  const bool use = b < b_hi && tb < seq_T(seq, b);
  const float *from = (src_new && use && pending[b]) ? src_new : src;
  dec_stage_row<1>(&st->x[w][0], from, nullptr, b, use, lane);
  if (lane == 0) {
    st->use[w] = use;
    st->enc_row[w] = use ? seq_frame_off(seq, b) + tb : 0;
  }
}

// pk_joint's pred projection and hidden (csrc/decoder.c:44-67): for the active
// rows hidden = relu((enc_t + b_enc) + (h1 joint.pred + b_pred)), zeros for the
// others; h1 is the new state (h1n) for the rows with a decoder step this
// iteration. JpT: joint.pred transposed, [640 out, 640 in]. Warp w of a
// segment's group owns outputs 4 (8 group + w) .. +3. Resets the live count
// the select accumulates.
__global__ void __launch_bounds__(256, 2) dec_pred_joint_kernel(const float *__restrict__ JpT, const float *__restrict__ h1,
                                                                const float *__restrict__ h1n, const int *__restrict__ pending,
                                                                const float *__restrict__ encp, const float *__restrict__ enc_b,
                                                                const float *__restrict__ pred_b, float *__restrict__ hidden,
                                                                const int *__restrict__ t, SeqDev seq, int B, int per,
                                                                int *live, int *pcount) {
  extern __shared__ __align__(16) unsigned char dec_smem[];
  RowStage *stage = reinterpret_cast<RowStage *>(dec_smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  DEC_SEGMENTS(DEC_H / (8 * DEC_RW))
  const int n0 = (grp * 8 + warp) * DEC_RW;
  float4 w[DEC_RW][DEC_RK / 4];
  const int rows[DEC_RW] = {n0, n0 + 1, n0 + 2, n0 + 3};
  dec_load_rows(w, JpT, rows, DEC_H, lane);
  const int n = n0 + ((lane >> 1) & 3);
  const float eb = __ldg(enc_b + n), pb = __ldg(pred_b + n);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *live = 0;
    *pcount = 0;   // both LSTM layers of this iteration have read it
  }
  row_stage(stage, h1, h1n, pending, t, seq, b_lo, b_hi);
  cp_async_commit();
  for (int g0 = b_lo, it = 0; g0 < b_hi; g0 += DEC_G, it++) {
    const RowStage *cur = stage + (it & 1);
    if (g0 + DEC_G < b_hi) row_stage(stage + ((it + 1) & 1), h1, h1n, pending, t, seq, g0 + DEC_G, b_hi);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
#pragma unroll
    for (int h = 0; h < DEC_G / 4; h++) {
      float v[16];
#pragma unroll
      for (int k = 0; k < 4; k++) {
        if (cur->use[4 * h + k]) {
          dec_dot_partial(w, cur->x[4 * h + k], lane, v + 4 * k);
        } else {
          v[4 * k] = v[4 * k + 1] = v[4 * k + 2] = v[4 * k + 3] = 0.f;
        }
      }
      const float t = dec_reduce16(v, lane);
      const int bb = 4 * h + (lane >> 3);   // lane pair (l, l + 1): row bb, output n0 + ((l >> 1) & 3)
      if ((lane & 1) == 0 && g0 + bb < b_hi) {
        float *dst = hidden + (long long)(g0 + bb) * DEC_H + n;
        if (cur->use[bb]) {
          const float e = __ldg(encp + cur->enc_row[bb] * DEC_H + n);
          const float hv = (e + eb) + (t + pb);
          *dst = hv < 0.f ? 0.f : hv;
        } else {
          *dst = 0.f;
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  }
}

// The joint.out product (csrc/decoder.c:69-72) of the active rows; JoT:
// joint.out transposed, [1025, 640]. The select kernel adds the bias. Warps
// past the last row still take part in staging and barriers.
__global__ void __launch_bounds__(256, 2) dec_out_kernel(const float *__restrict__ JoT, const float *__restrict__ hidden,
                                                         float *__restrict__ out, const int *__restrict__ t, SeqDev seq,
                                                         int B, int per) {
  extern __shared__ __align__(16) unsigned char dec_smem[];
  RowStage *stage = reinterpret_cast<RowStage *>(dec_smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  DEC_SEGMENTS((DEC_V + 8 * DEC_RW - 1) / (8 * DEC_RW))
  const int n0 = (grp * 8 + warp) * DEC_RW;
  const bool has_rows = n0 < DEC_V;
  float4 w[DEC_RW][DEC_RK / 4];
  const int rows[DEC_RW] = {n0, n0 + 1, n0 + 2, n0 + 3};
  dec_load_rows(w, JoT, rows, DEC_V, lane);
  const int n = n0 + ((lane >> 1) & 3);
  row_stage(stage, hidden, nullptr, nullptr, t, seq, b_lo, b_hi);
  cp_async_commit();
  for (int g0 = b_lo, it = 0; g0 < b_hi; g0 += DEC_G, it++) {
    const RowStage *cur = stage + (it & 1);
    if (g0 + DEC_G < b_hi) row_stage(stage + ((it + 1) & 1), hidden, nullptr, nullptr, t, seq, g0 + DEC_G, b_hi);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (has_rows) {
#pragma unroll
      for (int h = 0; h < DEC_G / 4; h++) {
        float v[16];
#pragma unroll
        for (int k = 0; k < 4; k++) {
          if (cur->use[4 * h + k]) {   // false past b_hi
            dec_dot_partial(w, cur->x[4 * h + k], lane, v + 4 * k);
          } else {
            v[4 * k] = v[4 * k + 1] = v[4 * k + 2] = v[4 * k + 3] = 0.f;
          }
        }
        const float t = dec_reduce16(v, lane);
        const int bb = 4 * h + (lane >> 3);
        if ((lane & 1) == 0 && n < DEC_V && cur->use[bb]) out[(long long)(g0 + bb) * DEC_V + n] = t;
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  }
}

// dst [cols, rows] = src [rows, cols]^T (the joint weights, once per
// pkcu_decoder_set_weights).
__global__ void dec_transpose_kernel(const float *__restrict__ src, float *__restrict__ dst, int rows, int cols) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[(long long)r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[(long long)c * rows + r] = tile[threadIdx.x][i];
  }
}

static unsigned dec_grid(long long work) {
  long long g = (work + 255) / 256;
  const long long cap = (long long)pkcu_sm_count() * 8;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace pk

using namespace pk;

struct pkcu_decoder {
  pkcu_seq *seq;
  int B;
  long long F;
  void *block;             // one device allocation for everything below
  DecState st;
  float *lstm;             // h0, h1, c0, c1 [B, 640] each
  float *hb;               // h0n, h1n [B, 640]: the fused decode's new states of the pending rows
  float *x0, *hidden;      // [B, 640]
  float *encp, *pred, *out, *g0i, *g0r, *g1i, *g1r;
  int *tokens;             // [10 F]: utterance b's tokens from 10 * frame_off(b)
  int *live_host;          // page-locked poll targets, one per graph
  int iterations;          // of the last decode
  int device;
  // Without a hook (or with a capture-safe one, pkcu_greedy_decode_graph),
  // DEC_POLL iterations and the poll copy are one CUDA graph, captured on `gs`
  // for the parameter pointers in `gp` and the hook in `ghook` / `guser`, and
  // replayed.
  cudaStream_t gs;
  cudaEvent_t ev_in, ev_out, ev_done[2];
  cudaGraphExec_t graph[2];   // the same iterations; each copies the live count to its own slot
  pkcu_dec_params gp;
  pkcu_gemm_hook ghook;
  void *guser;
  int gfused;              // the graph holds the fused iteration (weights generation gwgen)
  unsigned gwgen;
  // pkcu_decoder_set_weights: the LSTM matrices (caller's) and the decoder's
  // transposed copies of joint.pred / joint.out
  const float *lw[4];
  float *jt;               // JpT [640, 640] then JoT [1025, 640]
  unsigned wgen;           // 0: no weights set
};

extern "C" void pkcu_decoder_destroy(pkcu_decoder *d) {
  if (!d) return;
  for (int c = 0; c < 2; c++) {
    if (d->graph[c]) cudaGraphExecDestroy(d->graph[c]);
    if (d->ev_done[c]) cudaEventDestroy(d->ev_done[c]);
  }
  if (d->ev_in) cudaEventDestroy(d->ev_in);
  if (d->ev_out) cudaEventDestroy(d->ev_out);
  if (d->gs) cudaStreamDestroy(d->gs);
  if (d->block) cudaFree(d->block);
  if (d->jt) cudaFree(d->jt);
  if (d->live_host) cudaFreeHost(d->live_host);
  pkcu_seq_destroy(d->seq);
  free(d);
}

extern "C" int pkcu_decoder_create(const int *frames, int n_utts, pkcu_decoder **out) {
  if (!out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_decoder_create: NULL out");
  *out = nullptr;
  if (!frames || n_utts <= 0)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_decoder_create: no utterances");
  for (int i = 0; i < n_utts; i++)
    if (frames[i] <= 0 || frames[i] > (1 << 20))
      return pkcu_fail(PKCU_ERR_ARG, "pkcu_decoder_create: utterance %d has %d frames (1 .. 2^20)",
                       i, frames[i]);
  long long F = 0;
  for (int i = 0; i < n_utts; i++) F += frames[i];
  pkcu_decoder *d = (pkcu_decoder *)calloc(1, sizeof(*d));
  if (!d) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_decoder_create: host allocation");
  int st = pkcu_seq_create(frames, n_utts, &d->seq);
  if (st) { pkcu_decoder_destroy(d); return st; }
  d->B = n_utts;
  d->F = F;
  cudaGetDevice(&d->device);
  const size_t B = (size_t)n_utts, H = DEC_H;
  auto up = [](size_t bytes) { return (bytes + 255) & ~(size_t)255; };
  const size_t sz_state = up(sizeof(int) * (7 * B + 2));
  const size_t sz_lstm = up(sizeof(float) * 4 * B * H), sz_bh = up(sizeof(float) * B * H);
  const size_t sz_enc = up(sizeof(float) * (size_t)F * H), sz_out = up(sizeof(float) * B * DEC_V);
  const size_t sz_g = up(sizeof(float) * B * 4 * H), sz_tok = up(sizeof(int) * DEC_MAX_SYM * (size_t)F);
  const size_t total = sz_state + sz_lstm + 5 * sz_bh + sz_enc + sz_out + 4 * sz_g + sz_tok;
  if (cudaMalloc(&d->block, total) != cudaSuccess) {
    cudaGetLastError();
    d->block = nullptr;
    pkcu_decoder_destroy(d);
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_decoder_create: device allocation of %zu bytes", total);
  }
  if (cudaMallocHost(&d->live_host, 2 * sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    d->live_host = nullptr;
    pkcu_decoder_destroy(d);
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_decoder_create: page-locked host allocation");
  }
  char *p = (char *)d->block;
  int *si = (int *)p;
  d->st = DecState{si, si + B, si + 2 * B, si + 3 * B, si + 4 * B, si + 5 * B, si + 6 * B,
                   si + 6 * B + 1, si + 7 * B + 1};
  p += sz_state;
  d->lstm = (float *)p; p += sz_lstm;
  d->hb = (float *)p; p += 2 * sz_bh;
  d->x0 = (float *)p; p += sz_bh;
  d->hidden = (float *)p; p += sz_bh;
  d->pred = (float *)p; p += sz_bh;
  d->encp = (float *)p; p += sz_enc;
  d->out = (float *)p; p += sz_out;
  d->g0i = (float *)p; p += sz_g;
  d->g0r = (float *)p; p += sz_g;
  d->g1i = (float *)p; p += sz_g;
  d->g1r = (float *)p; p += sz_g;
  d->tokens = (int *)p;
  *out = d;
  return PKCU_OK;
}

extern "C" int pkcu_decoder_buffers(const pkcu_decoder *d, pkcu_dec_gemm_outputs *go,
                                    pkcu_dec_gemm_inputs *gi) {
  if (!d || !go || !gi) return pkcu_fail(PKCU_ERR_ARG, "pkcu_decoder_buffers: NULL argument");
  const size_t BH = (size_t)d->B * DEC_H;
  go->enc = d->encp;
  go->pred = d->pred;
  go->out = d->out;
  go->g0i = d->g0i;
  go->g0r = d->g0r;
  go->g1i = d->g1i;
  go->g1r = d->g1r;
  gi->x0 = d->x0;
  gi->h0 = d->lstm;
  gi->h1 = d->lstm + BH;
  gi->hidden = d->hidden;
  return PKCU_OK;
}

extern "C" int pkcu_decoder_iterations(const pkcu_decoder *d) { return d ? d->iterations : -1; }

constexpr int DEC_POLL = 8;   // iterations between two reads of the live count

// One iteration (kernels and hooks) on stream s.
static int dec_iteration(pkcu_decoder *d, const pkcu_dec_params *prm, pkcu_gemm_hook hook,
                         void *hook_user, cudaStream_t s) {
  const int B = d->B;
  const SeqDev seq = d->seq->dev;
  const size_t BH = (size_t)B * DEC_H;
  float *h0 = d->lstm, *h1 = d->lstm + BH, *c0 = d->lstm + 2 * BH, *c1 = d->lstm + 3 * BH;
  const pkcu_stream_t ps = (pkcu_stream_t)s;
  int st = PKCU_OK;
  if (hook) st = hook(hook_user, -1, PKCU_GEMM_DEC_L0_WI, ps);
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_DEC_L0_WR, ps);
  if (st) return st;
  dec_cell_kernel<<<dec_grid(BH), 256, 0, s>>>(d->g0i, d->g0r, prm->lstm0_b, h0, c0, d->st.pending, B);
  st = pkcu_launch_status("pkcu_greedy_decode: lstm 0");
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_DEC_L1_WI, ps);
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_DEC_L1_WR, ps);
  if (st) return st;
  dec_cell_kernel<<<dec_grid(BH), 256, 0, s>>>(d->g1i, d->g1r, prm->lstm1_b, h1, c1, d->st.pending, B);
  st = pkcu_launch_status("pkcu_greedy_decode: lstm 1");
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_DEC_PRED, ps);
  if (st) return st;
  dec_joint_kernel<<<dec_grid(BH / 4), 256, 0, s>>>(d->encp, prm->joint_enc_b, d->pred,
                                                   prm->joint_pred_b, d->hidden, d->st.t, seq, B,
                                                   d->st.live);
  st = pkcu_launch_status("pkcu_greedy_decode: joint");
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_DEC_OUT, ps);
  if (st) return st;
  dec_select_kernel<<<(unsigned)((B + SEL_ROWS - 1) / SEL_ROWS), 32 * SEL_ROWS, 0, s>>>(
      d->out, prm->joint_out_b, d->st, d->tokens, prm->embed, d->x0, seq, B, DecCommit{});
  return pkcu_launch_status("pkcu_greedy_decode: select");
}

static bool same_params(const pkcu_dec_params &a, const pkcu_dec_params &b) {
  return a.embed == b.embed && a.lstm0_b == b.lstm0_b && a.lstm1_b == b.lstm1_b &&
         a.joint_enc_b == b.joint_enc_b && a.joint_pred_b == b.joint_pred_b &&
         a.joint_out_b == b.joint_out_b;
}

// Rows per CTA share for a product kernel over n_groups x B rows: about two
// CTAs per SM, at least one staging group of rows; returns the grid size.
static unsigned dec_share(int n_groups, int B, int *per) {
  const long long total = (long long)n_groups * B, slots = 2LL * pkcu_sm_count();
  long long p = (total + slots - 1) / slots;
  if (p < DEC_G) p = DEC_G;
  *per = (int)p;
  return (unsigned)((total + p - 1) / p);
}

// One iteration of the fused decode on stream s: the LSTM layers on the
// pending list (new states into h0n / h1n), pred + joint, out, select (which
// commits the new states and builds the next list).
static int dec_iteration_fused(pkcu_decoder *d, const pkcu_dec_params *prm, cudaStream_t s) {
  const int B = d->B;
  const size_t BH = (size_t)B * DEC_H;
  float *h0 = d->lstm, *h1 = d->lstm + BH, *c0 = d->lstm + 2 * BH, *c1 = d->lstm + 3 * BH;
  float *h0n = d->hb, *h1n = d->hb + BH;
  const SeqDev seq = d->seq->dev;
  int pp, po, pl;
  const unsigned gl = dec_share(DEC_H / LSTM_UNITS, B, &pl);   // sized for a full list
  const unsigned gp = dec_share(DEC_H / (8 * DEC_RW), B, &pp);
  const unsigned go = dec_share((DEC_V + 8 * DEC_RW - 1) / (8 * DEC_RW), B, &po);
  dec_lstm_kernel<<<gl, 256, DEC_LSTM_SMEM, s>>>(d->lw[0], d->lw[1], prm->lstm0_b, d->x0, h0, h0n, c0,
                                                 d->st.plist, d->st.pcount);
  dec_lstm_kernel<<<gl, 256, DEC_LSTM_SMEM, s>>>(d->lw[2], d->lw[3], prm->lstm1_b, h0n, h1, h1n, c1,
                                                 d->st.plist, d->st.pcount);
  dec_pred_joint_kernel<<<gp, 256, DEC_ROW_SMEM, s>>>(d->jt, h1, h1n, d->st.pending, d->encp, prm->joint_enc_b,
                                                      prm->joint_pred_b, d->hidden, d->st.t, seq, B, pp,
                                                      d->st.live, d->st.pcount);
  dec_out_kernel<<<go, 256, DEC_ROW_SMEM, s>>>(d->jt + DEC_H * DEC_H, d->hidden, d->out, d->st.t, seq, B, po);
  dec_select_kernel<<<(unsigned)((B + SEL_ROWS - 1) / SEL_ROWS), 32 * SEL_ROWS, 0, s>>>(
      d->out, prm->joint_out_b, d->st, d->tokens, prm->embed, d->x0, seq, B, DecCommit{h0n, h1n, h0, h1});
  return pkcu_launch_status("pkcu_greedy_decode_fused: iteration");
}

// Captures DEC_POLL iterations (hook form, with the hook's GEMMs if any, or
// the fused form) + the copy of the live count, twice: graph[c] copies into
// live_host[c], so the host can read one batch's count while the next runs.
static int g_dec_flags[3][64];

static int dec_capture(pkcu_decoder *d, const pkcu_dec_params *prm, pkcu_gemm_hook hook,
                       void *hook_user, int fused) {
  if (fused) {   // no attribute call under capture
    smem_optin(dec_lstm_kernel, DEC_LSTM_SMEM, g_dec_flags[0]);
    smem_optin(dec_pred_joint_kernel, DEC_ROW_SMEM, g_dec_flags[1]);
    smem_optin(dec_out_kernel, DEC_ROW_SMEM, g_dec_flags[2]);
  }
  for (int c = 0; c < 2; c++)
    if (d->graph[c]) {
      cudaGraphExecDestroy(d->graph[c]);
      d->graph[c] = nullptr;
    }
  if (!d->gs && (cudaStreamCreateWithFlags(&d->gs, cudaStreamNonBlocking) != cudaSuccess ||
                 cudaEventCreateWithFlags(&d->ev_in, cudaEventDisableTiming) != cudaSuccess ||
                 cudaEventCreateWithFlags(&d->ev_out, cudaEventDisableTiming) != cudaSuccess ||
                 cudaEventCreateWithFlags(&d->ev_done[0], cudaEventDisableTiming) != cudaSuccess ||
                 cudaEventCreateWithFlags(&d->ev_done[1], cudaEventDisableTiming) != cudaSuccess))
    return pkcu_launch_status("pkcu_greedy_decode: graph stream");
  int st = PKCU_OK;
  for (int c = 0; c < 2 && !st; c++) {
    if (cudaStreamBeginCapture(d->gs, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
      return pkcu_launch_status("pkcu_greedy_decode: begin capture");
    for (int i = 0; i < DEC_POLL && !st; i++)
      st = fused ? dec_iteration_fused(d, prm, d->gs) : dec_iteration(d, prm, hook, hook_user, d->gs);
    if (!st && cudaMemcpyAsync(d->live_host + c, d->st.live, sizeof(int), cudaMemcpyDeviceToHost, d->gs) !=
                   cudaSuccess)
      st = pkcu_launch_status("pkcu_greedy_decode: capture poll copy");
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(d->gs, &g);
    if (!st && ce != cudaSuccess) st = pkcu_launch_status("pkcu_greedy_decode: end capture");
    if (!st && cudaGraphInstantiate(&d->graph[c], g, 0) != cudaSuccess) {
      d->graph[c] = nullptr;
      st = pkcu_launch_status("pkcu_greedy_decode: instantiate");
    }
    if (g) cudaGraphDestroy(g);
  }
  if (!st) {
    d->gp = *prm;
    d->ghook = hook;
    d->guser = hook_user;
    d->gfused = fused;
    d->gwgen = d->wgen;
  }
  return st;
}

static int check_params(const pkcu_dec_params *prm) {
  const float *need[] = {prm->embed, prm->lstm0_b, prm->lstm1_b, prm->joint_enc_b,
                         prm->joint_pred_b, prm->joint_out_b};
  for (const float *q : need)
    if (!q) return pkcu_fail(PKCU_ERR_ARG, "pkcu_greedy_decode: NULL parameter");
  if (!PK_ALIGNED16(prm->embed) || !PK_ALIGNED16(prm->joint_enc_b) ||
      !PK_ALIGNED16(prm->joint_pred_b))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_greedy_decode: embed, joint_enc_b, joint_pred_b must be 16-byte aligned");
  return PKCU_OK;
}

// every evaluation emits or advances; at most 10 emissions per frame, then one
// more iteration for the last pending decoder step
static long long max_iterations(const pkcu_decoder *d) {
  int max_T = 0;
  for (int b = 0; b < d->B; b++) max_T = d->seq->lengths[b] > max_T ? d->seq->lengths[b] : max_T;
  return (long long)DEC_MAX_SYM * max_T + 2;
}

static int dec_start(pkcu_decoder *d, const pkcu_dec_params *prm, pkcu_gemm_hook hook,
                     void *hook_user, cudaStream_t s) {
  d->iterations = 0;
  dec_init_kernel<<<dec_grid((long long)d->B * DEC_H), 256, 0, s>>>(d->st, d->lstm, d->x0,
                                                                    prm->embed, d->B);
  int st = pkcu_launch_status("pkcu_greedy_decode: init");
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_DEC_ENC, s);
  return st;
}

// Replays the captured DEC_POLL-iteration graphs on d->gs until no utterance
// is live, joined to the caller's stream on both sides. The host keeps one
// batch ahead: batch k + 1 is launched before batch k's live count is read, so
// the GPU never waits for the host's check. When batch k's count is zero the
// batch already launched after it does nothing (finished rows are skipped by
// every kernel); the iterations reported end with batch k, as without it.
static int dec_replay(pkcu_decoder *d, const pkcu_dec_params *prm, pkcu_gemm_hook hook,
                      void *hook_user, int fused, cudaStream_t s) {
  int st = PKCU_OK;
  if (!d->graph[0] || !d->graph[1] || !same_params(d->gp, *prm) || d->ghook != hook ||
      d->guser != hook_user || d->gfused != fused || (fused && d->gwgen != d->wgen))
    st = dec_capture(d, prm, hook, hook_user, fused);
  if (st) return st;
  if (cudaEventRecord(d->ev_in, s) != cudaSuccess || cudaStreamWaitEvent(d->gs, d->ev_in, 0) != cudaSuccess)
    return pkcu_launch_status("pkcu_greedy_decode: join");
  const long long max_iters = max_iterations(d);
  if (cudaGraphLaunch(d->graph[0], d->gs) != cudaSuccess || cudaEventRecord(d->ev_done[0], d->gs) != cudaSuccess)
    return pkcu_launch_status("pkcu_greedy_decode: graph");
  for (long long k = 0;; k++) {
    const int cur = (int)(k & 1), next = cur ^ 1;
    if ((k + 1) * DEC_POLL < max_iters &&
        (cudaGraphLaunch(d->graph[next], d->gs) != cudaSuccess ||
         cudaEventRecord(d->ev_done[next], d->gs) != cudaSuccess))
      return pkcu_launch_status("pkcu_greedy_decode: graph");
    if (cudaEventSynchronize(d->ev_done[cur]) != cudaSuccess) return pkcu_launch_status("pkcu_greedy_decode: graph");
    d->iterations = (int)((k + 1) * DEC_POLL);
    if (d->live_host[cur] == 0 || (k + 1) * DEC_POLL >= max_iters) break;
  }
  if (cudaEventRecord(d->ev_out, d->gs) != cudaSuccess || cudaStreamWaitEvent(s, d->ev_out, 0) != cudaSuccess)
    return pkcu_launch_status("pkcu_greedy_decode: join");
  return PKCU_OK;
}

extern "C" int pkcu_greedy_decode_graph(pkcu_decoder *d, const pkcu_dec_params *prm,
                                        pkcu_gemm_hook hook, void *hook_user,
                                        pkcu_stream_t stream) {
  if (!d || !prm) return pkcu_fail(PKCU_ERR_ARG, "pkcu_greedy_decode_graph: NULL argument");
  int st = check_params(prm);
  if (!st) st = dec_start(d, prm, hook, hook_user, (cudaStream_t)stream);
  if (!st) st = dec_replay(d, prm, hook, hook_user, 0, (cudaStream_t)stream);
  return st;
}

extern "C" int pkcu_decoder_set_weights(pkcu_decoder *d, const pkcu_dec_weights *w, pkcu_stream_t stream) {
  if (!d || !w) return pkcu_fail(PKCU_ERR_ARG, "pkcu_decoder_set_weights: NULL argument");
  const float *m[] = {w->lstm0_wi, w->lstm0_wr, w->lstm1_wi, w->lstm1_wr, w->joint_pred, w->joint_out};
  for (const float *q : m)
    if (!q || !PK_ALIGNED16(q))
      return pkcu_fail(PKCU_ERR_ARG, "pkcu_decoder_set_weights: NULL or not 16-byte aligned weight");
  const size_t n = (size_t)DEC_H * DEC_H + (size_t)DEC_V * DEC_H;
  if (!d->jt && cudaMalloc((void **)&d->jt, sizeof(float) * n) != cudaSuccess) {
    cudaGetLastError();
    d->jt = nullptr;
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_decoder_set_weights: device allocation");
  }
  cudaStream_t s = (cudaStream_t)stream;
  const dim3 tb(32, 8);
  dec_transpose_kernel<<<dim3(DEC_H / 32, DEC_H / 32), tb, 0, s>>>(w->joint_pred, d->jt, DEC_H, DEC_H);
  dec_transpose_kernel<<<dim3((DEC_V + 31) / 32, DEC_H / 32), tb, 0, s>>>(w->joint_out, d->jt + DEC_H * DEC_H,
                                                                         DEC_H, DEC_V);
  const int st = pkcu_launch_status("pkcu_decoder_set_weights");
  if (st) return st;
  for (int i = 0; i < 4; i++) d->lw[i] = m[i];
  d->wgen += 1;
  return PKCU_OK;
}

extern "C" int pkcu_greedy_decode_fused(pkcu_decoder *d, const pkcu_dec_params *prm, pkcu_stream_t stream) {
  if (!d || !prm) return pkcu_fail(PKCU_ERR_ARG, "pkcu_greedy_decode_fused: NULL argument");
  if (!d->wgen) return pkcu_fail(PKCU_ERR_ARG, "pkcu_greedy_decode_fused: no weights (pkcu_decoder_set_weights)");
  int st = check_params(prm);
  if (!st) st = dec_start(d, prm, nullptr, nullptr, (cudaStream_t)stream);
  if (!st) st = dec_replay(d, prm, nullptr, nullptr, 1, (cudaStream_t)stream);
  return st;
}

extern "C" int pkcu_greedy_decode(pkcu_decoder *d, const pkcu_dec_params *prm, pkcu_gemm_hook hook,
                                  void *hook_user, pkcu_stream_t stream) {
  if (!d || !prm) return pkcu_fail(PKCU_ERR_ARG, "pkcu_greedy_decode: NULL argument");
  cudaStream_t s = (cudaStream_t)stream;
  int st = check_params(prm);
  if (!st) st = dec_start(d, prm, hook, hook_user, s);
  if (st) return st;
  if (!hook) return dec_replay(d, prm, nullptr, nullptr, 0, s);
  const long long max_iters = max_iterations(d);
  for (long long it = 0; it < max_iters; it++) {
    st = dec_iteration(d, prm, hook, hook_user, s);
    if (st) return st;
    d->iterations = (int)(it + 1);
    if ((it + 1) % DEC_POLL == 0 || it + 1 == max_iters) {
      if (cudaMemcpyAsync(d->live_host, d->st.live, sizeof(int), cudaMemcpyDeviceToHost, s) !=
              cudaSuccess ||
          cudaStreamSynchronize(s) != cudaSuccess)
        return pkcu_launch_status("pkcu_greedy_decode: poll");
      if (*d->live_host == 0) break;
    }
  }
  return PKCU_OK;
}

extern "C" int pkcu_decoder_results(const pkcu_decoder *d, int *n_tokens, int *evals, int *tokens,
                                    pkcu_stream_t stream) {
  if (!d) return pkcu_fail(PKCU_ERR_ARG, "pkcu_decoder_results: NULL decoder");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t B = (size_t)d->B;
  if ((n_tokens && cudaMemcpyAsync(n_tokens, d->st.ntok, sizeof(int) * B, cudaMemcpyDeviceToHost, s)) ||
      (evals && cudaMemcpyAsync(evals, d->st.evals, sizeof(int) * B, cudaMemcpyDeviceToHost, s)) ||
      (tokens && cudaMemcpyAsync(tokens, d->tokens, sizeof(int) * DEC_MAX_SYM * (size_t)d->F,
                                 cudaMemcpyDeviceToHost, s)) ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return pkcu_launch_status("pkcu_decoder_results");
  return PKCU_OK;
}
