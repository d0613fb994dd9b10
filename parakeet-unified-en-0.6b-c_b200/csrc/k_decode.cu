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
#include "pk_common.cuh"

namespace pk {

constexpr int DEC_H = 640, DEC_V = 1025, DEC_BLANK = 1024, DEC_MAX_SYM = 10;
constexpr int DEC_H4 = DEC_H / 4;

struct DecState {      // one entry per utterance
  int *t, *s, *ntok, *last, *pending, *evals;
  int *live;           // rows still active or pending after the last select
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
  }
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

// Logits = joint.out product + bias, first-maximum argmax (strict '>' in index
// order, csrc/decoder.c:106-114; a NaN never wins, a NaN first logit keeps 0),
// then the greedy state machine of csrc/decoder.c:99-129 for one row.
__global__ void __launch_bounds__(32 * SEL_ROWS)
dec_select_kernel(const float *__restrict__ out, const float *__restrict__ out_b, DecState st,
                  int *__restrict__ tokens, const float *__restrict__ embed, float *__restrict__ x0,
                  SeqDev seq, int B) {
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * SEL_ROWS + (threadIdx.x >> 5);
  if (b >= B) return;
  const int T = seq_T(seq, b);
  const int tb = st.t[b];
  if (tb >= T) {                       // finished: its last decoder step (if any) has run
    if (lane == 0) st.pending[b] = 0;
    return;
  }
  const float *l = out + (long long)b * DEC_V;
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int v = lane; v < DEC_V; v += 32) {
    const float x = l[v] + __ldg(out_b + v);
    if (x > bv) { bv = x; bi = v; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(PK_FULL_MASK, bv, o);
    const int oi = __shfl_xor_sync(PK_FULL_MASK, bi, o);
    if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
  }
  const int best = (isnan(l[0] + __ldg(out_b)) || bi == INT_MAX) ? 0 : bi;
  if (best != DEC_BLANK) {             // the next decoder step's input (csrc/decoder.c:19)
    const float4 *src = reinterpret_cast<const float4 *>(embed + (long long)best * DEC_H);
    float4 *dst = reinterpret_cast<float4 *>(x0 + (long long)b * DEC_H);
    for (int j = lane; j < DEC_H4; j += 32) dst[j] = __ldg(src + j);
  }
  if (lane != 0) return;
  st.evals[b] += 1;
  int t = tb, s = st.s[b], pend = 0;
  if (best == DEC_BLANK) {
    t += 1;
    s = 0;
  } else {
    const int n = st.ntok[b];
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
  if (t < T || pend) atomicAdd(st.live, 1);
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
  float *x0, *hidden;      // [B, 640]
  float *encp, *pred, *out, *g0i, *g0r, *g1i, *g1r;
  int *tokens;             // [10 F]: utterance b's tokens from 10 * frame_off(b)
  int *live_host;          // page-locked poll target
  int iterations;          // of the last decode
  int device;
  // Without a hook, DEC_POLL iterations and the poll copy are one CUDA graph,
  // captured on `gs` for the parameter pointers in `gp` and replayed.
  cudaStream_t gs;
  cudaEvent_t ev_in, ev_out;
  cudaGraphExec_t graph;
  pkcu_dec_params gp;
};

extern "C" void pkcu_decoder_destroy(pkcu_decoder *d) {
  if (!d) return;
  if (d->graph) cudaGraphExecDestroy(d->graph);
  if (d->ev_in) cudaEventDestroy(d->ev_in);
  if (d->ev_out) cudaEventDestroy(d->ev_out);
  if (d->gs) cudaStreamDestroy(d->gs);
  if (d->block) cudaFree(d->block);
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
  const size_t sz_state = up(sizeof(int) * (6 * B + 1));
  const size_t sz_lstm = up(sizeof(float) * 4 * B * H), sz_bh = up(sizeof(float) * B * H);
  const size_t sz_enc = up(sizeof(float) * (size_t)F * H), sz_out = up(sizeof(float) * B * DEC_V);
  const size_t sz_g = up(sizeof(float) * B * 4 * H), sz_tok = up(sizeof(int) * DEC_MAX_SYM * (size_t)F);
  const size_t total = sz_state + sz_lstm + 3 * sz_bh + sz_enc + sz_out + 4 * sz_g + sz_tok;
  if (cudaMalloc(&d->block, total) != cudaSuccess) {
    cudaGetLastError();
    d->block = nullptr;
    pkcu_decoder_destroy(d);
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_decoder_create: device allocation of %zu bytes", total);
  }
  if (cudaMallocHost(&d->live_host, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    d->live_host = nullptr;
    pkcu_decoder_destroy(d);
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_decoder_create: page-locked host allocation");
  }
  char *p = (char *)d->block;
  int *si = (int *)p;
  d->st = DecState{si, si + B, si + 2 * B, si + 3 * B, si + 4 * B, si + 5 * B, si + 6 * B};
  p += sz_state;
  d->lstm = (float *)p; p += sz_lstm;
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
      d->out, prm->joint_out_b, d->st, d->tokens, prm->embed, d->x0, seq, B);
  return pkcu_launch_status("pkcu_greedy_decode: select");
}

static bool same_params(const pkcu_dec_params &a, const pkcu_dec_params &b) {
  return a.embed == b.embed && a.lstm0_b == b.lstm0_b && a.lstm1_b == b.lstm1_b &&
         a.joint_enc_b == b.joint_enc_b && a.joint_pred_b == b.joint_pred_b &&
         a.joint_out_b == b.joint_out_b;
}

// Captures DEC_POLL iterations + the copy of the live count into d->graph.
static int dec_capture(pkcu_decoder *d, const pkcu_dec_params *prm) {
  if (d->graph) {
    cudaGraphExecDestroy(d->graph);
    d->graph = nullptr;
  }
  if (!d->gs && (cudaStreamCreateWithFlags(&d->gs, cudaStreamNonBlocking) != cudaSuccess ||
                 cudaEventCreateWithFlags(&d->ev_in, cudaEventDisableTiming) != cudaSuccess ||
                 cudaEventCreateWithFlags(&d->ev_out, cudaEventDisableTiming) != cudaSuccess))
    return pkcu_launch_status("pkcu_greedy_decode: graph stream");
  if (cudaStreamBeginCapture(d->gs, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
    return pkcu_launch_status("pkcu_greedy_decode: begin capture");
  int st = PKCU_OK;
  for (int i = 0; i < DEC_POLL && !st; i++) st = dec_iteration(d, prm, nullptr, nullptr, d->gs);
  if (!st && cudaMemcpyAsync(d->live_host, d->st.live, sizeof(int), cudaMemcpyDeviceToHost, d->gs) !=
                 cudaSuccess)
    st = pkcu_launch_status("pkcu_greedy_decode: capture poll copy");
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(d->gs, &g);
  if (!st && ce != cudaSuccess) st = pkcu_launch_status("pkcu_greedy_decode: end capture");
  if (!st && cudaGraphInstantiate(&d->graph, g, 0) != cudaSuccess) {
    d->graph = nullptr;
    st = pkcu_launch_status("pkcu_greedy_decode: instantiate");
  }
  if (g) cudaGraphDestroy(g);
  if (!st) d->gp = *prm;
  return st;
}

extern "C" int pkcu_greedy_decode(pkcu_decoder *d, const pkcu_dec_params *prm, pkcu_gemm_hook hook,
                                  void *hook_user, pkcu_stream_t stream) {
  if (!d || !prm) return pkcu_fail(PKCU_ERR_ARG, "pkcu_greedy_decode: NULL argument");
  const float *need[] = {prm->embed, prm->lstm0_b, prm->lstm1_b, prm->joint_enc_b,
                         prm->joint_pred_b, prm->joint_out_b};
  for (const float *q : need)
    if (!q) return pkcu_fail(PKCU_ERR_ARG, "pkcu_greedy_decode: NULL parameter");
  if (!PK_ALIGNED16(prm->embed) || !PK_ALIGNED16(prm->joint_enc_b) ||
      !PK_ALIGNED16(prm->joint_pred_b))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_greedy_decode: embed, joint_enc_b, joint_pred_b must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const int B = d->B;
  const size_t BH = (size_t)B * DEC_H;
  int max_T = 0;
  for (int b = 0; b < B; b++) max_T = d->seq->lengths[b] > max_T ? d->seq->lengths[b] : max_T;
  // every evaluation emits or advances; at most 10 emissions per frame, then
  // one more iteration for the last pending decoder step
  const long long max_iters = (long long)DEC_MAX_SYM * max_T + 2;
  d->iterations = 0;
  dec_init_kernel<<<dec_grid((long long)BH), 256, 0, s>>>(d->st, d->lstm, d->x0, prm->embed, B);
  int st = pkcu_launch_status("pkcu_greedy_decode: init");
  if (!st && hook) st = hook(hook_user, -1, PKCU_GEMM_DEC_ENC, stream);
  if (st) return st;
  if (!hook) {
    if (!d->graph || !same_params(d->gp, *prm)) st = dec_capture(d, prm);
    if (st) return st;
    if (cudaEventRecord(d->ev_in, s) != cudaSuccess || cudaStreamWaitEvent(d->gs, d->ev_in, 0) != cudaSuccess)
      return pkcu_launch_status("pkcu_greedy_decode: join");
    for (long long it = 0; it < max_iters; it += DEC_POLL) {
      if (cudaGraphLaunch(d->graph, d->gs) != cudaSuccess || cudaStreamSynchronize(d->gs) != cudaSuccess)
        return pkcu_launch_status("pkcu_greedy_decode: graph");
      d->iterations += DEC_POLL;
      if (*d->live_host == 0) break;
    }
    if (cudaEventRecord(d->ev_out, d->gs) != cudaSuccess || cudaStreamWaitEvent(s, d->ev_out, 0) != cudaSuccess)
      return pkcu_launch_status("pkcu_greedy_decode: join");
    return PKCU_OK;
  }
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
