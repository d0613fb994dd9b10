// k_chunk.cu -- long audio: the chunked encoder's split and stitch.
//
// The reference encodes an utterance of more than PK_CHUNK_THRESHOLD (500)
// encoder frames in chunks (csrc/encoder.c:514-575, chosen by should_chunk
// :597-610): chunk c owns output frames [400c, min(400c + 400, T)) and runs
// the 24 blocks over its input frames, the owned ones plus up to 8 frames of
// overlap each side, clipped to [0, T), with the positional encoding of its
// own input length; the owned centre is copied back. The positional slice
// depends only on the length, so every chunk is exactly an utterance of that
// many frames, and here the chunks of all utterances (and the utterances
// that are not chunked, as one item each) form one ragged batch
// (pkcu_chunk_plan_seq) that a single pass of the blocks processes.
//
// Split and stitch are the same row gather, dst[r, :] = src[idx[r], :], over
// rows of 1024 floats with a device index array built once per plan: split
// maps each chunk-batch row to its utterance frame, stitch maps each
// utterance frame to the chunk-batch row of the chunk that owns it.
#include <cstdlib>
#include <cstring>

#include "pk_common.cuh"

struct pkcu_chunk_plan {
  pkcu_seq *seq;         // the chunk batch
  int n_utts, n_items, n_chunked;
  long long frames_in;   // utterance frames (sum of T)
  long long frames_ch;   // chunk-batch frames (with overlaps)
  int *idx;              // device: [frames_ch] split sources, then [frames_in] stitch sources
  int *item_utt;         // host: [n_items] utterance of each chunk item
  int *item_start;       // host: [n_items] first input frame of each chunk item
};

namespace {

// Warp per row of D floats (D a multiple of 128): lane moves D/128 float4.
__global__ void __launch_bounds__(256) row_gather_kernel(float4 *__restrict__ dst,
                                                         const float4 *__restrict__ src,
                                                         const int *__restrict__ idx,
                                                         long long n_rows, int d4) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const int lane = threadIdx.x & 31;
  const float4 *s = src + (long long)__ldg(idx + row) * d4;
  float4 *d = dst + row * d4;
  for (int c = lane; c < d4; c += 32) d[c] = __ldg(s + c);
}

int gather(float *dst, const float *src, const int *idx, long long n_rows, cudaStream_t s,
           const char *what) {
  if (n_rows == 0) return PKCU_OK;
  const long long blocks = (n_rows + 7) / 8;
  row_gather_kernel<<<(unsigned)blocks, 256, 0, s>>>(reinterpret_cast<float4 *>(dst),
                                                     reinterpret_cast<const float4 *>(src), idx,
                                                     n_rows, PK_D / 4);
  return pkcu_launch_status(what);
}

}  // namespace

extern "C" int pkcu_should_chunk(int frames, int mode) {
  if (mode == PKCU_CHUNK_OFF) return 0;
  if (mode == PKCU_CHUNK_ON) return 1;
  // PKCU_CHUNK_AUTO: the reference's rule, including its PK_CHUNK override
  const char *env = getenv("PK_CHUNK");
  if (env) {
    if (env[0] == '0' || strcmp(env, "off") == 0) return 0;
    if (env[0] == '1' || strcmp(env, "on") == 0) return 1;
  }
  return frames > PKCU_CHUNK_THRESHOLD;
}

extern "C" void pkcu_chunk_plan_destroy(pkcu_chunk_plan *p) {
  if (!p) return;
  pkcu_seq_destroy(p->seq);
  if (p->idx) cudaFree(p->idx);
  free(p->item_utt);
  free(p->item_start);
  free(p);
}

extern "C" int pkcu_chunk_bounds(int frames, int mode, int cap, int *in_start, int *in_len,
                                 int *out_start, int *out_len) {
  if (frames <= 0) return -1;
  const int chunk = pkcu_should_chunk(frames, mode);
  const int C = chunk ? PKCU_CHUNK_SIZE : frames, ov = chunk ? PKCU_CHUNK_OVERLAP : 0;
  const int n = (frames + C - 1) / C;
  if (!in_start && !in_len && !out_start && !out_len) return n;
  if (n > cap) return -1;
  for (int c = 0; c < n; c++) {   // encode_blocks_chunked's bounds (csrc/encoder.c:531-541)
    const int o0 = c * C, o1 = o0 + C < frames ? o0 + C : frames;
    const int i0 = o0 - ov > 0 ? o0 - ov : 0, i1 = o1 + ov < frames ? o1 + ov : frames;
    if (in_start) in_start[c] = i0;
    if (in_len) in_len[c] = i1 - i0;
    if (out_start) out_start[c] = o0;
    if (out_len) out_len[c] = o1 - o0;
  }
  return n;
}

extern "C" int pkcu_chunk_plan_create(const int *frames, int n_utts, int mode, pkcu_chunk_plan **out) {
  if (!out) return pkcu_fail(PKCU_ERR_ARG, "pkcu_chunk_plan_create: NULL out");
  *out = nullptr;
  if (!frames || n_utts <= 0) return pkcu_fail(PKCU_ERR_ARG, "pkcu_chunk_plan_create: no utterances");
  if (mode != PKCU_CHUNK_AUTO && mode != PKCU_CHUNK_OFF && mode != PKCU_CHUNK_ON)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_chunk_plan_create: unknown mode %d", mode);
  // the decisions once per utterance (AUTO reads PK_CHUNK: one reading for the whole plan)
  int *nch = (int *)malloc(sizeof(int) * (size_t)n_utts);
  if (!nch) return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_chunk_plan_create: host allocation");
  long long n_items = 0, frames_in = 0;
  int n_chunked = 0, max_n = 1;
  for (int u = 0; u < n_utts; u++) {
    const int T = frames[u];
    if (T <= 0 || T > (1 << 20)) {
      free(nch);
      return pkcu_fail(PKCU_ERR_ARG, "pkcu_chunk_plan_create: utterance %d has %d frames", u, T);
    }
    const int m = pkcu_should_chunk(T, mode) ? PKCU_CHUNK_ON : PKCU_CHUNK_OFF;
    nch[u] = m;
    n_chunked += m == PKCU_CHUNK_ON;
    const int n = pkcu_chunk_bounds(T, m, 0, nullptr, nullptr, nullptr, nullptr);
    if (n > max_n) max_n = n;
    n_items += n;
    frames_in += T;
  }
  pkcu_chunk_plan *p = (pkcu_chunk_plan *)calloc(1, sizeof(*p));
  int *len = (int *)malloc(sizeof(int) * (size_t)n_items);
  int *bnd = (int *)malloc(sizeof(int) * 4 * (size_t)max_n);
  if (p) {
    p->item_utt = (int *)malloc(sizeof(int) * (size_t)n_items);
    p->item_start = (int *)malloc(sizeof(int) * (size_t)n_items);
  }
  if (!p || !len || !bnd || !p->item_utt || !p->item_start) {
    free(nch);
    free(len);
    free(bnd);
    pkcu_chunk_plan_destroy(p);
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_chunk_plan_create: host allocation");
  }
  long long frames_ch = 0, item = 0;
  for (int u = 0; u < n_utts; u++) {
    const int n = pkcu_chunk_bounds(frames[u], nch[u], max_n, bnd, bnd + max_n, nullptr, nullptr);
    for (int c = 0; c < n; c++, item++) {
      len[item] = bnd[max_n + c];
      p->item_utt[item] = u;
      p->item_start[item] = bnd[c];
      frames_ch += bnd[max_n + c];
    }
  }
  int *hidx = (int *)malloc(sizeof(int) * (size_t)(frames_ch + frames_in));
  if (!hidx) {
    free(nch);
    free(len);
    free(bnd);
    pkcu_chunk_plan_destroy(p);
    return pkcu_fail(PKCU_ERR_NOMEM, "pkcu_chunk_plan_create: host allocation");
  }
  p->n_utts = n_utts;
  p->n_items = (int)n_items;
  p->n_chunked = n_chunked;
  p->frames_in = frames_in;
  p->frames_ch = frames_ch;
  // split: chunk-batch row -> utterance frame; stitch: utterance frame -> the
  // chunk-batch row of the chunk that owns it
  int *split = hidx, *stitch = hidx + frames_ch;
  long long row = 0, ubase = 0;
  for (int u = 0; u < n_utts; u++) {
    const int n = pkcu_chunk_bounds(frames[u], nch[u], max_n, bnd, bnd + max_n, bnd + 2 * max_n,
                                    bnd + 3 * max_n);
    for (int c = 0; c < n; c++) {
      const int i0 = bnd[c], il = bnd[max_n + c], o0 = bnd[2 * max_n + c], ol = bnd[3 * max_n + c];
      for (int t = 0; t < il; t++) split[row + t] = (int)(ubase + i0 + t);
      for (int t = 0; t < ol; t++) stitch[ubase + o0 + t] = (int)(row + o0 - i0 + t);
      row += il;
    }
    ubase += frames[u];
  }
  free(nch);
  free(bnd);
  int st = pkcu_seq_create(len, (int)n_items, &p->seq);
  free(len);
  if (!st && cudaMalloc((void **)&p->idx, sizeof(int) * (size_t)(frames_ch + frames_in)) != cudaSuccess) {
    cudaGetLastError();
    p->idx = nullptr;
    st = pkcu_fail(PKCU_ERR_NOMEM, "pkcu_chunk_plan_create: index arrays");
  }
  if (!st && cudaMemcpy(p->idx, hidx, sizeof(int) * (size_t)(frames_ch + frames_in),
                        cudaMemcpyHostToDevice) != cudaSuccess)
    st = pkcu_fail(PKCU_ERR_CUDA, "pkcu_chunk_plan_create: %s", cudaGetErrorString(cudaGetLastError()));
  free(hidx);
  if (st) {
    pkcu_chunk_plan_destroy(p);
    return st;
  }
  *out = p;
  return PKCU_OK;
}

extern "C" const pkcu_seq *pkcu_chunk_plan_seq(const pkcu_chunk_plan *p) { return p ? p->seq : nullptr; }
extern "C" int pkcu_chunk_plan_chunked(const pkcu_chunk_plan *p) { return p ? p->n_chunked : 0; }
extern "C" int pkcu_chunk_plan_items(const pkcu_chunk_plan *p) { return p ? p->n_items : 0; }

extern "C" int pkcu_chunk_plan_item(const pkcu_chunk_plan *p, int item, int *utt, int *first_frame,
                                    int *frames) {
  if (!p || item < 0 || item >= p->n_items)
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_chunk_plan_item: bad item %d", item);
  if (utt) *utt = p->item_utt[item];
  if (first_frame) *first_frame = p->item_start[item];
  if (frames) *frames = p->seq->lengths[item];
  return PKCU_OK;
}

extern "C" int pkcu_chunk_split(const pkcu_chunk_plan *p, const float *x, float *xc, pkcu_stream_t stream) {
  if (!p || !x || !xc) return pkcu_fail(PKCU_ERR_ARG, "pkcu_chunk_split: NULL argument");
  if (!PK_ALIGNED16(x) || !PK_ALIGNED16(xc))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_chunk_split: arrays must be 16-byte aligned");
  return gather(xc, x, p->idx, p->frames_ch, (cudaStream_t)stream, "pkcu_chunk_split");
}

extern "C" int pkcu_chunk_stitch(const pkcu_chunk_plan *p, const float *xc, float *x, pkcu_stream_t stream) {
  if (!p || !x || !xc) return pkcu_fail(PKCU_ERR_ARG, "pkcu_chunk_stitch: NULL argument");
  if (!PK_ALIGNED16(x) || !PK_ALIGNED16(xc))
    return pkcu_fail(PKCU_ERR_ARG, "pkcu_chunk_stitch: arrays must be 16-byte aligned");
  return gather(x, xc, p->idx + p->frames_ch, p->frames_in, (cudaStream_t)stream, "pkcu_chunk_stitch");
}
