/*  ref_full_harness.c -- TEST INFRASTRUCTURE ONLY (checker, never shipped).
 *
 *  One entry point into the reference engine built whole, with nothing
 *  redirected (oracle/_ref/libpkref_full.so: csrc/encoder.c, decoder.c,
 *  weights.c, tensor_ops.c, blas.c, threadpool.c with the reference's flags):
 *  load a weights.bin / weights.json checkpoint with pk_load_weights, encode a
 *  mel spectrogram with pk_encoder (pre-encode, 24 conformer blocks, its own
 *  GEMMs) and decode it with pk_greedy_decode -- the reference's transcription
 *  path minus audio I/O, the mel front end and the tokenizer. It is the
 *  end-to-end checker of the GPU pipeline run on the same checkpoint.
 */
#include <stdlib.h>
#include <string.h>

#include "parakeet.h"

/* mel [128, n_frames]. Writes the encoder output [T', 1024] (up to enc_cap
 * floats) and up to tok_cap tokens; *n_tokens = number emitted. Returns T', or
 * -1 if the checkpoint does not load. */
int pkref_transcribe(const char *bin_path, const char *json_path, const float *mel, int n_frames,
                     float *enc_out, long long enc_cap, int *tokens, int tok_cap, int *n_tokens)
{
    pk_verbose = 0;
    PkModel *m = (PkModel *)calloc(1, sizeof(PkModel));
    if (!m) return -1;
    if (pk_load_weights(m, bin_path, json_path) != 0) {
        free(m);
        return -1;
    }
    float *enc = NULL;
    int Tp = 0;
    pk_encoder(m, mel, n_frames, &enc, &Tp);
    const long long n = (long long)Tp * PK_D_MODEL;
    memcpy(enc_out, enc, sizeof(float) * (size_t)(n < enc_cap ? n : enc_cap));
    int *tok = NULL;
    const int nt = pk_greedy_decode(m, enc, Tp, &tok);
    for (int i = 0; i < nt && i < tok_cap; i++) tokens[i] = tok[i];
    *n_tokens = nt;
    free(tok);
    free(enc);
    pk_free_weights(m);
    free(m);
    return Tp;
}

/* For timing the reference encoder alone: load once, encode many times. */
static PkModel *g_model;

int pkref_model_load(const char *bin_path, const char *json_path)
{
    pk_verbose = 0;
    if (g_model) return -1;
    g_model = (PkModel *)calloc(1, sizeof(PkModel));
    if (!g_model) return -1;
    if (pk_load_weights(g_model, bin_path, json_path) != 0) {
        free(g_model);
        g_model = NULL;
        return -1;
    }
    return 0;
}

/* pk_encoder on mel [128, n_frames] with the loaded model; returns T'. */
int pkref_model_encode(const float *mel, int n_frames, float *enc_out, long long enc_cap)
{
    if (!g_model) return -1;
    float *enc = NULL;
    int Tp = 0;
    pk_encoder(g_model, mel, n_frames, &enc, &Tp);
    const long long n = (long long)Tp * PK_D_MODEL;
    if (enc_out) memcpy(enc_out, enc, sizeof(float) * (size_t)(n < enc_cap ? n : enc_cap));
    free(enc);
    return Tp;
}

void pkref_model_free(void)
{
    if (!g_model) return;
    pk_free_weights(g_model);
    free(g_model);
    g_model = NULL;
}

/* pk_encoder + pk_greedy_decode on mel [128, n_frames] with the loaded model
 * (pkref_model_load); returns the number of tokens, or -1. */
int pkref_model_transcribe(const float *mel, int n_frames, int *tokens, int tok_cap)
{
    if (!g_model) return -1;
    float *enc = NULL;
    int Tp = 0;
    pk_encoder(g_model, mel, n_frames, &enc, &Tp);
    int *tok = NULL;
    const int nt = pk_greedy_decode(g_model, enc, Tp, &tok);
    for (int i = 0; i < nt && i < tok_cap; i++) tokens[i] = tok[i];
    free(tok);
    free(enc);
    return nt;
}

/* pk_greedy_decode (its own sgemv products) on encoder output enc [T, 1024]
 * with the loaded model; returns the number of tokens, or -1. */
int pkref_model_decode(const float *enc, int T, int *tokens, int tok_cap)
{
    if (!g_model) return -1;
    int *tok = NULL;
    const int nt = pk_greedy_decode(g_model, enc, T, &tok);
    for (int i = 0; i < nt && i < tok_cap; i++) tokens[i] = tok[i];
    free(tok);
    return nt;
}
