/* geode_host.h - the C++ host side of the CUDA verify backend (libgeode_host.so), as a C ABI.
 *
 * It reads a geode-pack (geode.json and its data files, engine/src/pack.cpp), moves every tensor into the CUDA
 * backend (libgeode_cuda.so, loaded at run time beside this library) and drives the engine's speculation loop around
 * it: verify a batch (the accepted token + the drafts), accept with the engine's sampler rule
 * (engine/src/geode.cpp:327-350, the Sampler's mt19937_64 stream), roll back the rejected rows. Mirrors the Model
 * seam engine/src/model.hpp:189-205 (verify_n, verify_keep, can_verify, spec_tokens).
 *
 * Conventions as engine/include/geode/geode.h: 0 = ok, else an error code, the message in err (err_len > 0).
 * One ghost_model is driven by one thread at a time.
 */
#ifndef GEODE_HOST_H
#define GEODE_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    GHOST_OK = 0,
    GHOST_E_ARG = 1,      /* a bad argument (as GEODE_E_ARG) */
    GHOST_E_IO = 2,       /* the pack is missing or unreadable (as GEODE_E_IO) */
    GHOST_E_BACKEND = 7,  /* the CUDA backend failed or is absent (no CPU fallback) */
};

typedef struct ghost_model ghost_model;

typedef struct {
    float temperature;   /* 0 = greedy */
    float top_p;         /* 1 = off */
    int32_t top_k;       /* 0 = off */
    uint64_t seed;       /* the sampler's mt19937_64 seed (set once per generation, as geode_generate) */
} ghost_sampling;

/* Opens the pack in dir on CUDA device `device` with `context` positions of KV cache (0 = 4096) and verify batches
 * of up to max_tokens rows (<= 8). */
int ghost_open(const char *dir, int32_t device, int32_t context, int32_t max_tokens, ghost_model **out, char *err,
               size_t err_len);
void ghost_close(ghost_model *m);
/* Model::spec_tokens: the drafts a batch can carry (max_tokens - 1); Model::position */
int32_t ghost_spec_tokens(ghost_model *m);
int32_t ghost_position(ghost_model *m);
/* Model::verify_n: n tokens through every layer at the next positions; logits [n][vocab] (NULL: not wanted) */
int ghost_verify(ghost_model *m, const int32_t *toks, int32_t n, float *logits, char *err, size_t err_len);
/* Model::verify_keep: keep the first `kept` rows of the last batch (1 <= kept < n; with every row kept, no call) */
int ghost_keep(ghost_model *m, int32_t kept, char *err, size_t err_len);
/* The sampling of the steps that follow; seeds the sampler's stream */
int ghost_set_sampling(ghost_model *m, const ghost_sampling *s);
/* One speculation step: verify batch[0..n) (the accepted token, then n - 1 drafts), accept (kept = 1 + the drafts
 * that stood; next = the first sample that is no draft, -1 when a stop token stood), roll back to kept rows. */
int ghost_step(ghost_model *m, const int32_t *batch, int32_t n, const int32_t *stops, int32_t n_stops, int32_t *kept,
               int32_t *next, char *err, size_t err_len);
/* The pack's manifest as this host reads it, one line (arch, layers, hidden, vocab, experts, tensors, bytes); no GPU
 * needed. */
int ghost_pack_summary(const char *dir, char *out, size_t out_len, char *err, size_t err_len);

#ifdef __cplusplus
}
#endif
#endif
