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
    GHOST_E_IO = 2,       /* a file is missing, unreadable or the wrong size (as GEODE_E_IO) */
    GHOST_E_FORMAT = 3,   /* another model's, format's or version's file, or a damaged one (as GEODE_E_FORMAT) */
    GHOST_E_BACKEND = 7,  /* the CUDA backend failed or is absent (no CPU fallback) */
};

typedef struct ghost_model ghost_model;

typedef struct {
    float temperature;        /* 0 = greedy */
    float top_p;              /* 1 = off */
    int32_t top_k;            /* 0 = off */
    uint64_t seed;            /* the sampler's mt19937_64 seed (set once per generation, as geode_generate) */
    float presence_penalty;   /* 0 = off: subtracted from the logits of the answer's tokens so far before each row is
                                 sampled (engine/src/geode.cpp:234-255) */
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
/* Model::draft / draft_next (engine/src/model.cpp:1295-1480) on the device's MTP layer (packs with mtp.*; else
 * GHOST_E_BACKEND): the MTP pass over positions pos .. pos+n-1 - toks the tokens after them, hidden n rows of hidden
 * floats or NULL for the last verified batch's rows - the greedy draft from the last position, prob (NULL: not wanted)
 * its softmax probability; ghost_draft_next: one chained position pos from the last pass's own output row and tok. The
 * engine's loop: after a step that kept k rows of a batch at P, ghost_draft(the k tokens after P .. P+k-1, k, P, NULL)
 * drafts the next batch's first draft, ghost_draft_next chains the rest while the probability stays high. */
int ghost_draft(ghost_model *m, const int32_t *toks, int32_t n, int32_t pos, const float *hidden, int32_t *draft,
                float *prob, char *err, size_t err_len);
int ghost_draft_next(ghost_model *m, int32_t tok, int32_t pos, int32_t *draft, float *prob, char *err, size_t err_len);
/* geode_reset (engine/include/geode/geode.h:216): the conversation empty - position 0, zero states, no pending token, a
 * new conversation (an append of a later save goes to a new file). */
int ghost_reset(ghost_model *m, char *err, size_t err_len);
/* geode_prefill (engine/include/geode/geode.h:166-169): the prompt's n tokens appended to the conversation, nothing
 * generated. It runs through the verify step, max_tokens positions a launch (correct at any length; not a tensor-core
 * prefill). With an MTP layer the layer runs over the prompt's positions too, as the engine's prompt does
 * (engine/src/geode.cpp:132-150), all but the last, whose row the device keeps for the first draft:
 * ghost_draft(m, &pending, 1, position - 1, NULL, ...). A token id out of range or a prompt past the context:
 * GHOST_E_ARG, the conversation then holds the batches before the failing one. */
int ghost_prefill(ghost_model *m, const int32_t *prompt, int32_t n, char *err, size_t err_len);
/* Model::verify_keep: keep the first `kept` rows of the last batch (1 <= kept < n; with every row kept, no call) */
int ghost_keep(ghost_model *m, int32_t kept, char *err, size_t err_len);
/* The sampling of the steps that follow - a new answer, as a geode_generate call: seeds the sampler's stream and
 * empties the answer's tokens for the presence penalty */
int ghost_set_sampling(ghost_model *m, const ghost_sampling *s);
/* One speculation step: verify batch[0..n) (the accepted token, then n - 1 drafts), accept (kept = 1 + the drafts
 * that stood; next = the first sample that is no draft, -1 when a stop token stood), roll back to kept rows. With a
 * presence penalty, batch[0] (the answer's last sampled token) and every row sampled join the answer's tokens. */
int ghost_step(ghost_model *m, const int32_t *batch, int32_t n, const int32_t *stops, int32_t n_stops, int32_t *kept,
               int32_t *next, char *err, size_t err_len);
/* The pack's manifest as this host reads it, one line (arch, layers, hidden, vocab, experts, tensors, bytes); no GPU
 * needed. */
int ghost_pack_summary(const char *dir, char *out, size_t out_len, char *err, size_t err_len);

/* ------------------------------------------------------------------------------------ the conversation on disk ----
 * geode_state_save / geode_state_load (engine/include/geode/geode.h:171-191) for this host, in the engine's own state
 * file (engine/src/state.cpp): a state saved by the reference engine - its CPU or its GPU path - continues here, and
 * one saved here continues there. Between steps only. The file holds the KV rows of every attention layer, the Gated
 * DeltaNet conv and recurrent states and the token passed on but not computed yet (ghost_pending).
 * ghost_state_save: append = the file holds an earlier state of this conversation - only what changed is written, its
 * header last; otherwise it is written whole to path.tmp, then renamed over path. ghost_state_load: the saved
 * conversation replaces this one; GHOST_E_FORMAT for another model's / format's / version's or a damaged file,
 * GHOST_E_ARG when it is longer than this model's context, GHOST_E_IO when unreadable or cut short; on failure the
 * conversation is empty. A pack with an MTP layer keeps that layer's KV rows and the last hidden row in the file (a
 * load gives the row back to the device, so the next draft can take it); packs with a vision encoder: GHOST_E_ARG
 * (save) / GHOST_E_FORMAT (load).
 * out_position (may be NULL): the conversation's length in tokens. */
int ghost_state_save(ghost_model *m, const char *path, int32_t append, int32_t *out_position, char *err,
                     size_t err_len);
int ghost_state_load(ghost_model *m, const char *path, int32_t *out_position, char *err, size_t err_len);
/* The token passed on but not computed yet: the last ghost_step's next, or a loaded state's (-1: none) - the
 * engine's `pending` (engine/src/geode.cpp:490-519, the `extra` its state file carries). */
int32_t ghost_pending(ghost_model *m);

/* The state file alone, with host buffers (no GPU): what ghost_state_save / ghost_state_load write and read. Shapes:
 * n_attn attention layers (with the MTP layer's slot, after them, when the pack has one), kv_heads, kv_row =
 * kv_heads x head_dim, hidden, n_layers, conv_n and gdn_n floats of the Gated DeltaNet conv and recurrent states, mtp
 * 1 when the pack has an MTP layer. Buffers in the layouts of gcuda_state_get / gcuda_state_put: conv, gdn the
 * engine's own; kv [n_attn][2][position][kv_row] int8, kv_scale [n_attn][2][position][kv_heads] f32; hidden the last
 * position's row after the final norm (the engine keeps it with an MTP layer; write: NULL for none, read: has_hidden
 * says whether the file holds one). */
typedef struct {
    uint32_t n_attn, kv_heads, kv_row, hidden, n_layers;
    uint64_t conv_n, gdn_n;
    uint32_t mtp;
} ghost_state_shapes;
/* The fingerprint a state of this pack (geode.json in pack_dir) and these shapes carries (Model::fingerprint). */
uint64_t ghost_state_fingerprint(const char *pack_dir, const ghost_state_shapes *s);
int ghost_state_write(const char *path, uint64_t fingerprint, const ghost_state_shapes *s, int32_t position,
                      int32_t extra, uint64_t conv_id, const float *conv, const float *gdn, const int8_t *kv,
                      const float *kv_scale, const float *hidden, int32_t append, char *err, size_t err_len);
/* The header, checked against the fingerprint, the shapes and context (position < context): position, extra and
 * conversation id out, to size the buffers of ghost_state_read. */
int ghost_state_peek(const char *path, uint64_t fingerprint, const ghost_state_shapes *s, int32_t context,
                     int32_t *position, int32_t *extra, uint64_t *conv_id, char *err, size_t err_len);
int ghost_state_read(const char *path, uint64_t fingerprint, const ghost_state_shapes *s, int32_t context, float *conv,
                     float *gdn, int8_t *kv, float *kv_scale, float *hidden, int32_t *has_hidden, char *err,
                     size_t err_len);

#ifdef __cplusplus
}
#endif
#endif
