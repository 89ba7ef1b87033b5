/* geode_oracle.h - TEST INFRASTRUCTURE: a plain-C restatement of the reference engine's CPU verify path
 * (sergqwer/geode, engine/src/model.cpp forward_batch / gdn / attention / attend / moe / route_topk, the int8
 * kernels of engine/src/kernels.cpp, the sampler of engine/src/sampler.cpp and the acceptance rule of
 * engine/src/geode.cpp:327-350). It is the checker the parity tests compare the CUDA path with; it is never the
 * product path and the CUDA library never links it. Every function cites the reference lines it restates.
 *
 * Pinned against the reference itself: tests/test_oracle.py runs the reference's own code (oracle/_ref, compiled
 * from the reference sources) on the same inputs and requires bit-identical results, and the committed golden
 * fixtures in tests/golden/ were produced by that reference build (tests/golden/make_golden.py).
 */
#ifndef GEODE_ORACLE_H
#define GEODE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A q4 matrix in the pack's layout: each row = cols/2 code bytes, then cols/16 E4M3 scale bytes. */
typedef struct {
    const uint8_t *data;
    int64_t rows, cols;
    float global;
} go_q4;

typedef struct {
    int hidden, n_layers, vocab;
    float eps;
    int n_heads, n_kv_heads, head_dim, rope_dim;
    float rope_theta;
    int gdn_k_heads, gdn_v_heads, gdn_k_dim, gdn_v_dim, conv_kernel;
    int n_experts, top_k, moe_ff, shared_ff;
    int dense;       /* arch qwen35: an ungated MLP (shared_ff wide), no router */
    int attn_block;  /* positions per softmax block (engine/src/model.hpp:458, 1024) */
} go_config;

typedef struct {
    int attn;
    const float *in_norm, *post_norm;
    /* Gated DeltaNet */
    go_q4 qkv, z, out;
    const uint16_t *a, *b;
    const float *A_log, *dt_bias, *conv, *gnorm;
    /* gated attention */
    go_q4 q, k, v, o;
    const float *q_norm, *k_norm;
    /* MLP: the dense model's gate/up/down, or the MoE's shared expert */
    go_q4 sh_gate, sh_up, sh_down;
    const uint16_t *router, *shared_gate;
    const uint8_t *experts;      /* expert e's block at experts + e * expert_stride: gate_up rows, then down rows */
    uint64_t expert_stride;
    const float *expert_scales;  /* [E][2]: the globals of gate_up and down */
} go_layer;

typedef struct {
    go_config cfg;
    const go_layer *layers;
    go_q4 embed, lm_head;
    const float *final_norm;
} go_model;

/* A conversation's state (the layouts of the reference's own buffers, engine/src/model.hpp:548-555):
 *   conv  [n_gdn][conv_dim][K-1]
 *   gdn   [n_gdn][nv][dv/16][dk][16]   (strip layout; dv % 16 == 0)
 *   kv    [n_attn][2][ctx][nkv*hd]     int8 (K then V)
 *   kvs   [n_attn][2][ctx][nkv]        f32 scales */
typedef struct {
    int pos, ctx;
    float *conv, *gdn;
    int8_t *kv;
    float *kvs;
} go_state;

/* Per-layer trace of the last go_forward (optional): rows [layer][token][hidden] and picks [layer][token][k]. */
typedef struct {
    float *x, *mixer, *moe, *out;
    int *ids;
    float *weights, *gate;
} go_trace;

/* n tokens at state->pos.. ; logits [n][vocab] (every token's, the verify pass) or NULL; hidden [n][H] (after the
 * final norm) or NULL. Returns 0, or -1 on a bad argument. */
int go_forward(const go_model *m, go_state *s, const int *toks, int n, float *logits, float *hidden,
               const go_trace *tr);

/* The MTP drafting layer (a pack with one: engine/src/model.cpp:175-191): fc [hidden][2 hidden] over
 * [norm(embedding of the next token) | norm(hidden state)], then a full-attention decoder layer (mtp.layers.0.) whose
 * MLP takes the routed experts after the main layers', then mtp.norm. */
typedef struct {
    go_layer layer;
    go_q4 fc;
    const float *norm, *pre_e, *pre_h;
} go_mtp;

/* Model::forward_mtp (engine/src/model.cpp:4965-5039): n positions from pos, position t taking hidden row t (the main
 * model's, after its final norm) and the embedding of next[t]; each attends to the MTP layer's own positions up to it,
 * whose KV (kv [2][ctx][nkv*hd] int8 K then V, kvs [2][ctx][nkv] f32 scales) it writes. logits [vocab] of the last
 * position (NULL: none) from lm_head; out_hidden [hidden] (NULL: not wanted): that position's output after mtp.norm.
 * Returns 0, or -1 on a bad argument. */
int go_forward_mtp(const go_model *m, const go_mtp *mtp, int8_t *kv, float *kvs, int ctx, const int *next,
                   const float *hidden, int n, int pos, float *logits, float *out_hidden);

/* ---- the kernels, exposed for kernel-level tests ---- */
float go_e4m3_value(uint8_t b);
void go_dequant_row(const go_q4 *w, int64_t r, float *out);
void go_quantize_activation(const float *x, int64_t cols, int8_t *q, float *scale, int32_t *bsum);
void go_matvec_q(const go_q4 *w, const int8_t *q, const float *scale, float *y, int64_t r0, int64_t r1);
void go_matvec_bf16(const uint16_t *w, int64_t rows, int64_t cols, int n, const float *xs, float *ys);
void go_rmsnorm(const float *x, const float *w, float *out, int n, float eps, int zero_centered);
float go_fast_exp(float x);
void go_route_topk(const float *logits, int E, int K, int *ids, float *weights);
void go_q4_block(const float *x, float s2, uint8_t *scale_byte, uint8_t codes[16]);
/* quantize a [rows][cols] f32 matrix into the pack's q4 layout with global s2 (out: rows * cols*9/16 bytes) */
void go_quantize_q4(const float *w, int64_t rows, int64_t cols, float s2, uint8_t *out, int threads);

/* ---- the sampler and acceptance rule ---- */
typedef struct {
    uint64_t mt[312];
    int mti;
} go_mt64;
void go_mt64_seed(go_mt64 *g, uint64_t seed);
uint64_t go_mt64_next(go_mt64 *g);
double go_canonical(go_mt64 *g);
/* engine/src/sampler.cpp:16-50 with an explicit uniform u in [0,1) (the draw the sampler would make) */
int go_sample(const float *logits, int n, float temperature, float top_p, int top_k, double u);
/* engine/src/geode.cpp:327-350: returns kept; *next the first non-draft sample (-1 if none); samples[n] */
int go_accept(const float *rows, int n, int V, const int *batch, float temperature, float top_p, int top_k,
              uint64_t seed, const int *stops, int n_stops, int *next, int *samples);
/* go_accept with geode_generate's presence penalty (engine/src/geode.cpp:234-255): seen in/out, room for n more */
int go_accept_seen(const float *rows, int n, int V, const int *batch, float temperature, float top_p, int top_k,
                   uint64_t seed, const int *stops, int n_stops, float penalty, int *seen, int *n_seen, int *next,
                   int *samples);

/* Standard speculative (rejection) sampling (Leviathan et al. 2023; Chen et al. 2023), with Philox4x32-10
 * uniforms. NOT in the reference: parity unpinned. target [n_drafts+1][V], draft [n_drafts][V] logits; the
 * temperature / top-k / top-p filter is applied to both. Returns accepted drafts; *next the resampled/bonus token. */
int go_spec_reject(const float *target, const float *draft, int n_drafts, int V, const int *drafts,
                   float temperature, float top_p, int top_k, uint64_t seed, uint64_t seq, int *next);
void go_philox4x32(uint64_t key, uint64_t counter_hi, uint64_t counter_lo, uint32_t out[4]);

/* The exp premise (test infrastructure): float bit patterns in [lo, hi) where glibc's expf(x) differs from
 * go_expf_restated(x) (restated = 1) or from (float)exp((double)x) (restated = 0) (go_expf_mismatch), or from a
 * device-computed table vals[n] for patterns lo.. (go_expf_check_table); NaNs equal; the first cap differing
 * patterns in first[]. */
float go_expf_restated(float x);
uint64_t go_expf_mismatch(uint64_t lo, uint64_t hi, int restated, int threads, uint32_t *first, int cap);
uint64_t go_expf_check_table(uint64_t lo, uint64_t n, const float *vals, int threads, uint32_t *first, int cap);

/* one routed pick of Model::moe (engine/src/model.cpp:4496-4543): y [H] from h [H] and the expert block */
void go_expert_pair(const uint8_t *blk, float g_gu, float g_dn, int H, int ff, const float *h, float *y);

#ifdef __cplusplus
}
#endif
#endif
