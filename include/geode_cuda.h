/* geode_cuda.h - libgeode_cuda.so: the CUDA (B200, sm_100a) backend of the engine's speculative-decoding verify
 * step, as a C ABI with no CUDA or torch type in it, so the engine can dlopen it beside its CPU, Adreno and Hexagon
 * backends exactly as it opens libgeode_npu.so (engine/src/model.cpp:2255-2320, npu/host/npu_api.h:12-40).
 *
 * Two layers:
 *   1. The backend (gcuda_*): an opaque handle that owns the model's weights in device memory (adopted from the
 *      pack's bytes), the conversation's device state (Gated DeltaNet conv / recurrent states, the int8 KV cache)
 *      and the verify step. It replaces the Adreno branch of Model::verify_n / verify_keep
 *      (engine/src/model.cpp:1529-1592, 1594-1634) and the acceptance of geode_generate
 *      (engine/src/geode.cpp:327-350).
 *   2. Operators (gcuda_op_*): the kernels one at a time on caller-owned device buffers (a CUDA stream passed as
 *      void *), the products Model::matmul / matmul_bf16 / quantize_activation / route_topk compute
 *      (engine/src/model.cpp:3336-3495, engine/src/kernels.cpp:1254-1322, engine/src/model.cpp:4021-4065).
 *
 * Conventions (as npu_api.h): 0 = ok, negative = an error; the message of the last error via gcuda_last_error.
 * A handle is driven by one thread at a time (engine/include/geode/geode.h:6-7); it runs on one device and one
 * CUDA stream of its own. Host buffers passed in are read or written before the call returns; adopted weights
 * are copied to the device (the caller's bytes are not kept).
 */
#ifndef GEODE_CUDA_H
#define GEODE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GCUDA_OK 0
#define GCUDA_E_ARG (-1)      /* a bad argument (shape, id, batch size, position) */
#define GCUDA_E_CUDA (-2)     /* a CUDA runtime error */
#define GCUDA_E_DEVICE (-3)   /* a kernel reported an error (a bounded wait that gave up, a bad token id) */
#define GCUDA_E_MEMORY (-4)   /* device memory exhausted */
#define GCUDA_E_STATE (-5)    /* a call out of order (verify before setup, keep without a verified batch) */

typedef struct gcuda gcuda;

/* ------------------------------------------------------------------------------------------- the backend ---- */

/* The model geometry (engine/src/pack.hpp:31-60 ModelConfig; dense = arch "qwen35"). */
typedef struct {
    int hidden, n_layers, vocab;
    float eps;
    int n_heads, n_kv_heads, head_dim, rope_dim;
    float rope_theta;
    int gdn_k_heads, gdn_v_heads, gdn_k_dim, gdn_v_dim, conv_kernel;
    int n_experts, top_k, moe_ff, shared_ff;
    int dense;
    int context;      /* KV positions to hold (Model's context_length, engine/src/model.hpp:295) */
    int max_tokens;   /* the largest verified batch (spec_tokens, engine/src/model.hpp:197), 2..8 */
} gcuda_shape;

/* One layer's tensors, as ids returned by the gcuda_adopt_* calls (-1 where the layer has none); the pack's names
 * (engine/src/model.cpp:94-156). */
typedef struct {
    int attn;
    int in_norm, post_norm;
    int qkv, z, out, a, b, A_log, dt_bias, conv, gnorm; /* linear_attn.* (Gated DeltaNet) */
    int q, k, v, o, q_norm, k_norm;                     /* self_attn.* (gated attention) */
    int sh_gate, sh_up, sh_down;                        /* mlp.shared_expert.* (or the dense mlp.*) */
    int router, shared_gate;                            /* mlp.gate, mlp.shared_expert_gate (bf16) */
    int experts;                                        /* gcuda_adopt_experts */
} gcuda_layer;

/* Opens device `device` (its own stream). NULL with the reason in err when CUDA or the device is unusable. */
gcuda *gcuda_open(int device, char *err, int err_len);
void gcuda_close(gcuda *g);
/* The last error's message (0 = none). */
int gcuda_last_error(gcuda *g, char *buf, int len);

/* A q4 matrix in the pack's layout (rows x cols; each row cols/2 code bytes, then cols/16 E4M3 scale bytes, level
 * 2c+1 for c < 8, -(2(c-8)+1) above), copied to the device in the GEMV's tile layout (the same bytes, permuted
 * within 16-row tiles). cols a multiple of 64. Its id (>= 0), or < 0. Mirrors gnpu_adopt_q4 (npu/host/npu_api.h:34). */
int gcuda_adopt_q4(gcuda *g, const uint8_t *data, int64_t rows, int64_t cols, size_t row_bytes, float global);
/* f32 or bf16 parameters (norm weights, conv taps, A_log, dt_bias, router / gate / a / b rows), copied as they are. */
int gcuda_adopt_raw(gcuda *g, const void *data, size_t bytes);
/* One layer's routed experts: n blocks of stride bytes (gate_up [2 ff][hidden] then down [hidden][ff], q4,
 * engine/src/pack.cpp:333-337) and their globals scales[n][2] (mlp.experts.scales). Its id, or < 0. */
int gcuda_adopt_experts(gcuda *g, const uint8_t *blocks, int n, size_t stride, const float *scales);
/* The model: the geometry, the layers, the embedding (q4), lm_head (q4) and norm.weight ids. Allocates the state
 * (context positions) and the scratch, and records the verify step as CUDA graphs. */
int gcuda_setup(gcuda *g, const gcuda_shape *shape, const gcuda_layer *layers, int embed, int lm_head, int final_norm);

/* Expert parallelism (no counterpart in the reference, which runs on one device): the MoE layers' routed experts
 * striped over `world` (<= 8) handles, one per GPU of one node (expert e on rank e % world); everything else computed
 * on every rank. In each MoE layer every rank stores the rows of the picks it owns into every peer's buffer over
 * NVLink (peer memory mapped through CUDA IPC at gcuda_setup; per-layer flags with bounded waits - a peer that never
 * arrives makes the step fail with GCUDA_E_DEVICE), and every rank combines in rank order: the logits equal the
 * one-GPU step's bit for bit. gcuda_ep_unique_id fills NCCL's 128-byte id on one rank, which the caller hands to
 * every rank; gcuda_set_ep (before gcuda_setup, same id, ranks 0..world-1, each its own device) joins the group, and
 * every rank must then reach gcuda_setup (it gathers the buffers' handles through NCCL) and run the same calls.
 * libnccl.so.2 is loaded on first use; world 1 needs none. */
int gcuda_ep_unique_id(void *id_out);
int gcuda_set_ep(gcuda *g, int rank, int world, const void *id);

/* Model::verify_n (engine/src/model.cpp:1483): n tokens (toks[0] the last accepted token, then the drafts) at the
 * next positions through every layer; logits [n][vocab] (host; NULL: left on the device) and hidden [n][hidden]
 * (the rows after the final norm, the MTP layer's input; NULL: not wanted). The position moves on by n. A token id
 * outside [0, vocab): GCUDA_E_ARG before anything runs, the conversation as it was (engine/src/model.cpp:1551-1555). */
int gcuda_verify(gcuda *g, const int *toks, int n, float *logits, float *hidden);
/* Model::verify_keep (engine/src/model.cpp:1594): keep the first `kept` (1 .. n-1) of the last verified batch - the
 * Gated DeltaNet states as after token kept-1, the position back by n - kept. Returns once the states' copies are
 * queued on the handle's stream (every later call is ordered behind them). */
int gcuda_keep(gcuda *g, int kept);
int gcuda_position(gcuda *g);

/* The MTP drafting layer (Model::forward_mtp, engine/src/model.cpp:4965-5039; the pack's mtp.* tensors,
 * engine/src/model.cpp:175-191): its fc [hidden][2 hidden] (q4), the norms mtp.pre_fc_norm_embedding / _hidden and
 * mtp.norm (f32), and its decoder layer (an attention layer with the model's MLP; routed experts by
 * gcuda_adopt_experts). Before gcuda_setup, which gives the layer its own KV cache of `context` positions. */
int gcuda_set_mtp(gcuda *g, int fc, int pre_e, int pre_h, int norm, const gcuda_layer *layer);
/* The draft head (engine/src/model.cpp:803-827, 2135-2161): the pack's draft_vocab.bin tokens ids[0..n) (int32, those
 * outside the vocabulary left out, then padded to whole tiles of 32 rows with copies of ids[0], as the engine's GPU
 * branch does - the copies never win the first maximum) and `head`, a q4 tensor of lm_head's rows of those ids in
 * that order (gcuda_adopt_q4, lm_head's global). The MTP pass then multiplies only these rows: its logits are n wide,
 * the draft is ids[their first maximum] and prob its softmax probability over the n (copies included). Before
 * gcuda_setup; n a multiple of 32. */
int gcuda_set_draft_head(gcuda *g, int head, const int *ids, int n);
/* The MTP pass's logits per row: n of gcuda_set_draft_head, else the vocabulary (after gcuda_setup). */
int gcuda_draft_rows(gcuda *g);
/* Model::draft (engine/src/model.cpp:1295-1446, its GPU branch): the MTP pass over the positions pos .. pos+n-1 of
 * its KV (n <= max_tokens), position i taking the embedding of toks[i] and hidden row i - hidden [n][hidden] on the
 * host, or NULL for the rows the device holds (the last verified batch's, the kept ones after gcuda_keep, or the row
 * of gcuda_put_last_hidden; n at most their count) - then
 * draft = the first maximum of the last position's logits and prob (NULL: not wanted) its softmax probability
 * (softmax_at, engine/src/model.cpp:1287-1292); logits (NULL: not wanted) gets those logits (gcuda_draft_rows of
 * them: the vocabulary's, or the draft head's rows'). */
int gcuda_draft(gcuda *g, const int *toks, int n, int pos, const float *hidden, int *draft, float *prob, float *logits);
/* Model::draft_next (engine/src/model.cpp:1448-1480): one chained MTP position `pos` from the last pass's output row
 * after mtp.norm and the embedding of tok (the draft just made). */
int gcuda_draft_next(gcuda *g, int tok, int pos, int *draft, float *prob, float *logits);
/* The conversation from the start (position 0, zero states; the device-side rejection sampler's random sequence
 * restarts too, so a repeated conversation with the same seed draws the same uniforms). */
int gcuda_reset(gcuda *g);

/* Sampling parameters (engine/src/sampler.hpp:11-15, and geode_sampling's presence_penalty,
 * engine/include/geode/geode.h). */
typedef struct {
    float temperature;      /* 0 = greedy */
    float top_p;            /* 1 = off */
    int top_k;              /* 0 = off (then 1024 candidates, engine/src/sampler.cpp:11) */
    float presence_penalty; /* 0 = off; used by gcuda_accept only (the rejection samplers take none and ignore it) */
} gcuda_sampling;

/* The acceptance of geode_generate (engine/src/geode.cpp:327-350) on the last verified batch's logits (on the
 * device): row i sampled with uniforms[i] (the draw Sampler::sample makes for row i, in [0,1); ignored when
 * greedy); draft i+1 stands while row i's sample equals toks[i+1] and is not in stops. Returns kept (1 .. n) in
 * *kept, the first sample that is no draft in *next, and every row's sample in samples[n] (NULL: not wanted).
 * With a presence penalty (engine/src/geode.cpp:234-255), seen[n_seen] lists the tokens the answer has sampled so
 * far, each once (ids in [0, vocab); GCUDA_E_ARG otherwise): before row i is sampled, the penalty is subtracted from
 * its logit of every listed token and of every draft toks[1..i] not listed (the samples of rows 0..i-1 when their
 * drafts stood), once per token - in place, in the device logits. The caller then adds the samples of rows
 * 0..kept-1 that are new to its list. seen is ignored when the penalty is 0. */
int gcuda_accept(gcuda *g, const gcuda_sampling *s, const double *uniforms, const int *stops, int n_stops,
                 const int *seen, int n_seen, int *kept, int *next, int *samples);
/* Speculative (rejection) sampling (Leviathan et al. 2023) over S sequences x (k+1) target rows and k draft rows of V
 * logits already on the device (target [S][k+1][V], draft [S][k][V]), Philox4x32-10 uniforms (key seed, counter
 * (sequence, row)); accepted[S] and next[S] on the host. Not in the reference: no counterpart there. */
int gcuda_spec_reject(gcuda *g, const float *d_target, const float *d_draft, const int *drafts, int S, int k, int V,
                      const gcuda_sampling *s, uint64_t seed, int *accepted, int *next);

/* The conversation's state to and from the host, in the reference's own buffer layouts (engine/src/model.hpp:548-555):
 * conv [n_gdn][conv_dim][K-1] f32, gdn [n_gdn][nv][dv/16][dk][16] f32, kv [A][2][positions][nkv*hd] int8,
 * kv_scale [A][2][positions][nkv] f32 for positions 0..pos-1, A the attention layers and, with an MTP layer, its slot
 * after them (engine/src/model.cpp:354: the engine counts it among n_attn); pos the new position (put). */
int gcuda_state_get(gcuda *g, float *conv, float *gdn, int8_t *kv, float *kv_scale, int positions);
int gcuda_state_put(gcuda *g, const float *conv, const float *gdn, const int8_t *kv, const float *kv_scale, int pos);
/* The last position's hidden row after the final norm (the engine's last_hid_, which a state file keeps for the MTP
 * layer, engine/src/state.cpp:275): the last verified batch's row n-1, or kept-1 after gcuda_keep. GCUDA_E_STATE when
 * the device holds none (after gcuda_reset or gcuda_state_put). gcuda_put_last_hidden: that row given back after a
 * gcuda_state_put (a loaded state's); a gcuda_draft with hidden NULL and n = 1 then takes it. */
int gcuda_last_hidden(gcuda *g, float *out);
int gcuda_put_last_hidden(gcuda *g, const float *row);

/* Device pointers of the last batch's results (the verify step's outputs stay resident): logits [max_tokens][vocab]. */
const float *gcuda_device_logits(gcuda *g);
/* The verify step with the tokens already on the device (d_toks: n int32) and the results left there - the resident
 * form of gcuda_verify for callers that keep their batches on the GPU. Token ids are checked on the device only: one
 * out of range gives GCUDA_E_DEVICE after the step has run on a zero row in its place, the position unmoved but the
 * recurrent states advanced - reset or load the conversation after it. */
int gcuda_verify_device(gcuda *g, const int *d_toks, int n);
/* Milliseconds of the last gcuda_verify / gcuda_verify_device on the device (CUDA events on the handle's stream). */
float gcuda_last_ms(gcuda *g);
/* Kernels this library launched since the handle opened. */
uint64_t gcuda_launches(gcuda *g);
/* The stream the handle enqueues on (a cudaStream_t), for callers that time it with their own events. */
void *gcuda_stream(gcuda *g);
/* The embedding table in the pack's own row layout (rows are gathered, not streamed): an id for gcuda_setup's embed. */
int gcuda_adopt_embedding(gcuda *g, const uint8_t *data, int64_t rows, int64_t cols, float global);

/* ------------------------------------------------------------------------------------ the device-resident loop ----
 * The speculative step without host round trips (the drafts are the previous batch's own tokens - a measuring loop):
 * gcuda_begin_device_loop puts the position and the first batch on the device; each gcuda_step_device(n) enqueues the
 * verify graph, the greedy acceptance of every row, the decision (kept, next, position += kept) and the rollback;
 * gcuda_sync_step waits and returns the steps taken, the sum over the routed layers of the experts this rank read
 * (the union of the picks; under expert parallelism this rank's members of it) and the last kept count. No counterpart in the reference (its loop is host code, engine/src/geode.cpp:318-370). */
int gcuda_begin_device_loop(gcuda *g, const int *toks, int n);
int gcuda_step_device(gcuda *g, int n);
int gcuda_sync_step(gcuda *g, int *steps, int *union_sum, int *last_kept);
/* gcuda_step_device with speculative (rejection) sampling in place of the greedy acceptance (the draft-model
 * configurations): the verified rows against the draft model's rows d_draft [n-1][vocab] on the device, the drafts
 * toks[1..n-1]; Philox4x32-10 key = seed plus the handle's count of these steps times a constant. As
 * gcuda_spec_reject for one sequence, chained on the device with the decision and the rollback. No counterpart in
 * the reference (it has no rejection sampling, and its loop is host code). */
int gcuda_step_device_reject(gcuda *g, int n, const float *d_draft, const gcuda_sampling *s, uint64_t seed);

/* ----------------------------------------------------------------------------------------- synthetic models ----
 * Seeded weights made straight in device memory, for measuring runs whose values do not matter (the self-test
 * weights of engine/src/gpu_check.cpp:51-63: random q4 codes, E4M3 scale bytes in 0x30..0x48). Each returns an id
 * like its gcuda_adopt_* counterpart. synth_raw: dtype 0 f32, 1 bf16, values N(mean, stdv). gcuda_state_randomize
 * fills the KV cache up to pos with random int8 rows (scales 0.5) and the conv and recurrent states with small
 * random values, and sets the position to pos. */
int gcuda_synth_q4(gcuda *g, int64_t rows, int64_t cols, float global, uint64_t seed);
int gcuda_synth_raw(gcuda *g, size_t count, int dtype, float mean, float stdv, uint64_t seed);
int gcuda_synth_embedding(gcuda *g, int64_t rows, int64_t cols, float global, uint64_t seed);
int gcuda_synth_experts(gcuda *g, int n, int hidden, int ff, float global, uint64_t seed);
int gcuda_state_randomize(gcuda *g, int pos, uint64_t seed);

/* ------------------------------------------------------------------------------------------------ test hooks ----
 * gcuda_debug_read: the device copy of one of the last step's intermediate rows (what: 0 x, 1 hf, 2 core_f,
 * 3 route, 4 hidden, 5 conv output, 6 a|b, 7 z, 8 qkv product); gcuda_debug_step_eager: the step launched kernel by
 * kernel instead of through the graph (pdl 0/1). */
int gcuda_debug_read(gcuda *g, int what, void *out, size_t bytes);
/* The kernels' float exp (the reference's: glibc's expf, restated) of the floats whose bit patterns are first ..
 * first + count - 1, into d_out [count] on `stream`: for checking it against the host's expf. */
int gcuda_debug_expf_table(uint32_t first, int64_t count, float *d_out, void *stream);
int gcuda_debug_step_eager(gcuda *g, const int *toks, int n, int pdl);
/* One step as gcuda_verify (position and batch advance; logits left on the device) launched kernel by kernel with a
 * per-layer trace, the reference's LayerTrace (engine/src/model.hpp:92-105): x [n_layers + 1][n][hidden] (each layer's
 * input, then the last layer's output); for MoE models (else untouched; each may be NULL) router_logits
 * [n_layers][n][n_experts + 1] (the router's logits, then the shared expert's gate logit), ids and weights
 * [n_layers][n][top_k] (route_topk's picks), gate [n_layers][n] (the shared expert's sigmoid gate) and n_union
 * [n_layers] (distinct experts picked). */
int gcuda_debug_trace(gcuda *g, const int *toks, int n, float *x, float *router_logits, int *ids, float *weights,
                      float *gate, int *n_union);
/* Device time per kind of launch: `reps` steps of the n tokens at the current position (the position does not move),
 * launched kernel by kernel without programmatic overlap so that CUDA events bracket each launch. ms[4] and
 * launches[4] per step for GCUDA_KT_GATE_UP (the routed and shared experts' gate|up product with SwiGLU), GCUDA_KT_DOWN
 * (their down product), GCUDA_KT_LM_HEAD and GCUDA_KT_DENSE (the layers' other q4 products); *step_ms the whole step
 * (NULL: not wanted), *union_sum the routed experts the step's MoE layers read on this rank (summed over layers;
 * NULL: not wanted). */
#define GCUDA_KT_GATE_UP 0
#define GCUDA_KT_DOWN 1
#define GCUDA_KT_LM_HEAD 2
#define GCUDA_KT_DENSE 3
int gcuda_debug_kernel_times(gcuda *g, const int *toks, int n, int reps, float *ms, int *launches, float *step_ms,
                             int *union_sum);

/* ------------------------------------------------------------------------------------------- operators ---- */
/* All on caller-owned device memory, enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream).
 * They return once enqueued. */
/* The operators' status word on the current device, after the work enqueued so far (synchronous): 0, or the flags
 * kernels raised (1: a bounded wait gave up, 2: a shape out of range, 4: a bad token id); clear != 0 zeroes it. */
int gcuda_op_status(int clear);

/* tiles: the bytes gcuda_op_q4_tiled_bytes gives; the pack's rows -> the GEMV's tile layout */
size_t gcuda_op_q4_tiled_bytes(int64_t rows, int64_t cols);
int gcuda_op_q4_relayout(const uint8_t *d_pack, int64_t rows, int64_t cols, uint8_t *d_tiles, void *stream);
/* quantize_activation for n rows of cols floats (engine/src/kernels.cpp:1254-1295): q [n][cols], scale and bsum
 * [n][cols/16] */
int gcuda_op_quantize(const float *d_x, int n, int cols, int8_t *d_q, float *d_scale, int32_t *d_bsum, void *stream);
/* The step's norm-and-quantize kernel for n rows of H floats: hf = rmsnorm(x, w) with the zero-centred weight (1 + w)
 * and the sum of squares in double (engine/src/kernels.cpp:1520-1529), then quantize_activation of hf
 * (engine/src/kernels.cpp:1254-1295): hf [n][H] (NULL: not written), q [n][H], scale and bsum [n][H/16]. H a multiple
 * of 16, at most 4096. */
int gcuda_op_norm_quant(const float *d_x, int n, int H, const float *d_w, float eps, float *d_hf, int8_t *d_q,
                        float *d_scale, int32_t *d_bsum, void *stream);
/* y[t][r] = matvec_rows_q_ref (engine/src/kernels.cpp:1304-1322) of the tiled matrix with n (<= 8) quantized rows;
 * bit for bit the reference's int8 product. y [n][rows]. */
int gcuda_op_q4_gemv(const uint8_t *d_tiles, int64_t rows, int64_t cols, float global, const int8_t *d_q,
                     const float *d_scale, const int32_t *d_bsum, int n, float *d_y, void *stream);
/* The tensor-core (tcgen05) q4 product for any number of token rows. The matrix first goes to its "U" layout
 * (gcuda_op_q4_umma_bytes: 9/16 byte per value, as the pack; rows a multiple of 128, cols of 256; 0 otherwise; the
 * product takes cols up to 4096) from
 * the pack's rows (C/2 code bytes then C/16 E4M3 bytes). y [n][rows] = matvec_rows_q_ref (engine/src/kernels.cpp:
 * 1304-1322) of each of the n quantized rows (q [n][cols], scale and bsum [n][cols/16]), bit for bit: int8 MMAs give
 * each 16-value block's own integer sum, the float chain over the blocks runs in block order. A wait inside the
 * kernel that gives up sets the operators' status word (gcuda_op_status). */
size_t gcuda_op_q4_umma_bytes(int64_t rows, int64_t cols);
int gcuda_op_q4_umma_relayout(const uint8_t *d_pack, int64_t rows, int64_t cols, uint8_t *d_u, void *stream);
int gcuda_op_q4_gemm_umma(const uint8_t *d_u, int64_t rows, int64_t cols, float global, const int8_t *d_q,
                          const float *d_scale, const int32_t *d_bsum, int n, float *d_y, void *stream);
/* The routed experts of many token rows at once on the tensor core (the batched configuration), bit for bit the
 * reference's per-pick products (Model::moe, engine/src/model.cpp:4496-4543): out [n*K][H] row p = t * K + k =
 * down(quant(silu(gate) * up)) of expert ids[p] on token t's quantized h (q [n][H], scale and bsum [n][H/16]), where
 * gate | up = gate_up . h. The experts in the U layout, expert e's block (gate_up 2 ff x H, then down H x ff) at
 * d_u + e * gcuda_op_moe_umma_expert_bytes(H, ff), made from the pack's blocks by gcuda_op_moe_umma_relayout;
 * d_globals [E][2] their per-matrix scales. H and ff multiples of 256, at most 4096; E <= 1024. d_work: the caller's
 * scratch of gcuda_op_moe_umma_work_bytes (256-byte aligned): the picks grouped by expert and the units of the two
 * grouped products are planned on the device. The combine (weights, shared expert) is the caller's. An expert id out
 * of range: its pick is left out and the status word (gcuda_op_status) raised. */
/* The verify step's expert kernels (a lane a weight row: dp4a on the codes for only the tokens that picked each expert,
 * the reference's block chain in that lane) for n <= 8 token rows, K <= 8 picks each: every pick p = t * K + k of
 * expert ids[p] gives d_out row p = W_dn[e] . quant(silu(g) * u), [g | u] = W_gu[e] . quant(h_t) - bit for bit the
 * reference's per-pick product (engine/src/model.cpp:4496-4543). d_r16: E expert blocks in the kernels' R16 layout,
 * gcuda_op_moe_lane_expert_bytes(H, ff) apart, made from the pack's blocks by gcuda_op_moe_lane_relayout (which
 * allocates a temporary and synchronises `stream`); d_q/d_scale/d_bsum: h quantized (gcuda_op_quantize); d_work:
 * scratch of gcuda_op_moe_lane_work_bytes, 256-byte aligned. At most 64 distinct experts among the picks. */
size_t gcuda_op_moe_lane_expert_bytes(int H, int ff);
size_t gcuda_op_moe_lane_work_bytes(int n, int K, int H, int ff);
int gcuda_op_moe_lane_relayout(const uint8_t *d_pack, size_t pack_stride, int E, int H, int ff, uint8_t *d_out,
                               void *stream);
int gcuda_op_moe_lane(const uint8_t *d_r16, const float *d_globals, int E, int H, int ff, const int8_t *d_q,
                      const float *d_scale, const int32_t *d_bsum, int n, const int *d_ids, int K, float *d_out,
                      void *d_work, size_t work_bytes, void *stream);
size_t gcuda_op_moe_umma_expert_bytes(int H, int ff);
size_t gcuda_op_moe_umma_work_bytes(int n, int K, int E, int H, int ff);
int gcuda_op_moe_umma_relayout(const uint8_t *d_pack, size_t pack_stride, int E, int H, int ff, uint8_t *d_u,
                               void *stream);
int gcuda_op_moe_umma(const uint8_t *d_u, const float *d_globals, int E, int H, int ff, const int8_t *d_q,
                      const float *d_scale, const int32_t *d_bsum, int n, const int *d_ids, int K, float *d_out,
                      void *d_work, size_t work_bytes, void *stream);
/* dequant_row (engine/src/kernels.cpp:1214-1228) of nrows rows (d_rows int64) of a tiled matrix: out [nrows][cols] */
int gcuda_op_q4_dequant(const uint8_t *d_tiles, int64_t cols, float global, const int64_t *d_rows, int nrows,
                        float *d_out, void *stream);
/* matvec_rows_bf16_multi (engine/src/kernels.cpp:1449-1518), bit for bit: y [n][rows] = W [rows][cols] x [n][cols] */
int gcuda_op_bf16_gemv(const uint16_t *d_w, int rows, int cols, const float *d_x, int n, float *d_y, void *stream);
/* route_topk (engine/src/model.cpp:4021-4065) for n rows of E logits: ids [n][K], weights [n][K] */
int gcuda_op_route_topk(const float *d_logits, int n, int E, int K, int *d_ids, float *d_weights, void *stream);
/* The verify step's MoE routing for n <= 8 tokens (one kernel): route_topk per token (engine/src/model.cpp:4021-4065),
 * the shared expert's gate sigmoid (engine/src/model.cpp:4564-4567) and the union of the picked experts
 * (engine/src/model.cpp:4183-4196). d_logits: n rows of E + 1 floats (E router logits, then the shared expert's gate
 * logit); E <= 1024, K <= 8. d_out (out_bytes >= gcuda_op_route_out_bytes()) receives, as 32-bit fields:
 *   int n_union; int ex[64] (union members, ascending ids); int mask[64] (bit t: token t picked ex[u]);
 *   int slot[64][8] (slot[u][t] = t * K + k of that pick, where mask bit t is set); int ids[64] ([n][K]);
 *   float w[64] ([n][K] normalised weights); float gs[8] (the shared expert's gate per token). */
size_t gcuda_op_route_out_bytes(void);
int gcuda_op_route_union(const float *d_logits, int n, int E, int K, void *d_out, size_t out_bytes, void *stream);
/* Greedy speculative acceptance of S sequences at once (geode_generate's rule at temperature 0,
 * engine/src/geode.cpp:327-350, no stop tokens): row i's sample is its first maximum (Sampler::sample at temperature
 * 0, std::max_element, engine/src/sampler.cpp:16-22; NaN never the maximum, a row of NaN only gives 0); draft i
 * stands while row i's sample equals it. d_target [S][k+1][V], d_drafts [S][k]; d_accepted[S] = drafts that stood,
 * d_next[S] = the sample of the first row whose draft fell (row k's when all stood). d_scratch: S*(k+1) 64-bit words
 * the call zeroes first. No counterpart in the reference as one call (its rule runs per sequence on the host). */
int gcuda_op_greedy_verify(const float *d_target, const int *d_drafts, int S, int k, int V, uint64_t *d_scratch,
                           int *d_accepted, int *d_next, void *stream);

/* gcuda_spec_reject without a handle and without allocating: for callers that must not allocate device memory when
 * they call it (a serving loop that holds a fixed device-memory budget, or one that cannot take the implicit
 * synchronisation of cudaMalloc / cudaFree in its step). Same arguments and results as gcuda_spec_reject (d_target
 * [S][k+1][V] and d_draft [S][k][V] on the device, drafts [S][k] and accepted[S] / next[S] on the host), on `stream`;
 * every call copies the drafts from host memory and synchronises `stream`, so it blocks the calling thread until the
 * results are on the host. Its scratch is a fixed device array of the library, so S <= 1024 and k <= 16 (GCUDA_E_ARG
 * beyond). The first call on a device looks that array up (cudaGetSymbolAddress, with the device current) and keeps
 * the address for the life of the process: make that first call before any stream capture, and do not call
 * cudaDeviceReset on a device between calls (the kept address would no longer be valid). Calls that overlap on one
 * device - from several threads or streams - share the array and race; serialise them. No counterpart in the
 * reference. */
int gcuda_op_spec_reject_static(const float *d_target, const float *d_draft, const int *drafts, int S, int k, int V,
                                const gcuda_sampling *s, uint64_t seed, int *accepted, int *next, void *stream);

#ifdef __cplusplus
}
#endif
#endif
