// backend.cu - the gcuda_* backend of geode_cuda.h: weights adopted into device memory, the conversation's device
// state, and the verify step (Model::verify_n's Adreno branch, engine/src/model.cpp:1529-1592, redone for sm_100a)
// recorded once per batch size as a CUDA graph of dependent launches.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/geode_cuda.h"
#include "gemv_kernels.cuh"
#include "launch.hpp"
#include "ops_impl.cuh"
#include "accept.cuh"
#include "noalloc_impl.cuh"
#include "ep_exchange.cuh"
#include "experts_lane.cuh"

using namespace gcu;

namespace {

enum TensorKind { kQ4Tiled = 0, kRaw = 1 };

struct DevTensor {
    void *d = nullptr;
    size_t bytes = 0;
    int64_t rows = 0, cols = 0;
    float global = 1.0f;
    int kind = kRaw;
};

struct DevExperts {
    uint8_t *d = nullptr;
    bool tiled = false;   // already in the GEMV's tile layout (synthesized on the device)
    bool r16 = false;     // in the expert kernels' R16 layout (experts_lane.cuh)
    int n = 0;
    size_t stride = 0;
    float *scales = nullptr;   // device [n][2]
    std::vector<float> host_scales;
};

struct ActBuf {
    int8_t *q = nullptr;
    float *scale = nullptr;
    int32_t *bsum = nullptr;
    int cols = 0, n = 0;
    ActSet set() const { return ActSet{q, scale, bsum, cols, n, cols, cols / 16}; }
};

struct LayerPlan {
    int gi = -1, ai = -1;                 // index among GDN / attention layers
    int u_in = 0, n_in = 0;               // unit table range: the mixer's input products
    int u_out = 0, n_out = 0;             // the mixer's output product
    int u_mlp = 0, n_mlp = 0, u_dn = 0, n_dn = 0;   // dense MLP
    uint16_t *ab_w = nullptr;             // GDN a|b rows (bf16 [2 nv][H])
    uint16_t *router_w = nullptr;         // MoE router rows + the shared gate row ([E+1][H])
};

}  // namespace

namespace {
// NCCL, loaded on first use (single-GPU users need no NCCL): the few functions the expert-parallel step calls
struct NcclApi {
    bool tried = false, ok = false;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};
NcclApi &nccl() {
    static NcclApi a;
    if (!a.tried) {
        a.tried = true;
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            a.get_unique_id = reinterpret_cast<decltype(&ncclGetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
            a.comm_init_rank = reinterpret_cast<decltype(&ncclCommInitRank)>(dlsym(h, "ncclCommInitRank"));
            a.all_reduce = reinterpret_cast<decltype(&ncclAllReduce)>(dlsym(h, "ncclAllReduce"));
            a.all_gather = reinterpret_cast<decltype(&ncclAllGather)>(dlsym(h, "ncclAllGather"));
            a.comm_destroy = reinterpret_cast<decltype(&ncclCommDestroy)>(dlsym(h, "ncclCommDestroy"));
            a.error_string = reinterpret_cast<decltype(&ncclGetErrorString)>(dlsym(h, "ncclGetErrorString"));
            a.ok = a.get_unique_id && a.comm_init_rank && a.all_reduce && a.all_gather && a.comm_destroy && a.error_string;
        }
    }
    return a;
}

}  // namespace

struct gcuda {
    int device = 0;
    cudaStream_t st = nullptr;
    std::string err;
    std::vector<DevTensor> tensors;
    std::vector<DevExperts> experts;
    bool ready = false;
    gcuda_shape sh{};
    std::vector<gcuda_layer> layers;
    std::vector<LayerPlan> plan;
    int embed = -1, lm_head = -1, final_norm = -1;
    int n_gdn = 0, n_attn = 0, conv_dim = 0, vd = 0, kd = 0, qw = 0, kvrow = 0, corew = 0;
    // state
    float *conv = nullptr, *gdn = nullptr, *conv_bk = nullptr, *gdn_bk = nullptr;
    size_t conv_n = 0, gdn_n = 0;   // floats per copy (all GDN layers)
    int8_t *kc = nullptr, *vc = nullptr;
    float *ks = nullptr, *vs = nullptr;
    // scratch
    int *d_toks = nullptr, *d_pos = nullptr;
    uint32_t *d_status = nullptr;
    float *x = nullptr, *hf = nullptr, *big = nullptr, *zb = nullptr, *ab = nullptr, *kb = nullptr, *vb = nullptr,
          *qn = nullptr, *rlog = nullptr, *eout = nullptr, *shout = nullptr, *part = nullptr, *logits = nullptr,
          *hid = nullptr, *core_f = nullptr, *inv_freq = nullptr, *convd = nullptr;
    ActBuf hq, core, amid, shact;
    RouteOut *route = nullptr;
    GemvUnit *units = nullptr;
    int n_units = 0, lm_u = 0;
    int nchunks = 0;
    // graphs per batch size
    cudaGraphExec_t graph[kMaxTok + 1] = {};
    uint64_t graph_kernels[kMaxTok + 1] = {};   // kernels one launch of graph[n] runs
    int pos = 0, last_batch = 0;
    // hid's rows that hold positions of the conversation (the final norm's rows, the MTP pass's input): the last
    // verified batch's n, its kept ones after gcuda_keep, 1 after gcuda_put_last_hidden; row hid_rows - 1 is the last
    // position's (the engine's last_hid_, engine/src/model.cpp:1585, 1602)
    int hid_rows = 0;
    int last_toks[kMaxTok] = {};
    uint32_t *h_status = nullptr;  // pinned: the status word's copy, read after the step's one synchronization
    StepState *step = nullptr;     // the device-side loop's decision and counters
    double *d_u = nullptr;
    int *d_samples = nullptr;
    unsigned long long *d_best = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    // a second stream for work beside the main chain (the Gated DeltaNet's a|b product beside its input product),
    // forked and joined by events - also inside the step's captured graphs
    cudaStream_t st2 = nullptr;
    cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
    float last_ms = 0.0f;
    bool pdl = true;
    int *rej = nullptr;   // gcuda_spec_reject's device buffers: drafts, accepted, next
    size_t rej_cap = 0;
    int *d_rej_step = nullptr;      // gcuda_step_device_reject's result: accepted, next
    // gcuda_debug_kernel_times: events around each launch of the timed kinds inside eager steps (off: null)
    struct KernelMarks {
        std::vector<cudaEvent_t> pool;          // created on demand, kept for the handle's life
        std::vector<std::pair<int, int>> marks; // (kind, first of the two pool events)
        size_t used = 0;
    };
    KernelMarks *kt = nullptr;
    // gcuda_debug_trace: per-layer copies enqueued inside one eager step (null outside it)
    float *tr_x = nullptr;          // [n_layers + 1][n][H]: each layer's input x, then the last layer's output
    float *tr_rlog = nullptr;       // [n_layers][n][E + 1]: the router's logits (and the shared expert's gate logit)
    RouteOut *tr_route = nullptr;   // [n_layers]
    int *d_seen = nullptr;          // gcuda_accept's presence-penalty list on the device (grown on demand)
    size_t seen_cap = 0;
    std::vector<uint8_t> seen_mark; // (a host bitmap over the vocabulary, all zero between calls)
    uint64_t reject_steps = 0;      // (its Philox sequence index: one per step)
    std::vector<void *> allocs;
    // expert parallelism (gcuda_set_ep): this rank's experts are e % ep_world == ep_rank; the expert outputs meet
    // through the down kernel's peer stores over NVLink and per-layer flags; NCCL only carries the set-up's handles
    int ep_rank = 0, ep_world = 1;
    ncclComm_t comm = nullptr;
    void *xbuf = nullptr;               // this rank's exchange buffer: flags [n_layers][world] (padded), then eout
    uint32_t *xflags = nullptr;
    size_t eout_stride = 0;             // expert parallelism: floats of one layer's slot of eout (a slot per layer)
    int *ep_epoch = nullptr;            // (device) the step's epoch, one per step
    unsigned int *xcount = nullptr;     // (device) the exchange kernel's arrival counter
    void *peer_base[kMaxEpWorld] = {};  // the peers' exchange buffers, mapped here
    float *peer_eout[kMaxEpWorld] = {};
    uint32_t *peer_flags[kMaxEpWorld] = {};
    // the MTP drafting layer (gcuda_set_mtp): an attention layer with the model's MLP on its own KV slot (attention
    // slot n_attn), its fc and norms; one pass per draft, captured per row count
    bool has_mtp = false;
    int mtp_fc = -1, mtp_pre_e = -1, mtp_pre_h = -1, mtp_norm = -1;
    gcuda_layer mtp_layer{};
    LayerPlan mtp_plan;
    int mtp_fc_u = 0, mtp_lm_u = 0;
    ActBuf mtp_in;                      // [T][2H]: the fc's input rows, quantized
    float *mtp_hin = nullptr;           // [T][H]: the hidden rows the pass takes
    float *mtp_hf = nullptr;            // [T][H]: its rows after mtp.norm (a chained draft's hidden row)
    float *mtp_logits = nullptr;        // [V]: the last row's logits
    float *mtp_prob = nullptr;
    double *mtp_part = nullptr;         // k_softmax_at's partial sums
    unsigned int *mtp_count = nullptr;
    int *d_mtp_toks = nullptr, *d_mtp_pos = nullptr, *d_mtp_draft = nullptr;
    unsigned long long *d_mtp_best = nullptr;
    cudaGraphExec_t mtp_graph[kMaxTok + 1] = {};
    uint64_t mtp_graph_kernels[kMaxTok + 1] = {};
    int mtp_rows = 0;                   // the last pass's rows (a chained draft goes on from row mtp_rows - 1)
    // the draft head (gcuda_set_draft_head): lm_head's rows of a draft vocabulary, the MTP pass's logits over them
    int draft_head = -1;
    std::vector<int> draft_ids;
    int mtp_vocab = 0;                  // the MTP pass's logits: draft_ids.size(), or the vocabulary
};

namespace {

int fail(gcuda *g, int code, const std::string &msg) {
    if (g) g->err = msg;
    return code;
}

int cuda_fail(gcuda *g, cudaError_t e, const char *what) {
    return fail(g, e == cudaErrorMemoryAllocation ? GCUDA_E_MEMORY : GCUDA_E_CUDA,
                std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename T>
bool dalloc(gcuda *g, T **p, size_t count) {
    void *q = nullptr;
    if (count == 0) count = 1;
    const cudaError_t e = cudaMalloc(&q, count * sizeof(T));
    if (e != cudaSuccess) {
        cuda_fail(g, e, "cudaMalloc");
        return false;
    }
    cudaMemsetAsync(q, 0, count * sizeof(T), g->st);
    g->allocs.push_back(q);
    *p = static_cast<T *>(q);
    return true;
}

bool act_alloc(gcuda *g, ActBuf &a, int n, int cols) {
    a.n = n;
    a.cols = cols;
    return dalloc(g, &a.q, static_cast<size_t>(n) * cols) && dalloc(g, &a.scale, static_cast<size_t>(n) * cols / 16) &&
           dalloc(g, &a.bsum, static_cast<size_t>(n) * cols / 16);
}

const DevTensor *tensor(gcuda *g, int id, int kind) {
    if (id < 0 || id >= static_cast<int>(g->tensors.size())) return nullptr;
    const DevTensor &t = g->tensors[static_cast<size_t>(id)];
    return t.kind == kind ? &t : nullptr;
}

// units of a plain matrix: rows / 32 units of adjacent tile pairs, outputs y + row (ystride between tokens)
void plain_units(std::vector<GemvUnit> &out, const DevTensor &m, float *y, int ystride, int mode) {
    const size_t tb = static_cast<size_t>(tile_bytes(static_cast<int>(m.cols)));
    const int64_t units = (m.rows + 31) / 32;
    for (int64_t u = 0; u < units; ++u) {
        GemvUnit U{};
        U.w0 = static_cast<const uint8_t *>(m.d) + (2 * u) * tb;
        U.w1 = U.w0 + tb;
        U.g0 = U.g1 = m.global;
        U.y0 = y + 32 * u;
        U.y1 = U.y0 + 16;
        U.ngroups = static_cast<int>(m.cols / 64);
        U.ystride = ystride;
        U.mode = mode;
        U.tok_mask = 0xFF;
        for (int t = 0; t < kMaxTok; ++t) U.slot[t] = t;
        out.push_back(U);
    }
}

// silu(gate) * up units: gate tile i with up tile i (rows multiples of 16), into act rows t
void swiglu_units(std::vector<GemvUnit> &out, const DevTensor &gt, const DevTensor &up, const ActBuf &a) {
    const size_t tb = static_cast<size_t>(tile_bytes(static_cast<int>(gt.cols)));
    for (int64_t i = 0; i < gt.rows / 16; ++i) {
        GemvUnit U{};
        U.w0 = static_cast<const uint8_t *>(gt.d) + i * tb;
        U.w1 = static_cast<const uint8_t *>(up.d) + i * tb;
        U.g0 = gt.global;
        U.g1 = up.global;
        U.ngroups = static_cast<int>(gt.cols / 64);
        U.mode = kSwiglu;
        U.tok_mask = 0xFF;
        for (int t = 0; t < kMaxTok; ++t) U.slot[t] = t;
        U.aq = a.q;
        U.as = a.scale;
        U.ab = a.bsum;
        U.acols = a.cols;
        U.arow0 = static_cast<int>(16 * i);
        out.push_back(U);
    }
}

// act_cols: the width of the activation rows the units multiply (0: the buffer's own width); the rows are packed
// at that width (a narrower writer, e.g. the Gated DeltaNet core, packs them so)
// swiglu: the units pair gate and up tiles (they cannot be split into one-tile units)
// The launches gcuda_debug_kernel_times tells apart (kind ids of include/geode_cuda.h's GCUDA_KT_*).
enum { kKtGateUp = 0, kKtDown = 1, kKtLmHead = 2, kKtDense = 3, kKtKinds = 4 };

// Records an event on the handle's stream before (begin) or after (end) a launch of `kind` while kernel timing is
// on; nothing otherwise (and never inside a graph capture: the timing runs eager steps only).
bool kt_mark(gcuda *g, int kind, bool begin) {
    if (!g->kt) return true;
    gcuda::KernelMarks &m = *g->kt;
    if (m.used >= m.pool.size()) {
        cudaEvent_t e = nullptr;
        if (cudaEventCreate(&e) != cudaSuccess) return false;
        m.pool.push_back(e);
    }
    const int id = static_cast<int>(m.used++);
    if (begin) m.marks.emplace_back(kind, id);
    return cudaEventRecord(m.pool[static_cast<size_t>(id)], g->st) == cudaSuccess;
}

int launch_units(gcuda *g, int u0, int nu, const ActBuf &act, int n, bool pdl, int act_cols = 0, bool swiglu = false) {
    StaticGemv p{};
    p.units = g->units + u0;
    p.n_units = nu;
    p.act = act.set();
    if (act_cols > 0) p.act = ActSet{act.q, act.scale, act.bsum, act_cols, act.n, act_cols, act_cols / 16};
    p.ncols = n;
    p.allow_half = swiglu ? 0 : 1;
    p.allow_split = 1;
    p.status = g->d_status;
    const bool head = u0 == g->lm_u;
    if (!kt_mark(g, head ? kKtLmHead : kKtDense, true)) return GCUDA_E_CUDA;
    const int rc = launch_static_gemv(p, g->st, pdl);
    if (!kt_mark(g, head ? kKtLmHead : kKtDense, false)) return GCUDA_E_CUDA;
    return rc;
}

#define LAUNCH_OK(call)                                                        \
    do {                                                                       \
        const cudaError_t e_ = (call);                                         \
        if (e_ != cudaSuccess) return cuda_fail(g, e_, #call);                 \
    } while (0)
#define RC_OK(call)                                                            \
    do {                                                                       \
        const int r_ = (call);                                                 \
        if (r_ != GCUDA_OK) return g->err.empty() ? fail(g, r_, #call) : r_;   \
    } while (0)

// The expert outputs of layer l: one buffer on one GPU; under expert parallelism a slot per layer (the MTP layer's
// after the model's), so that a peer storing layer l + 1's rows never meets this rank still combining layer l's.
float *eout_of(gcuda *g, int l) { return g->eout + (g->ep_world > 1 ? static_cast<size_t>(l) * g->eout_stride : 0); }

const float *raw_of(gcuda *g, int id) {
    const DevTensor *t = tensor(g, id, kRaw);
    return t ? static_cast<const float *>(t->d) : nullptr;
}

// rmsnorm (+ quantize) of the n rows of x into `out` from column col0 (out's rows may be wider than H: the two halves
// of the MTP layer's input); with combine, the MoE combine of layer moe_layer into x first.
int enqueue_norm(gcuda *g, int n, float *x, const float *w, bool combine, float *hf_out, int moe_layer,
                 const ActBuf &out, int col0 = 0) {
    const gcuda_shape &s = g->sh;
    NormArgs a{};
    a.x = x;
    a.w = w;
    a.eps = s.eps;
    a.H = s.hidden;
    a.n = n;
    a.hf = hf_out;
    a.q = out.q + col0;
    a.scale = out.scale + col0 / 16;
    a.bsum = out.bsum + col0 / 16;
    a.ostride = out.cols;
    if (combine) {
        a.sh = g->shout;
        a.gs = g->route->gs;
        a.eout = eout_of(g, moe_layer);
        a.wk = g->route->w;
        a.K = s.top_k;
    }
    LAUNCH_OK(launch_ex(k_norm_quant, dim3(n), dim3(kNormThreads), 0, g->st, g->pdl, a));
    return GCUDA_OK;
}

// Expert parallelism's step start: the epoch advanced and every peer met (k_ep_tick).
int enqueue_tick(gcuda *g) {
    TickArgs ta{};
    ta.epoch = g->ep_epoch;
    ta.flags = g->xflags;
    for (int r = 0; r < kMaxEpWorld; ++r) ta.peer_flags[r] = g->peer_flags[r];
    ta.status = g->d_status;
    ta.rank = g->ep_rank;
    ta.world = g->ep_world;
    ta.row = g->sh.n_layers + 1;
    k_ep_tick<<<1, 32, 0, g->st>>>(ta);
    count_launch();
    LAUNCH_OK(cudaGetLastError());
    return GCUDA_OK;
}

// One decoder layer over the n rows of g->x, whose rmsnorm(x, in_norm) is in g->hf / g->hq already: the mixer at
// the positions d_pos.. (attention over KV slot P.ai), the MLP, then the next norm (next_norm into next_hf and g->hq,
// with the MoE combine). l: the layer's index (the MTP layer: n_layers).
int enqueue_layer(gcuda *g, int n, int l, const gcuda_layer &L, const LayerPlan &P, const int *d_pos,
                  const float *next_norm, float *next_hf) {
    const gcuda_shape &s = g->sh;
    const int H = s.hidden;
    const bool pdl = g->pdl;
    auto norm = [&](const float *w, bool combine, float *hf_out, int moe_layer = 0) -> int {
        return enqueue_norm(g, n, g->x, w, combine, hf_out, moe_layer, g->hq);
    };
    auto raw = [&](int id) { return raw_of(g, id); };
    if (!L.attn) {
        // the a|b product (the recurrence's gates) on the side stream, beside the input product and the conv
        LAUNCH_OK(cudaEventRecord(g->fork_ev, g->st));
        LAUNCH_OK(cudaStreamWaitEvent(g->st2, g->fork_ev, 0));
        RC_OK(launch_bf16_gemv(static_cast<const uint16_t *>(P.ab_w), 2 * s.gdn_v_heads, H, g->hf, H, n, g->ab,
                               2 * s.gdn_v_heads, g->d_status, g->st2, false));
        LAUNCH_OK(cudaEventRecord(g->join_ev, g->st2));
        RC_OK(launch_units(g, P.u_in, P.n_in, g->hq, n, pdl));
        GdnArgs a{};
        a.proj = g->big;
        a.z = g->zb;
        a.ab = g->ab;
        a.convw = raw(L.conv);
        a.A_log = raw(L.A_log);
        a.dt_bias = raw(L.dt_bias);
        a.gnorm = raw(L.gnorm);
        const size_t conv_l = static_cast<size_t>(g->conv_dim) * (s.conv_kernel - 1);
        const size_t st_l = static_cast<size_t>(s.gdn_v_heads) * s.gdn_v_dim * s.gdn_k_dim;
        a.conv_st = g->conv + P.gi * conv_l;
        a.state = g->gdn + P.gi * st_l;
        a.conv_bk = g->conv_bk + P.gi * conv_l;
        a.state_bk = g->gdn_bk + P.gi * st_l;
        a.bk_conv_stride = g->conv_n;
        a.bk_state_stride = g->gdn_n;
        a.n = n;
        a.nk = s.gdn_k_heads;
        a.nv = s.gdn_v_heads;
        a.dk = s.gdn_k_dim;
        a.dv = s.gdn_v_dim;
        a.K = s.conv_kernel;
        a.eps = s.eps;
        a.q = g->core.q;
        a.scale = g->core.scale;
        a.bsum = g->core.bsum;
        a.core_f = g->core_f;
        LAUNCH_OK(launch_ex(k_gdn_conv, dim3((g->conv_dim + 127) / 128), dim3(128), 0, g->st, pdl, a, g->conv_dim,
                            g->convd));
        a.proj = g->convd;
        cudaLaunchConfig_t cfg{};
        const int S = s.gdn_v_dim / 16;
        cfg.gridDim = dim3(s.gdn_v_heads * S);
        cfg.blockDim = dim3(128);
        cfg.stream = g->st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = S;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 2 : 1;
        cudaError_t e;
        LAUNCH_OK(cudaStreamWaitEvent(g->st, g->join_ev, 0));   // (the gates)
        if (s.gdn_k_dim == 128) e = cudaLaunchKernelEx(&cfg, k_gdn<128>, a);
        else if (s.gdn_k_dim == 64) e = cudaLaunchKernelEx(&cfg, k_gdn<64>, a);
        else e = cudaLaunchKernelEx(&cfg, k_gdn<32>, a);
        count_launch();
        LAUNCH_OK(e);
        RC_OK(launch_units(g, P.u_out, P.n_out, g->core, n, pdl, g->vd));
    } else {
        RC_OK(launch_units(g, P.u_in, P.n_in, g->hq, n, pdl));
        AttnPrepArgs pa{};
        pa.qg = g->big;
        pa.kb = g->kb;
        pa.vb = g->vb;
        pa.q_norm = raw(L.q_norm);
        pa.k_norm = raw(L.k_norm);
        pa.inv_freq = g->inv_freq;
        pa.pos = d_pos;
        pa.n = n;
        pa.nh = s.n_heads;
        pa.nkv = s.n_kv_heads;
        pa.hd = s.head_dim;
        pa.half = s.rope_dim / 2;
        pa.eps = s.eps;
        pa.qn = g->qn;
        const size_t kvl = static_cast<size_t>(s.context) * g->kvrow;
        pa.kc = g->kc + P.ai * kvl;
        pa.vc = g->vc + P.ai * kvl;
        pa.ks = g->ks + P.ai * static_cast<size_t>(s.context) * s.n_kv_heads;
        pa.vs = g->vs + P.ai * static_cast<size_t>(s.context) * s.n_kv_heads;
        pa.ctx = s.context;
        pa.status = g->d_status;
        const int items = n * (s.n_heads + 2 * s.n_kv_heads);
        LAUNCH_OK(launch_ex(k_attn_prep, dim3((items + 3) / 4), dim3(128), 4 * s.head_dim * sizeof(float), g->st, pdl, pa));
        AttnArgs aa{};
        aa.qn = g->qn;
        aa.kc = pa.kc;
        aa.vc = pa.vc;
        aa.ks = pa.ks;
        aa.vs = pa.vs;
        aa.pos = d_pos;
        aa.n = n;
        aa.nh = s.n_heads;
        aa.nkv = s.n_kv_heads;
        aa.ctx = s.context;
        aa.scale = 1.0f / std::sqrt(static_cast<float>(s.head_dim));
        aa.part = g->part;
        aa.nchunks = g->nchunks;
        const dim3 grid(g->nchunks, s.n_kv_heads);
        if (s.head_dim == 256) {
            LAUNCH_OK(launch_ex(k_attn_decode<256>, grid, dim3(kAttnThreads), attn_smem_bytes<256>(), g->st, pdl, aa));
        } else if (s.head_dim == 128) {
            LAUNCH_OK(launch_ex(k_attn_decode<128>, grid, dim3(kAttnThreads), attn_smem_bytes<128>(), g->st, pdl, aa));
        } else {
            LAUNCH_OK(launch_ex(k_attn_decode<64>, grid, dim3(kAttnThreads), attn_smem_bytes<64>(), g->st, pdl, aa));
        }
        MergeArgs ma{};
        ma.part = g->part;
        ma.qg = g->big;
        ma.pos = d_pos;
        ma.n = n;
        ma.nh = s.n_heads;
        ma.hd = s.head_dim;
        ma.nchunks = g->nchunks;
        ma.q = g->core.q;
        ma.scale = g->core.scale;
        ma.bsum = g->core.bsum;
        ma.core_f = g->core_f;
        LAUNCH_OK(launch_ex(k_attn_merge, dim3(n * s.n_heads), dim3(s.head_dim), sizeof(float) * g->nchunks, g->st, pdl, ma));
        RC_OK(launch_units(g, P.u_out, P.n_out, g->core, n, pdl, s.n_heads * s.head_dim));
    }
    // x += mix happened in the output product's epilogue; h = rmsnorm(x, post_norm)
    RC_OK(norm(raw(L.post_norm), false, g->hf));
    if (s.dense) {
        RC_OK(launch_units(g, P.u_mlp, P.n_mlp, g->hq, n, pdl, 0, true));
        RC_OK(launch_units(g, P.u_dn, P.n_dn, g->shact, n, pdl));
        RC_OK(norm(next_norm, false, next_hf));
    } else {
        const int E = s.n_experts;
        RC_OK(launch_bf16_gemv(static_cast<const uint16_t *>(P.router_w), E + 1, H, g->hf, H, n, g->rlog, E + 1,
                               g->d_status, g->st, pdl));
        LAUNCH_OK(launch_ex(k_route, dim3(1), dim3(kRouteThreads), kMaxTok * E * sizeof(float), g->st, pdl,
                            static_cast<const float *>(g->rlog), n, E, s.top_k, g->route, l < s.n_layers ? &g->step->n_union_sum : nullptr,
                            g->ep_rank, g->ep_world));
        if (g->tr_route && l < s.n_layers) {
            LAUNCH_OK(cudaMemcpyAsync(g->tr_route + l, g->route, sizeof(RouteOut), cudaMemcpyDeviceToDevice, g->st));
            LAUNCH_OK(cudaMemcpyAsync(g->tr_rlog + static_cast<size_t>(l) * n * (E + 1), g->rlog,
                                      static_cast<size_t>(n) * (E + 1) * sizeof(float), cudaMemcpyDeviceToDevice,
                                      g->st));
        }
        const DevExperts &X = g->experts[static_cast<size_t>(L.experts)];
        const DevTensor *sg = tensor(g, L.sh_gate, kQ4Tiled), *su = tensor(g, L.sh_up, kQ4Tiled),
                        *sd = tensor(g, L.sh_down, kQ4Tiled);
        // the union's routed experts and the shared expert, a lane a weight row (experts_lane.cuh)
        LaneArgs la{};
        la.route = g->route;
        la.experts = X.d;
        la.stride = X.stride;
        la.down_off = static_cast<size_t>(2 * s.moe_ff / 16) * (H / 64) * kLaneTileGroup;
        la.globals = X.scales;
        la.sh_gate = static_cast<const uint8_t *>(sg->d);
        la.sh_up = static_cast<const uint8_t *>(su->d);
        la.sh_down = static_cast<const uint8_t *>(sd->d);
        la.sh_g0 = sg->global;
        la.sh_g1 = su->global;
        la.sh_g2 = sd->global;
        la.H = H;
        la.ff = s.moe_ff;
        la.K = s.top_k;
        la.n = n;
        la.hq = g->hq.set();
        la.amid = g->amid.set();
        la.shact = g->shact.set();
        la.eout = eout_of(g, l);
        la.shout = g->shout;
        la.status = g->d_status;
        la.world = 1;
        if (g->ep_world > 1) {
            // the down kernel stores every owned pick's row into the peers' slots too and meets them at the layer's flags
            la.rank = g->ep_rank;
            la.world = g->ep_world;
            la.layer = l;
            for (int r = 0; r < kMaxEpWorld; ++r)
                la.peer_eout[r] = g->peer_eout[r] ? g->peer_eout[r] + static_cast<size_t>(l) * g->eout_stride : nullptr;
            la.flags = g->xflags;
            for (int r = 0; r < kMaxEpWorld; ++r) la.peer_flags[r] = g->peer_flags[r];
            la.epoch = g->ep_epoch;
            la.count = g->xcount;
        }
        const int lrc = launch_lane_pair(la, n, s.top_k, H, s.moe_ff, pdl, g->st, [&](int which, bool start) {
            return kt_mark(g, which == 0 ? kKtGateUp : kKtDown, start);
        });
        if (lrc == GCUDA_E_ARG) return fail(g, lrc, "the expert kernels' activation rows leave no room for their rings");
        if (lrc != GCUDA_OK) return fail(g, lrc, "the expert kernels' launch");
        RC_OK(norm(next_norm, true, next_hf, l));
    }
    return GCUDA_OK;
}

// The verify step for n tokens on g->st (toks in g->d_toks, the position in g->d_pos).
int enqueue_step(gcuda *g, int n) {
    const gcuda_shape &s = g->sh;
    const int H = s.hidden;
    const DevTensor *emb = tensor(g, g->embed, kRaw);
    if (g->ep_world > 1) RC_OK(enqueue_tick(g));   // (the step's epoch: every rank runs the same steps)
    {
        const dim3 grid((H + 255) / 256, n);
        LAUNCH_OK(launch_ex(k_embed, grid, dim3(256), 0, g->st, false, static_cast<const uint8_t *>(emb->d),
                            static_cast<int64_t>(s.vocab), H, emb->global, static_cast<const int *>(g->d_toks), n, g->x,
                            g->d_status));
    }
    RC_OK(enqueue_norm(g, n, g->x, raw_of(g, g->layers[0].in_norm), false, g->hf, 0, g->hq));
    const size_t xrows = static_cast<size_t>(n) * H;
    for (int l = 0; l < s.n_layers; ++l) {
        if (g->tr_x)
            LAUNCH_OK(cudaMemcpyAsync(g->tr_x + static_cast<size_t>(l) * xrows, g->x, xrows * sizeof(float),
                                      cudaMemcpyDeviceToDevice, g->st));
        const float *next_norm = l + 1 < s.n_layers ? raw_of(g, g->layers[static_cast<size_t>(l) + 1].in_norm)
                                                    : raw_of(g, g->final_norm);
        float *next_hf = l + 1 < s.n_layers ? g->hf : g->hid;
        RC_OK(enqueue_layer(g, n, l, g->layers[static_cast<size_t>(l)], g->plan[static_cast<size_t>(l)], g->d_pos,
                            next_norm, next_hf));
    }
    if (g->tr_x)
        LAUNCH_OK(cudaMemcpyAsync(g->tr_x + static_cast<size_t>(s.n_layers) * xrows, g->x, xrows * sizeof(float),
                                  cudaMemcpyDeviceToDevice, g->st));
    // the logits of every row (engine/src/model.cpp:5397-5410): hq holds rmsnorm(x, final_norm) quantized
    RC_OK(launch_units(g, g->lm_u, static_cast<int>((s.vocab + 31) / 32), g->hq, n, g->pdl));
    return GCUDA_OK;
}

// The MTP pass (Model::forward_mtp, engine/src/model.cpp:4965-5039, as its GPU branch runs it for Model::draft,
// engine/src/model.cpp:1368-1446) over n positions from *d_mtp_pos: the embeddings of the n next tokens
// (d_mtp_toks) and the n hidden rows (mtp_hin) each through its norm into one 2H-wide row, the fc product, the
// decoder layer over the MTP's own KV slot, mtp.norm (into mtp_hf), the last row's logits, their first maximum (the
// greedy draft) and softmax_at's probability of it.
int enqueue_mtp(gcuda *g, int n) {
    const gcuda_shape &s = g->sh;
    const int H = s.hidden;
    const DevTensor *emb = tensor(g, g->embed, kRaw);
    if (g->ep_world > 1) RC_OK(enqueue_tick(g));
    {
        const dim3 grid((H + 255) / 256, n);
        LAUNCH_OK(launch_ex(k_embed, grid, dim3(256), 0, g->st, false, static_cast<const uint8_t *>(emb->d),
                            static_cast<int64_t>(s.vocab), H, emb->global, static_cast<const int *>(g->d_mtp_toks), n,
                            g->x, g->d_status));
    }
    // [rmsnorm(e, pre_e) | rmsnorm(hidden, pre_h)] quantized as one 2H row (its 16-value blocks never straddle the
    // halves, so the two norms quantize their halves alone), then x = fc . that row
    RC_OK(enqueue_norm(g, n, g->x, raw_of(g, g->mtp_pre_e), false, nullptr, 0, g->mtp_in, 0));
    RC_OK(enqueue_norm(g, n, g->mtp_hin, raw_of(g, g->mtp_pre_h), false, nullptr, 0, g->mtp_in, H));
    RC_OK(launch_units(g, g->mtp_fc_u, (H + 31) / 32, g->mtp_in, n, g->pdl));
    RC_OK(enqueue_norm(g, n, g->x, raw_of(g, g->mtp_layer.in_norm), false, g->hf, 0, g->hq));
    RC_OK(enqueue_layer(g, n, s.n_layers, g->mtp_layer, g->mtp_plan, g->d_mtp_pos, raw_of(g, g->mtp_norm), g->mtp_hf));
    // the last row's logits: hq's row n - 1 holds rmsnorm(x, mtp.norm) quantized
    ActBuf last = g->hq;
    last.q += static_cast<size_t>(n - 1) * H;
    last.scale += static_cast<size_t>(n - 1) * (H / 16);
    last.bsum += static_cast<size_t>(n - 1) * (H / 16);
    last.n = 1;
    // (over the draft head's rows when a draft vocabulary is set: d_mtp_draft then holds the row, run_mtp maps it)
    const int rows = g->mtp_vocab;
    RC_OK(launch_units(g, g->mtp_lm_u, (rows + 31) / 32, last, 1, g->pdl));
    LAUNCH_OK(launch_ex(k_argmax_rows, dim3(argmax_slices(1, sm_count()), 1), dim3(kArgmaxThreads), 0, g->st, false,
                        static_cast<const float *>(g->mtp_logits), rows, g->d_mtp_best));
    LAUNCH_OK(launch_ex(k_argmax_finish, dim3(1), dim3(32), 0, g->st, false, g->d_mtp_best, 1, g->d_mtp_draft));
    LAUNCH_OK(launch_ex(k_softmax_at, dim3(kSoftmaxCtas), dim3(kSoftmaxThreads), 0, g->st, false,
                        static_cast<const float *>(g->mtp_logits), rows, static_cast<const int *>(g->d_mtp_draft),
                        g->mtp_part, g->mtp_count, g->mtp_prob));
    return GCUDA_OK;
}

int set_attrs(gcuda *g) {
    const gcuda_shape &s = g->sh;
    if (gemv_opt_in() != GCUDA_OK) return GCUDA_E_CUDA;
    LAUNCH_OK(cudaFuncSetAttribute(k_attn_decode<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(attn_smem_bytes<256>())));
    LAUNCH_OK(cudaFuncSetAttribute(k_attn_decode<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(attn_smem_bytes<128>())));
    LAUNCH_OK(cudaFuncSetAttribute(k_attn_decode<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(attn_smem_bytes<64>())));
    if (lane_opt_in(nullptr) != GCUDA_OK) return GCUDA_E_CUDA;
    (void)s;
    return GCUDA_OK;
}

int record_graphs(gcuda *g) {
    for (int n = 1; n <= g->sh.max_tokens; ++n) {
        cudaGraph_t graph = nullptr;
        LAUNCH_OK(cudaStreamBeginCapture(g->st, cudaStreamCaptureModeThreadLocal));
        const uint64_t k0 = launch_counter().load();
        const int rc = enqueue_step(g, n);
        g->graph_kernels[n] = launch_counter().load() - k0;
        launch_counter().fetch_sub(g->graph_kernels[n]);   // (recorded, not run)
        const cudaError_t e = cudaStreamEndCapture(g->st, &graph);
        if (rc != GCUDA_OK) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        if (e != cudaSuccess) return cuda_fail(g, e, "cudaStreamEndCapture");
        const cudaError_t ei = cudaGraphInstantiate(&g->graph[n], graph, 0);
        cudaGraphDestroy(graph);
        if (ei != cudaSuccess) return cuda_fail(g, ei, "cudaGraphInstantiate");
    }
    for (int n = 1; g->has_mtp && n <= g->sh.max_tokens; ++n) {
        cudaGraph_t graph = nullptr;
        LAUNCH_OK(cudaStreamBeginCapture(g->st, cudaStreamCaptureModeThreadLocal));
        const uint64_t k0 = launch_counter().load();
        const int rc = enqueue_mtp(g, n);
        g->mtp_graph_kernels[n] = launch_counter().load() - k0;
        launch_counter().fetch_sub(g->mtp_graph_kernels[n]);
        const cudaError_t e = cudaStreamEndCapture(g->st, &graph);
        if (rc != GCUDA_OK) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        if (e != cudaSuccess) return cuda_fail(g, e, "cudaStreamEndCapture");
        const cudaError_t ei = cudaGraphInstantiate(&g->mtp_graph[n], graph, 0);
        cudaGraphDestroy(graph);
        if (ei != cudaSuccess) return cuda_fail(g, ei, "cudaGraphInstantiate");
    }
    return GCUDA_OK;
}

// the status word's outcome once its copy in h_status has landed
int status_outcome(gcuda *g, uint32_t st) {
    if (st) {
        cudaMemsetAsync(g->d_status, 0, 4, g->st);
        std::string why;
        if (st & kErrWaitTimeout) why += " a bounded wait gave up;";
        if (st & kErrBadToken) why += " a token id out of range;";
        if (st & kErrBadShape) why += " a position past the context;";
        return fail(g, GCUDA_E_DEVICE, "device status" + why);
    }
    return GCUDA_OK;
}

int check_status(gcuda *g) {
    LAUNCH_OK(cudaMemcpyAsync(g->h_status, g->d_status, 4, cudaMemcpyDeviceToHost, g->st));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    return status_outcome(g, *g->h_status);
}

}  // namespace

extern "C" {

gcuda *gcuda_open(int device, char *err, int err_len) {
    auto put = [&](const std::string &m) {
        if (err && err_len > 0) {
            std::strncpy(err, m.c_str(), static_cast<size_t>(err_len - 1));
            err[err_len - 1] = 0;
        }
    };
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
        put("no CUDA device " + std::to_string(device));
        return nullptr;
    }
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, device);
    if (prop.major != 10) {
        put(std::string("not an sm_100 device: ") + prop.name);
        return nullptr;
    }
    auto *g = new gcuda;
    g->device = device;
    cudaSetDevice(device);
    if (cudaStreamCreateWithFlags(&g->st, cudaStreamNonBlocking) != cudaSuccess) {
        put("cudaStreamCreate failed");
        delete g;
        return nullptr;
    }
    cudaEventCreate(&g->ev0);
    cudaEventCreate(&g->ev1);
    if (cudaStreamCreateWithFlags(&g->st2, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&g->fork_ev, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&g->join_ev, cudaEventDisableTiming) != cudaSuccess) {
        put("side stream / events");
        gcuda_close(g);
        return nullptr;
    }
    if (!dalloc(g, &g->d_status, 1)) {
        put(g->err);
        gcuda_close(g);
        return nullptr;
    }
    if (cudaMallocHost(&g->h_status, sizeof(uint32_t)) != cudaSuccess) {
        put("cudaMallocHost");
        gcuda_close(g);
        return nullptr;
    }
    return g;
}

void gcuda_close(gcuda *g) {
    if (!g) return;
    cudaSetDevice(g->device);
    if (g->st) cudaStreamSynchronize(g->st);
    for (auto &ge : g->graph)
        if (ge) cudaGraphExecDestroy(ge);
    for (auto &ge : g->mtp_graph)
        if (ge) cudaGraphExecDestroy(ge);
    for (auto &t : g->tensors)
        if (t.d) cudaFree(t.d);
    for (auto &x : g->experts) {
        if (x.d) cudaFree(x.d);
        if (x.scales) cudaFree(x.scales);
    }
    for (void *p : g->allocs) cudaFree(p);
    if (g->rej) cudaFree(g->rej);
    if (g->d_seen) cudaFree(g->d_seen);
    if (g->h_status) cudaFreeHost(g->h_status);
    if (g->ev0) cudaEventDestroy(g->ev0);
    if (g->ev1) cudaEventDestroy(g->ev1);
    for (int r = 0; r < kMaxEpWorld; ++r)
        if (g->peer_base[r]) cudaIpcCloseMemHandle(g->peer_base[r]);
    if (g->xbuf) cudaFree(g->xbuf);
    if (g->comm) nccl().comm_destroy(g->comm);
    if (g->fork_ev) cudaEventDestroy(g->fork_ev);
    if (g->join_ev) cudaEventDestroy(g->join_ev);
    if (g->st2) cudaStreamDestroy(g->st2);
    if (g->st) cudaStreamDestroy(g->st);
    delete g;
}

int gcuda_ep_unique_id(void *id_out) {
    if (!id_out) return GCUDA_E_ARG;
    if (!nccl().ok) return GCUDA_E_CUDA;
    ncclUniqueId id;
    if (nccl().get_unique_id(&id) != ncclSuccess) return GCUDA_E_CUDA;
    std::memcpy(id_out, &id, sizeof id);
    return GCUDA_OK;
}

int gcuda_set_ep(gcuda *g, int rank, int world, const void *id) {
    if (!g || world < 1 || world > kMaxEpWorld || rank < 0 || rank >= world || (world > 1 && !id)) return GCUDA_E_ARG;
    if (g->ready) return fail(g, GCUDA_E_STATE, "set_ep: before gcuda_setup");
    if (g->comm) return fail(g, GCUDA_E_STATE, "set_ep: already set");
    g->ep_rank = rank;
    g->ep_world = world;
    if (world == 1) return GCUDA_OK;
    if (!nccl().ok) return fail(g, GCUDA_E_CUDA, "set_ep: libnccl.so.2 not found");
    cudaSetDevice(g->device);
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    const ncclResult_t r = nccl().comm_init_rank(&g->comm, world, uid, rank);
    if (r != ncclSuccess) {
        g->comm = nullptr;
        return fail(g, GCUDA_E_CUDA, std::string("ncclCommInitRank: ") + nccl().error_string(r));
    }
    return GCUDA_OK;
}

int gcuda_last_error(gcuda *g, char *buf, int len) {
    if (!g) return GCUDA_E_ARG;
    if (buf && len > 0) {
        std::strncpy(buf, g->err.c_str(), static_cast<size_t>(len - 1));
        buf[len - 1] = 0;
    }
    return g->err.empty() ? 0 : 1;
}

int gcuda_adopt_q4(gcuda *g, const uint8_t *data, int64_t rows, int64_t cols, size_t row_bytes, float global) {
    if (!g || !data || rows <= 0 || cols <= 0 || cols % 64 || row_bytes != static_cast<size_t>(cols / 16) * 9)
        return fail(g, GCUDA_E_ARG, "adopt_q4: a q4 [rows][cols] with cols a multiple of 64");
    cudaSetDevice(g->device);
    const size_t src_bytes = static_cast<size_t>(rows) * row_bytes;
    const size_t tiled = gcuda_op_q4_tiled_bytes(rows, cols);
    void *stage = nullptr, *dst = nullptr;
    cudaError_t e = cudaMalloc(&dst, tiled);
    if (e != cudaSuccess) return cuda_fail(g, e, "adopt_q4 cudaMalloc");
    e = cudaMalloc(&stage, src_bytes);
    if (e != cudaSuccess) {
        cudaFree(dst);
        return cuda_fail(g, e, "adopt_q4 cudaMalloc (staging)");
    }
    e = cudaMemcpyAsync(stage, data, src_bytes, cudaMemcpyHostToDevice, g->st);
    if (e == cudaSuccess && gcuda_op_q4_relayout(static_cast<uint8_t *>(stage), rows, cols, static_cast<uint8_t *>(dst), g->st) != 0)
        e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(g->st);
    cudaFree(stage);
    if (e != cudaSuccess) {
        cudaFree(dst);
        return cuda_fail(g, e, "adopt_q4");
    }
    DevTensor t;
    t.d = dst;
    t.bytes = tiled;
    t.rows = rows;
    t.cols = cols;
    t.global = global;
    t.kind = kQ4Tiled;
    g->tensors.push_back(t);
    return static_cast<int>(g->tensors.size()) - 1;
}

int gcuda_adopt_raw(gcuda *g, const void *data, size_t bytes) {
    if (!g || !data || bytes == 0) return fail(g, GCUDA_E_ARG, "adopt_raw: no data");
    cudaSetDevice(g->device);
    void *dst = nullptr;
    cudaError_t e = cudaMalloc(&dst, bytes);
    if (e != cudaSuccess) return cuda_fail(g, e, "adopt_raw cudaMalloc");
    e = cudaMemcpy(dst, data, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(dst);
        return cuda_fail(g, e, "adopt_raw");
    }
    DevTensor t;
    t.d = dst;
    t.bytes = bytes;
    t.kind = kRaw;
    g->tensors.push_back(t);
    return static_cast<int>(g->tensors.size()) - 1;
}

// Internal: the embedding keeps the pack's row layout (rows are gathered, not streamed) with its global.
int gcuda_adopt_embedding(gcuda *g, const uint8_t *data, int64_t rows, int64_t cols, float global) {
    const int id = gcuda_adopt_raw(g, data, static_cast<size_t>(rows) * static_cast<size_t>(cols / 16) * 9);
    if (id >= 0) {
        g->tensors[static_cast<size_t>(id)].rows = rows;
        g->tensors[static_cast<size_t>(id)].cols = cols;
        g->tensors[static_cast<size_t>(id)].global = global;
    }
    return id;
}

int gcuda_adopt_experts(gcuda *g, const uint8_t *blocks, int n, size_t stride, const float *scales) {
    if (!g || !blocks || n <= 0 || !scales) return fail(g, GCUDA_E_ARG, "adopt_experts: no data");
    cudaSetDevice(g->device);
    DevExperts X;
    X.n = n;
    X.stride = stride;
    X.host_scales.assign(scales, scales + 2 * n);
    cudaError_t e = cudaMalloc(&X.d, static_cast<size_t>(n) * stride);
    if (e != cudaSuccess) return cuda_fail(g, e, "adopt_experts cudaMalloc");
    e = cudaMalloc(&X.scales, sizeof(float) * 2 * n);
    if (e == cudaSuccess) e = cudaMemcpy(X.scales, scales, sizeof(float) * 2 * n, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(X.d);
        return cuda_fail(g, e, "adopt_experts");
    }
    // the blocks stay raw until gcuda_setup knows hidden and ff (then each is relaid in place: see setup)
    e = cudaMemcpy(X.d, blocks, static_cast<size_t>(n) * stride, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(g, e, "adopt_experts copy");
    g->experts.push_back(X);
    return static_cast<int>(g->experts.size()) - 1;
}

// The exchange buffer of expert parallelism: this rank's [flags | eout] in one allocation (so one IPC handle maps it),
// the handles of every rank gathered through NCCL, the peers' buffers opened here. Flags [n_layers + 2][world]: a row
// per layer's exchange (the MTP layer's after the model's) and the step-start row; eout a slot of `slot_floats` per
// layer.
int ep_exchange_setup(gcuda *g, size_t slot_floats) {
    const int W = g->ep_world;
    const size_t fbytes = (static_cast<size_t>(g->sh.n_layers + 2) * W * sizeof(uint32_t) + 255) / 256 * 256;
    const size_t bytes = fbytes + static_cast<size_t>(g->sh.n_layers + 1) * slot_floats * sizeof(float);
    g->eout_stride = slot_floats;
    if (cudaMalloc(&g->xbuf, bytes) != cudaSuccess) {
        g->xbuf = nullptr;
        return fail(g, GCUDA_E_MEMORY, "ep exchange buffer: cudaMalloc");
    }
    LAUNCH_OK(cudaMemset(g->xbuf, 0, bytes));
    g->xflags = static_cast<uint32_t *>(g->xbuf);
    g->eout = reinterpret_cast<float *>(static_cast<uint8_t *>(g->xbuf) + fbytes);
    if (!dalloc(g, &g->ep_epoch, 1) || !dalloc(g, &g->xcount, 1)) return GCUDA_E_MEMORY;
    LAUNCH_OK(cudaMemset(g->ep_epoch, 0, sizeof(int)));
    LAUNCH_OK(cudaMemset(g->xcount, 0, sizeof(unsigned int)));
    cudaIpcMemHandle_t mine;
    LAUNCH_OK(cudaIpcGetMemHandle(&mine, g->xbuf));
    void *d_h = nullptr;
    if (cudaMalloc(&d_h, sizeof(cudaIpcMemHandle_t) * (W + 1)) != cudaSuccess) return fail(g, GCUDA_E_MEMORY, "cudaMalloc");
    std::vector<cudaIpcMemHandle_t> all(static_cast<size_t>(W));
    uint8_t *d_mine = static_cast<uint8_t *>(d_h) + sizeof(cudaIpcMemHandle_t) * W;
    cudaError_t e = cudaMemcpy(d_mine, &mine, sizeof mine, cudaMemcpyHostToDevice);
    ncclResult_t nr = ncclSuccess;
    if (e == cudaSuccess) nr = nccl().all_gather(d_mine, d_h, sizeof mine, ncclUint8, g->comm, g->st);
    if (e == cudaSuccess && nr == ncclSuccess) e = cudaStreamSynchronize(g->st);
    if (e == cudaSuccess && nr == ncclSuccess) e = cudaMemcpy(all.data(), d_h, sizeof(cudaIpcMemHandle_t) * W, cudaMemcpyDeviceToHost);
    cudaFree(d_h);
    if (nr != ncclSuccess) return fail(g, GCUDA_E_CUDA, std::string("ncclAllGather: ") + nccl().error_string(nr));
    LAUNCH_OK(e);
    for (int r = 0; r < W; ++r) {
        if (r == g->ep_rank) continue;
        void *p = nullptr;
        const cudaError_t eo = cudaIpcOpenMemHandle(&p, all[static_cast<size_t>(r)], cudaIpcMemLazyEnablePeerAccess);
        if (eo != cudaSuccess) return cuda_fail(g, eo, "cudaIpcOpenMemHandle (a peer's exchange buffer)");
        g->peer_base[r] = p;
        g->peer_flags[r] = static_cast<uint32_t *>(p);
        g->peer_eout[r] = reinterpret_cast<float *>(static_cast<uint8_t *>(p) + fbytes);
    }
    return GCUDA_OK;
}

int gcuda_setup(gcuda *g, const gcuda_shape *shape, const gcuda_layer *layers, int embed, int lm_head, int final_norm) {
    if (!g || !shape || !layers) return fail(g, GCUDA_E_ARG, "setup: no shape");
    if (g->ready) return fail(g, GCUDA_E_STATE, "setup: already set up");
    cudaSetDevice(g->device);
    const gcuda_shape &s = *shape;
    if (s.max_tokens < 1 || s.max_tokens > kMaxTok || s.hidden % 64 || s.hidden > kNormThreads * kNormPer ||
        s.n_layers <= 0 || s.context <= 0 ||
        (!s.dense && (s.top_k < 1 || s.top_k > 8 || s.n_experts > 1024 || s.moe_ff % 64 || s.shared_ff % 64)) ||
        (s.dense && s.shared_ff % 64) || s.head_dim % 64 || (s.head_dim != 64 && s.head_dim != 128 && s.head_dim != 256) ||
        s.n_heads % std::max(1, s.n_kv_heads) || s.max_tokens * (s.n_heads / std::max(1, s.n_kv_heads)) > 32)
        return fail(g, GCUDA_E_ARG, "setup: an unsupported geometry");
    g->sh = s;
    g->layers.assign(layers, layers + s.n_layers);
    g->embed = embed;
    g->lm_head = lm_head;
    g->final_norm = final_norm;
    const int H = s.hidden, T = s.max_tokens;
    g->kd = s.gdn_k_heads * s.gdn_k_dim;
    g->vd = s.gdn_v_heads * s.gdn_v_dim;
    g->conv_dim = 2 * g->kd + g->vd;
    g->qw = s.n_heads * 2 * s.head_dim;
    g->kvrow = s.n_kv_heads * s.head_dim;
    g->corew = std::max(g->vd, s.n_heads * s.head_dim);
    for (const auto &L : g->layers) (L.attn ? g->n_attn : g->n_gdn)++;
    if (g->n_gdn && (s.gdn_v_dim % 16 || s.gdn_v_dim / 16 > 8 || (s.gdn_k_dim != 32 && s.gdn_k_dim != 64 && s.gdn_k_dim != 128) ||
                     s.gdn_v_heads % std::max(1, s.gdn_k_heads) || s.conv_kernel < 1 || s.conv_kernel > 9))
        return fail(g, GCUDA_E_ARG, "setup: an unsupported Gated DeltaNet geometry");
    // the routed experts relaid into tiles, block by block: [gate_up tiles][down tiles], the same bytes
    if (!s.dense) {
        const size_t want = static_cast<size_t>(2 * s.moe_ff) * (H / 16) * 9 + static_cast<size_t>(H) * (s.moe_ff / 16) * 9;
        for (auto &X : g->experts) {
            if (X.stride != want) return fail(g, GCUDA_E_ARG, "setup: an expert block of unexpected size");
            if (X.r16) continue;
            uint8_t *tmp = nullptr;
            const size_t all = static_cast<size_t>(X.n) * X.stride;
            cudaError_t e = cudaMalloc(&tmp, X.tiled ? all : X.stride);
            if (e != cudaSuccess) return cuda_fail(g, e, "setup cudaMalloc");
            const size_t gu_tiled = gcuda_op_q4_tiled_bytes(2 * s.moe_ff, H);
            if (!X.tiled) {   // the pack's rows -> tiles, block by block
                for (int i = 0; i < X.n; ++i) {
                    uint8_t *blk = X.d + static_cast<size_t>(i) * X.stride;
                    cudaMemcpyAsync(tmp, blk, X.stride, cudaMemcpyDeviceToDevice, g->st);
                    gcuda_op_q4_relayout(tmp, 2 * s.moe_ff, H, blk, g->st);
                    gcuda_op_q4_relayout(tmp + static_cast<size_t>(2 * s.moe_ff) * (H / 16) * 9, H, s.moe_ff, blk + gu_tiled,
                                         g->st);
                }
                e = cudaStreamSynchronize(g->st);
                cudaFree(tmp);
                tmp = nullptr;
                if (e == cudaSuccess) e = cudaMalloc(&tmp, all);
                if (e != cudaSuccess) return cuda_fail(g, e, "setup relayout experts");
            }
            // tiles -> R16, the layout the expert kernels read: every block of the layer in two launches
            cudaMemcpyAsync(tmp, X.d, all, cudaMemcpyDeviceToDevice, g->st);
            const int64_t gt = 2 * s.moe_ff / 16, dt = H / 16;
            k_relayout_r16<<<relayout_grid(gt * (H / 64) * 16 * X.n), 256, 0, g->st>>>(tmp, gt, H, X.d, X.n, X.stride);
            k_relayout_r16<<<relayout_grid(dt * (s.moe_ff / 64) * 16 * X.n), 256, 0, g->st>>>(tmp + gu_tiled, dt, s.moe_ff,
                                                                                            X.d + gu_tiled, X.n, X.stride);
            e = cudaStreamSynchronize(g->st);
            cudaFree(tmp);
            if (e != cudaSuccess) return cuda_fail(g, e, "setup relayout experts");
            X.tiled = X.r16 = true;
        }
        if (s.shared_ff != s.moe_ff)
            return fail(g, GCUDA_E_ARG, "setup: the shared expert's width must equal the routed experts'");
        // the shared experts' matrices (read only by the expert kernels in a MoE model) to R16 too, each tensor once
        std::vector<char> done(g->tensors.size(), 0);
        auto to_r16 = [&](int id) -> int {
            const DevTensor *t = tensor(g, id, kQ4Tiled);
            if (!t || done[static_cast<size_t>(id)]) return GCUDA_OK;
            done[static_cast<size_t>(id)] = 1;
            if (t->rows % 16 || t->cols % 64) return fail(g, GCUDA_E_ARG, "setup: a shared expert matrix's shape");
            uint8_t *tmp = nullptr;
            cudaError_t e = cudaMalloc(&tmp, t->bytes);
            if (e != cudaSuccess) return cuda_fail(g, e, "setup cudaMalloc");
            cudaMemcpyAsync(tmp, t->d, t->bytes, cudaMemcpyDeviceToDevice, g->st);
            const int64_t tiles = t->rows / 16;
            k_relayout_r16<<<relayout_grid(tiles * (t->cols / 64) * 16), 256, 0, g->st>>>(
                tmp, tiles, static_cast<int>(t->cols), static_cast<uint8_t *>(t->d));
            e = cudaStreamSynchronize(g->st);
            cudaFree(tmp);
            return e == cudaSuccess ? GCUDA_OK : cuda_fail(g, e, "setup relayout the shared expert");
        };
        for (const gcuda_layer &L : g->layers) {
            RC_OK(to_r16(L.sh_gate));
            RC_OK(to_r16(L.sh_up));
            RC_OK(to_r16(L.sh_down));
        }
        if (g->has_mtp) {
            RC_OK(to_r16(g->mtp_layer.sh_gate));
            RC_OK(to_r16(g->mtp_layer.sh_up));
            RC_OK(to_r16(g->mtp_layer.sh_down));
        }
    }
    // state
    g->conv_n = static_cast<size_t>(g->n_gdn) * g->conv_dim * std::max(0, s.conv_kernel - 1);
    g->gdn_n = static_cast<size_t>(g->n_gdn) * s.gdn_v_heads * s.gdn_v_dim * s.gdn_k_dim;
    const int kv_slots = g->n_attn + (g->has_mtp ? 1 : 0);   // (the MTP layer's slot after the model's)
    const size_t kv = static_cast<size_t>(kv_slots) * s.context * g->kvrow;
    const size_t kvs = static_cast<size_t>(kv_slots) * s.context * s.n_kv_heads;
    g->nchunks = (s.context + kAttnChunk - 1) / kAttnChunk;
    const int E = s.dense ? 0 : s.n_experts, K = s.dense ? 1 : s.top_k;
    const int ffw = s.dense ? 64 : s.moe_ff;
    if (!dalloc(g, &g->conv, g->conv_n) || !dalloc(g, &g->gdn, g->gdn_n) ||
        !dalloc(g, &g->conv_bk, g->conv_n * (T - 1 > 0 ? T - 1 : 1)) || !dalloc(g, &g->gdn_bk, g->gdn_n * (T - 1 > 0 ? T - 1 : 1)) ||
        !dalloc(g, &g->kc, kv) || !dalloc(g, &g->vc, kv) || !dalloc(g, &g->ks, kvs) || !dalloc(g, &g->vs, kvs) ||
        !dalloc(g, &g->d_toks, kMaxTok) || !dalloc(g, &g->d_pos, 1) || !dalloc(g, &g->x, static_cast<size_t>(T) * H) ||
        !dalloc(g, &g->hf, static_cast<size_t>(T) * H) || !dalloc(g, &g->hid, static_cast<size_t>(T) * H) ||
        !dalloc(g, &g->big, static_cast<size_t>(T) * std::max(g->conv_dim, g->qw)) ||
        !dalloc(g, &g->zb, static_cast<size_t>(T) * std::max(1, g->vd)) ||
        !dalloc(g, &g->convd, static_cast<size_t>(T) * std::max(1, g->conv_dim)) ||
        !dalloc(g, &g->ab, static_cast<size_t>(T) * std::max(1, 2 * s.gdn_v_heads)) ||
        !dalloc(g, &g->kb, static_cast<size_t>(T) * g->kvrow) || !dalloc(g, &g->vb, static_cast<size_t>(T) * g->kvrow) ||
        !dalloc(g, &g->qn, static_cast<size_t>(T) * s.n_heads * s.head_dim) ||
        !dalloc(g, &g->rlog, static_cast<size_t>(T) * (E + 1)) ||
        (g->ep_world == 1 && !dalloc(g, &g->eout, static_cast<size_t>(T) * K * H)) ||
        !dalloc(g, &g->shout, static_cast<size_t>(T) * H) ||
        !dalloc(g, &g->part, static_cast<size_t>(T) * s.n_heads * g->nchunks * (s.head_dim + 2)) ||
        !dalloc(g, &g->logits, static_cast<size_t>(T) * s.vocab) || !dalloc(g, &g->core_f, static_cast<size_t>(T) * g->corew) ||
        !dalloc(g, &g->inv_freq, std::max(1, s.rope_dim / 2)) || !dalloc(g, &g->route, 1) ||
        !dalloc(g, &g->d_u, kMaxTok) || !dalloc(g, &g->d_samples, kMaxTok) || !dalloc(g, &g->step, 1) || !dalloc(g, &g->d_best, kMaxTok) ||
        !dalloc(g, &g->d_rej_step, 2) ||
        !act_alloc(g, g->hq, T, H) || !act_alloc(g, g->core, T, g->corew) ||
        !act_alloc(g, g->amid, T * K, ffw) || !act_alloc(g, g->shact, T, s.shared_ff))
        return GCUDA_E_MEMORY;
    if (g->ep_world > 1) RC_OK(ep_exchange_setup(g, static_cast<size_t>(T) * K * H));
    if (g->has_mtp &&
        (!act_alloc(g, g->mtp_in, T, 2 * H) || !dalloc(g, &g->mtp_hin, static_cast<size_t>(T) * H) ||
         !dalloc(g, &g->mtp_hf, static_cast<size_t>(T) * H) ||
         !dalloc(g, &g->mtp_logits, g->draft_ids.empty() ? s.vocab : g->draft_ids.size()) ||
         !dalloc(g, &g->mtp_prob, 1) || !dalloc(g, &g->mtp_part, kSoftmaxCtas) || !dalloc(g, &g->mtp_count, 1) ||
         !dalloc(g, &g->d_mtp_toks, kMaxTok) || !dalloc(g, &g->d_mtp_pos, 1) || !dalloc(g, &g->d_mtp_draft, 1) ||
         !dalloc(g, &g->d_mtp_best, 1)))
        return GCUDA_E_MEMORY;
    // inv_freq as the reference computes it (engine/src/model.cpp:737-740), host powf
    {
        std::vector<float> inv(static_cast<size_t>(std::max(1, s.rope_dim / 2)));
        for (int i = 0; i < s.rope_dim / 2; ++i)
            inv[static_cast<size_t>(i)] = 1.0f / std::pow(s.rope_theta, static_cast<float>(2 * i) / static_cast<float>(s.rope_dim));
        cudaMemcpy(g->inv_freq, inv.data(), inv.size() * sizeof(float), cudaMemcpyHostToDevice);
    }
    // the unit tables and the small merged weight buffers
    std::vector<GemvUnit> U;
    g->plan.assign(static_cast<size_t>(s.n_layers), LayerPlan{});
    int gi = 0, ai = 0;
    auto q4 = [&](int id) { return tensor(g, id, kQ4Tiled); };
    auto build = [&](const gcuda_layer &L, LayerPlan &P, const std::string &name) -> int {
        if (!tensor(g, L.in_norm, kRaw) || !tensor(g, L.post_norm, kRaw))
            return fail(g, GCUDA_E_ARG, "setup: layer " + name + " lacks its norms");
        if (!L.attn) {
            P.gi = gi++;
            const DevTensor *qkv = q4(L.qkv), *z = q4(L.z), *out = q4(L.out);
            const DevTensor *a = tensor(g, L.a, kRaw), *b = tensor(g, L.b, kRaw);
            if (!qkv || !z || !out || !a || !b || !tensor(g, L.conv, kRaw) || !tensor(g, L.A_log, kRaw) ||
                !tensor(g, L.dt_bias, kRaw) || !tensor(g, L.gnorm, kRaw) || qkv->rows != g->conv_dim || z->rows != g->vd ||
                out->rows != H || out->cols != g->vd)
                return fail(g, GCUDA_E_ARG, "setup: GDN layer " + name + " tensors");
            P.u_in = static_cast<int>(U.size());
            plain_units(U, *qkv, g->big, g->conv_dim, kStore);
            plain_units(U, *z, g->zb, g->vd, kStore);
            P.n_in = static_cast<int>(U.size()) - P.u_in;
            P.u_out = static_cast<int>(U.size());
            plain_units(U, *out, g->x, H, kAccumulate);
            P.n_out = static_cast<int>(U.size()) - P.u_out;
            if (!dalloc(g, &P.ab_w, static_cast<size_t>(2 * s.gdn_v_heads) * H)) return GCUDA_E_MEMORY;
            cudaMemcpy(P.ab_w, a->d, a->bytes, cudaMemcpyDeviceToDevice);
            cudaMemcpy(P.ab_w + static_cast<size_t>(s.gdn_v_heads) * H, b->d, b->bytes, cudaMemcpyDeviceToDevice);
        } else {
            P.ai = ai++;
            const DevTensor *q = q4(L.q), *k = q4(L.k), *v = q4(L.v), *o = q4(L.o);
            if (!q || !k || !v || !o || !tensor(g, L.q_norm, kRaw) || !tensor(g, L.k_norm, kRaw) || q->rows != g->qw ||
                k->rows != g->kvrow || v->rows != g->kvrow || o->rows != H || o->cols != s.n_heads * s.head_dim)
                return fail(g, GCUDA_E_ARG, "setup: attention layer " + name + " tensors");
            P.u_in = static_cast<int>(U.size());
            plain_units(U, *q, g->big, g->qw, kStore);
            plain_units(U, *k, g->kb, g->kvrow, kStore);
            plain_units(U, *v, g->vb, g->kvrow, kStore);
            P.n_in = static_cast<int>(U.size()) - P.u_in;
            P.u_out = static_cast<int>(U.size());
            plain_units(U, *o, g->x, H, kAccumulate);
            P.n_out = static_cast<int>(U.size()) - P.u_out;
        }
        const DevTensor *sg = q4(L.sh_gate), *su = q4(L.sh_up), *sd = q4(L.sh_down);
        if (!sg || !su || !sd || sg->rows != s.shared_ff || su->rows != s.shared_ff || sd->rows != H)
            return fail(g, GCUDA_E_ARG, "setup: layer " + name + " MLP tensors");
        if (s.dense) {
            P.u_mlp = static_cast<int>(U.size());
            swiglu_units(U, *sg, *su, g->shact);
            P.n_mlp = static_cast<int>(U.size()) - P.u_mlp;
            P.u_dn = static_cast<int>(U.size());
            plain_units(U, *sd, g->x, H, kAccumulate);
            P.n_dn = static_cast<int>(U.size()) - P.u_dn;
        } else {
            const DevTensor *r = tensor(g, L.router, kRaw), *gt = tensor(g, L.shared_gate, kRaw);
            if (!r || !gt || L.experts < 0 || L.experts >= static_cast<int>(g->experts.size()) ||
                g->experts[static_cast<size_t>(L.experts)].n != s.n_experts)
                return fail(g, GCUDA_E_ARG, "setup: MoE layer " + name + " tensors");
            if (!dalloc(g, &P.router_w, static_cast<size_t>(s.n_experts + 1) * H)) return GCUDA_E_MEMORY;
            cudaMemcpy(P.router_w, r->d, r->bytes, cudaMemcpyDeviceToDevice);
            cudaMemcpy(P.router_w + static_cast<size_t>(s.n_experts) * H, gt->d, gt->bytes, cudaMemcpyDeviceToDevice);
        }
        return GCUDA_OK;
    };
    for (int l = 0; l < s.n_layers; ++l)
        RC_OK(build(g->layers[static_cast<size_t>(l)], g->plan[static_cast<size_t>(l)], std::to_string(l)));
    if (g->has_mtp) {
        // the MTP layer: attention slot n_attn (its KV after the model's), the fc [H][2H], its norms
        if (!g->mtp_layer.attn) return fail(g, GCUDA_E_ARG, "setup: the MTP layer is no attention layer");
        RC_OK(build(g->mtp_layer, g->mtp_plan, "mtp"));
        const DevTensor *fc = q4(g->mtp_fc);
        if (!fc || fc->rows != H || fc->cols != 2 * H || !tensor(g, g->mtp_pre_e, kRaw) || !tensor(g, g->mtp_pre_h, kRaw) ||
            !tensor(g, g->mtp_norm, kRaw))
            return fail(g, GCUDA_E_ARG, "setup: the MTP layer's fc / norms");
        g->mtp_fc_u = static_cast<int>(U.size());
        plain_units(U, *fc, g->x, H, kStore);
    }
    const DevTensor *head = q4(lm_head);
    if (!head || head->rows != s.vocab || !tensor(g, final_norm, kRaw) || !tensor(g, embed, kRaw))
        return fail(g, GCUDA_E_ARG, "setup: lm_head / norm / embedding");
    g->lm_u = static_cast<int>(U.size());
    plain_units(U, *head, g->logits, s.vocab, kStore);
    if (g->has_mtp) {
        // the MTP pass's head: lm_head, or the draft head (its rows the draft vocabulary's, a multiple of 32)
        const DevTensor *dh = head;
        g->mtp_vocab = s.vocab;
        if (!g->draft_ids.empty()) {
            dh = q4(g->draft_head);
            bool ok = dh && dh->rows == static_cast<int64_t>(g->draft_ids.size()) && dh->cols == H &&
                      dh->global == head->global;
            for (const int id : g->draft_ids) ok = ok && id >= 0 && id < s.vocab;
            if (!ok) return fail(g, GCUDA_E_ARG, "setup: the draft head (lm_head's rows of the draft vocabulary)");
            g->mtp_vocab = static_cast<int>(g->draft_ids.size());
        }
        g->mtp_lm_u = static_cast<int>(U.size());
        plain_units(U, *dh, g->mtp_logits, g->mtp_vocab, kStore);
    }
    g->n_units = static_cast<int>(U.size());
    if (!dalloc(g, &g->units, U.size())) return GCUDA_E_MEMORY;
    cudaMemcpy(g->units, U.data(), U.size() * sizeof(GemvUnit), cudaMemcpyHostToDevice);
    RC_OK(set_attrs(g));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    RC_OK(record_graphs(g));
    g->ready = true;
    g->pos = 0;
    return GCUDA_OK;
}

namespace {
// the step's graph for n tokens already in d_toks at the handle's position, and the status word's copy behind it
int enqueue_verify(gcuda *g, int n) {
    LAUNCH_OK(cudaMemcpyAsync(g->d_pos, &g->pos, sizeof(int), cudaMemcpyHostToDevice, g->st));
    LAUNCH_OK(cudaEventRecord(g->ev0, g->st));
    LAUNCH_OK(cudaGraphLaunch(g->graph[n], g->st));
    count_launch(g->graph_kernels[n]);
    LAUNCH_OK(cudaEventRecord(g->ev1, g->st));
    LAUNCH_OK(cudaMemcpyAsync(g->h_status, g->d_status, 4, cudaMemcpyDeviceToHost, g->st));
    return GCUDA_OK;
}
}  // namespace

int gcuda_verify_device(gcuda *g, const int *d_toks, int n) {
    if (!g || !g->ready) return fail(g, GCUDA_E_STATE, "verify before setup");
    if (n < 1 || n > g->sh.max_tokens) return fail(g, GCUDA_E_ARG, "a verified batch of " + std::to_string(n) + " tokens");
    if (g->pos + n > g->sh.context) return fail(g, GCUDA_E_ARG, "the context is full");
    cudaSetDevice(g->device);
    if (d_toks != g->d_toks) LAUNCH_OK(cudaMemcpyAsync(g->d_toks, d_toks, sizeof(int) * n, cudaMemcpyDeviceToDevice, g->st));
    RC_OK(enqueue_verify(g, n));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    RC_OK(status_outcome(g, *g->h_status));
    cudaEventElapsedTime(&g->last_ms, g->ev0, g->ev1);
    LAUNCH_OK(cudaMemcpy(g->last_toks, g->d_toks, sizeof(int) * n, cudaMemcpyDeviceToHost));
    g->pos += n;
    g->last_batch = n;
    g->hid_rows = n;
    return GCUDA_OK;
}

int gcuda_verify(gcuda *g, const int *toks, int n, float *logits, float *hidden) {
    if (!g || !g->ready) return fail(g, GCUDA_E_STATE, "verify before setup");
    if (!toks || n < 1 || n > g->sh.max_tokens) return fail(g, GCUDA_E_ARG, "a verified batch of " + std::to_string(n) + " tokens");
    if (g->pos + n > g->sh.context) return fail(g, GCUDA_E_ARG, "the context is full");
    // every token's embedding row exists before anything runs (engine/src/model.cpp:1551-1555): a bad id is an error
    // that leaves the conversation as it was
    for (int t = 0; t < n; ++t)
        if (toks[t] < 0 || toks[t] >= g->sh.vocab)
            return fail(g, GCUDA_E_ARG, "cannot read the embedding of token " + std::to_string(toks[t]));
    cudaSetDevice(g->device);
    // the tokens in, the graph, the status word and the outputs back, then one synchronization
    LAUNCH_OK(cudaMemcpyAsync(g->d_toks, toks, sizeof(int) * n, cudaMemcpyHostToDevice, g->st));
    RC_OK(enqueue_verify(g, n));
    if (logits) LAUNCH_OK(cudaMemcpyAsync(logits, g->logits, sizeof(float) * n * g->sh.vocab, cudaMemcpyDeviceToHost, g->st));
    if (hidden) LAUNCH_OK(cudaMemcpyAsync(hidden, g->hid, sizeof(float) * n * g->sh.hidden, cudaMemcpyDeviceToHost, g->st));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    RC_OK(status_outcome(g, *g->h_status));
    cudaEventElapsedTime(&g->last_ms, g->ev0, g->ev1);
    std::memcpy(g->last_toks, toks, sizeof(int) * n);
    g->pos += n;
    g->last_batch = n;
    g->hid_rows = n;
    return GCUDA_OK;
}

int gcuda_set_mtp(gcuda *g, int fc, int pre_e, int pre_h, int norm, const gcuda_layer *layer) {
    if (!g || !layer) return fail(g, GCUDA_E_ARG, "set_mtp: no layer");
    if (g->ready) return fail(g, GCUDA_E_STATE, "set_mtp: after setup");
    if (!layer->attn) return fail(g, GCUDA_E_ARG, "set_mtp: the MTP layer is an attention layer");
    g->has_mtp = true;
    g->mtp_fc = fc;
    g->mtp_pre_e = pre_e;
    g->mtp_pre_h = pre_h;
    g->mtp_norm = norm;
    g->mtp_layer = *layer;
    return GCUDA_OK;
}

int gcuda_set_draft_head(gcuda *g, int head, const int *ids, int n) {
    if (!g) return GCUDA_E_ARG;
    if (g->ready) return fail(g, GCUDA_E_STATE, "set_draft_head: after setup");
    if (!ids || n < 32 || n % 32) return fail(g, GCUDA_E_ARG, "set_draft_head: a draft vocabulary of whole tiles (32 rows)");
    g->draft_head = head;
    g->draft_ids.assign(ids, ids + n);
    return GCUDA_OK;
}

int gcuda_draft_rows(gcuda *g) { return g && g->ready && g->has_mtp ? g->mtp_vocab : GCUDA_E_STATE; }

namespace {
// one MTP pass of n rows (its inputs in place): the captured pass, then the draft, its probability and the logits
int run_mtp(gcuda *g, int n, int *draft, float *prob, float *logits) {
    LAUNCH_OK(cudaGraphLaunch(g->mtp_graph[n], g->st));
    count_launch(g->mtp_graph_kernels[n]);
    RC_OK(check_status(g));
    g->mtp_rows = n;
    LAUNCH_OK(cudaMemcpyAsync(draft, g->d_mtp_draft, sizeof(int), cudaMemcpyDeviceToHost, g->st));
    if (prob) LAUNCH_OK(cudaMemcpyAsync(prob, g->mtp_prob, sizeof(float), cudaMemcpyDeviceToHost, g->st));
    if (logits)
        LAUNCH_OK(cudaMemcpyAsync(logits, g->mtp_logits, sizeof(float) * g->mtp_vocab, cudaMemcpyDeviceToHost, g->st));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    // a draft head's row -> its token (engine/src/model.cpp:1409, 1473)
    if (!g->draft_ids.empty()) {
        if (*draft < 0 || *draft >= static_cast<int>(g->draft_ids.size())) return fail(g, GCUDA_E_DEVICE, "draft: no row");
        *draft = g->draft_ids[static_cast<size_t>(*draft)];
    }
    return GCUDA_OK;
}

int mtp_checks(gcuda *g, const int *toks, int n, int pos, int *draft) {
    if (!g || !g->ready) return fail(g, GCUDA_E_STATE, "draft before setup");
    if (!g->has_mtp) return fail(g, GCUDA_E_STATE, "draft: no MTP layer (gcuda_set_mtp before gcuda_setup)");
    if (!toks || !draft || n < 1 || n > g->sh.max_tokens || pos < 0 || pos + n > g->sh.context)
        return fail(g, GCUDA_E_ARG, "bad draft");
    for (int t = 0; t < n; ++t)
        if (toks[t] < 0 || toks[t] >= g->sh.vocab)
            return fail(g, GCUDA_E_ARG, "cannot read the embedding of token " + std::to_string(toks[t]));
    return GCUDA_OK;
}
}  // namespace

int gcuda_draft(gcuda *g, const int *toks, int n, int pos, const float *hidden, int *draft, float *prob, float *logits) {
    RC_OK(mtp_checks(g, toks, n, pos, draft));
    if (!hidden && n > g->hid_rows)
        return fail(g, GCUDA_E_STATE, "draft: the device holds fewer than " + std::to_string(n) +
                                          " hidden rows of the conversation (the last verified batch's, as kept)");
    cudaSetDevice(g->device);
    const size_t rows = static_cast<size_t>(n) * g->sh.hidden * sizeof(float);
    LAUNCH_OK(cudaMemcpyAsync(g->d_mtp_toks, toks, sizeof(int) * n, cudaMemcpyHostToDevice, g->st));
    LAUNCH_OK(cudaMemcpyAsync(g->d_mtp_pos, &pos, sizeof(int), cudaMemcpyHostToDevice, g->st));
    if (hidden) LAUNCH_OK(cudaMemcpyAsync(g->mtp_hin, hidden, rows, cudaMemcpyHostToDevice, g->st));
    else LAUNCH_OK(cudaMemcpyAsync(g->mtp_hin, g->hid, rows, cudaMemcpyDeviceToDevice, g->st));
    return run_mtp(g, n, draft, prob, logits);
}

int gcuda_draft_next(gcuda *g, int tok, int pos, int *draft, float *prob, float *logits) {
    RC_OK(mtp_checks(g, &tok, 1, pos, draft));
    if (g->mtp_rows < 1) return fail(g, GCUDA_E_STATE, "draft_next without a draft before it");
    cudaSetDevice(g->device);
    const size_t H = static_cast<size_t>(g->sh.hidden);
    LAUNCH_OK(cudaMemcpyAsync(g->d_mtp_toks, &tok, sizeof(int), cudaMemcpyHostToDevice, g->st));
    LAUNCH_OK(cudaMemcpyAsync(g->d_mtp_pos, &pos, sizeof(int), cudaMemcpyHostToDevice, g->st));
    LAUNCH_OK(cudaMemcpyAsync(g->mtp_hin, g->mtp_hf + (g->mtp_rows - 1) * H, H * sizeof(float), cudaMemcpyDeviceToDevice,
                              g->st));
    return run_mtp(g, 1, draft, prob, logits);
}

int gcuda_spec_reject(gcuda *g, const float *d_target, const float *d_draft, const int *drafts, int S, int k, int V,
                      const gcuda_sampling *sp, uint64_t seed, int *accepted, int *next) {
    if (!g) return GCUDA_E_ARG;
    if (!d_target || !d_draft || !drafts || !sp || !accepted || !next || S < 1 || k < 1 || V < 1 || sp->temperature <= 0.0f ||
        sp->top_k > kMaxCand || !(sp->top_p > 0.0f && sp->top_p <= 1.0f))
        return fail(g, GCUDA_E_ARG, "spec_reject: bad arguments");
    cudaSetDevice(g->device);
    const size_t need = static_cast<size_t>(S) * (k + 2);
    if (need > g->rej_cap) {
        if (g->rej) cudaFree(g->rej);
        g->rej = nullptr;
        g->rej_cap = 0;
        if (cudaMalloc(&g->rej, need * sizeof(int)) != cudaSuccess) return fail(g, GCUDA_E_MEMORY, "spec_reject: cudaMalloc");
        g->rej_cap = need;
    }
    int *d_drafts = g->rej, *d_acc = g->rej + static_cast<size_t>(S) * k, *d_next = d_acc + S;
    LAUNCH_OK(cudaMemcpyAsync(d_drafts, drafts, sizeof(int) * S * k, cudaMemcpyHostToDevice, g->st));
    RejectArgs a{};
    a.target = d_target;
    a.draft = d_draft;
    a.drafts = d_drafts;
    a.k = k;
    a.V = V;
    a.temperature = sp->temperature;
    a.top_p = sp->top_p;
    a.top_k = sp->top_k;
    a.seed = seed;
    a.accepted = d_acc;
    a.next = d_next;
    LAUNCH_OK(launch_ex(k_spec_reject, dim3(S), dim3(kSampleThreads), 0, g->st, false, a));
    LAUNCH_OK(cudaMemcpyAsync(accepted, d_acc, sizeof(int) * S, cudaMemcpyDeviceToHost, g->st));
    LAUNCH_OK(cudaMemcpyAsync(next, d_next, sizeof(int) * S, cudaMemcpyDeviceToHost, g->st));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    return GCUDA_OK;
}

int gcuda_accept(gcuda *g, const gcuda_sampling *sp, const double *uniforms, const int *stops, int n_stops,
                 const int *seen, int n_seen, int *kept, int *next, int *samples) {
    if (!g || !g->ready) return fail(g, GCUDA_E_STATE, "accept before setup");
    if (!sp || !kept || !next || g->last_batch < 1) return fail(g, GCUDA_E_STATE, "accept without a verified batch");
    cudaSetDevice(g->device);
    const int n = g->last_batch;
    const bool greedy = sp->temperature <= 0.0f;
    if (!greedy && !uniforms) return fail(g, GCUDA_E_ARG, "accept: sampling needs the uniforms");
    if (sp->presence_penalty != 0.0f) {
        // engine/src/geode.cpp:234-255: the list holds each sampled id once; the drafts new to it are marked fresh
        const int V = g->sh.vocab;
        if (n_seen < 0 || (n_seen > 0 && !seen)) return fail(g, GCUDA_E_ARG, "accept: a bad seen list");
        g->seen_mark.resize(static_cast<size_t>(V), 0);
        PresenceArgs pa{};
        bool ok = true;
        for (int i = 0; i < n_seen && ok; ++i) {
            const int t = seen[i];
            ok = t >= 0 && t < V && !g->seen_mark[static_cast<size_t>(t)];
            if (ok) g->seen_mark[static_cast<size_t>(t)] = 1;
        }
        for (int j = 1; j < n && ok; ++j) {
            const int t = g->last_toks[j];
            pa.toks[j] = t;
            if (!g->seen_mark[static_cast<size_t>(t)]) {
                g->seen_mark[static_cast<size_t>(t)] = 1;
                pa.fresh |= 1u << j;
            }
        }
        for (int i = 0; i < n_seen; ++i)   // (the marks back to zero, as far as they were set)
            if (seen[i] >= 0 && seen[i] < V) g->seen_mark[static_cast<size_t>(seen[i])] = 0;
        for (int j = 1; j < n; ++j) g->seen_mark[static_cast<size_t>(g->last_toks[j])] = 0;
        if (!ok) return fail(g, GCUDA_E_ARG, "accept: the seen list holds an id twice or one outside the vocabulary");
        if (static_cast<size_t>(n_seen) > g->seen_cap) {
            LAUNCH_OK(cudaStreamSynchronize(g->st));
            if (g->d_seen) cudaFree(g->d_seen);
            g->d_seen = nullptr;
            g->seen_cap = 0;
            const size_t cap = std::max<size_t>(1024, static_cast<size_t>(n_seen));
            if (cudaMalloc(&g->d_seen, cap * sizeof(int)) != cudaSuccess) return fail(g, GCUDA_E_MEMORY, "accept: cudaMalloc");
            g->seen_cap = cap;
        }
        if (n_seen > 0)
            LAUNCH_OK(cudaMemcpyAsync(g->d_seen, seen, sizeof(int) * n_seen, cudaMemcpyHostToDevice, g->st));
        pa.logits = g->logits;
        pa.V = V;
        pa.n = n;
        pa.penalty = sp->presence_penalty;
        pa.seen = g->d_seen;
        pa.n_seen = n_seen;
        const int slices = std::max(1, std::min(64, (n_seen + 255) / 256));
        LAUNCH_OK(launch_ex(k_presence, dim3(slices, n), dim3(256), 0, g->st, false, pa));
    }
    if (!greedy) LAUNCH_OK(cudaMemcpyAsync(g->d_u, uniforms, sizeof(double) * n, cudaMemcpyHostToDevice, g->st));
    SampleArgs a{};
    a.logits = g->logits;
    a.V = g->sh.vocab;
    a.n = n;
    a.temperature = sp->temperature;
    a.top_p = sp->top_p;
    a.top_k = sp->top_k;
    a.u = g->d_u;
    a.out = g->d_samples;
    if (greedy) {
        LAUNCH_OK(launch_ex(k_argmax_rows, dim3(argmax_slices(n, sm_count()), n), dim3(kArgmaxThreads), 0, g->st, false,
                            static_cast<const float *>(g->logits), g->sh.vocab, g->d_best));
        LAUNCH_OK(launch_ex(k_argmax_finish, dim3(1), dim3(32), 0, g->st, false, g->d_best, n, g->d_samples));
    } else {
        LAUNCH_OK(launch_ex(k_sample_rows, dim3(n), dim3(kSampleThreads), 0, g->st, false, a));
    }
    int ys[kMaxTok];
    LAUNCH_OK(cudaMemcpyAsync(ys, g->d_samples, sizeof(int) * n, cudaMemcpyDeviceToHost, g->st));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    // engine/src/geode.cpp:327-350: draft i+1 stands while row i's sample is that draft and no stop token
    int k = 1, nx = -1;
    for (int i = 0; i < n; ++i) {
        bool stop = false;
        for (int j = 0; j < n_stops && stops; ++j) stop |= stops[j] == ys[i];
        if (i + 1 < n && ys[i] == g->last_toks[i + 1] && !stop) {
            ++k;
            continue;
        }
        nx = ys[i];
        break;
    }
    *kept = k;
    *next = nx;
    // the loop samples rows 0 .. kept-1 (the last of them ends it); the rows after were never drawn
    if (samples)
        for (int i = 0; i < n; ++i) samples[i] = i < k ? ys[i] : -1;
    return GCUDA_OK;
}

int gcuda_keep(gcuda *g, int kept) {
    if (!g || !g->ready) return fail(g, GCUDA_E_STATE, "keep before setup");
    if (kept < 1 || kept >= g->last_batch)
        return fail(g, GCUDA_E_ARG, "keeping " + std::to_string(kept) + " of a batch of " + std::to_string(g->last_batch));
    cudaSetDevice(g->device);
    const size_t b = static_cast<size_t>(kept - 1);
    if (g->conv_n)
        LAUNCH_OK(cudaMemcpyAsync(g->conv, g->conv_bk + b * g->conv_n, g->conv_n * sizeof(float), cudaMemcpyDeviceToDevice, g->st));
    if (g->gdn_n)
        LAUNCH_OK(cudaMemcpyAsync(g->gdn, g->gdn_bk + b * g->gdn_n, g->gdn_n * sizeof(float), cudaMemcpyDeviceToDevice, g->st));
    // (no wait: every later use of the states is ordered behind these copies on the handle's stream, and the calls
    // that hand data to the host synchronize it)
    g->pos -= g->last_batch - kept;
    g->last_batch = 0;
    g->hid_rows = kept;
    return GCUDA_OK;
}

int gcuda_position(gcuda *g) { return g ? g->pos : GCUDA_E_ARG; }

int gcuda_reset(gcuda *g) {
    if (!g || !g->ready) return fail(g, GCUDA_E_STATE, "reset before setup");
    cudaSetDevice(g->device);
    if (g->conv_n) cudaMemsetAsync(g->conv, 0, g->conv_n * sizeof(float), g->st);
    if (g->gdn_n) cudaMemsetAsync(g->gdn, 0, g->gdn_n * sizeof(float), g->st);
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    g->pos = 0;
    g->last_batch = 0;
    g->hid_rows = 0;
    g->reject_steps = 0;   // the device-side rejection sampler's Philox sequence starts over with the conversation
    g->mtp_rows = 0;
    return GCUDA_OK;
}

const float *gcuda_device_logits(gcuda *g) { return g ? g->logits : nullptr; }
float gcuda_last_ms(gcuda *g) { return g ? g->last_ms : 0.0f; }
uint64_t gcuda_launches(gcuda *) { return launch_counter().load(); }

// state bridge: the reference's layouts <-> the device's ([vh][dv][dk] recurrent states, [pos][nkv][hd] KV)
int gcuda_state_get(gcuda *g, float *conv, float *gdn, int8_t *kv, float *kv_scale, int positions) {
    if (!g || !g->ready || positions < 0 || positions > g->sh.context) return fail(g, GCUDA_E_ARG, "state_get");
    cudaSetDevice(g->device);
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    const gcuda_shape &s = g->sh;
    if (conv && g->conv_n) LAUNCH_OK(cudaMemcpy(conv, g->conv, g->conv_n * sizeof(float), cudaMemcpyDeviceToHost));
    if (gdn && g->gdn_n) {
        std::vector<float> d(g->gdn_n);
        LAUNCH_OK(cudaMemcpy(d.data(), g->gdn, g->gdn_n * sizeof(float), cudaMemcpyDeviceToHost));
        const int nv = s.gdn_v_heads, dv = s.gdn_v_dim, dk = s.gdn_k_dim;
        for (size_t l = 0; l < static_cast<size_t>(g->n_gdn); ++l)
            for (int h = 0; h < nv; ++h)
                for (int j = 0; j < dv; ++j)
                    for (int i = 0; i < dk; ++i) {
                        const size_t src = ((l * nv + h) * dv + j) * dk + i;
                        const size_t dst = (l * nv + h) * static_cast<size_t>(dv) * dk + static_cast<size_t>(j / 16) * dk * 16 +
                                           static_cast<size_t>(i) * 16 + (j % 16);
                        gdn[dst] = d[src];
                    }
    }
    // (the model's attention layers, then the MTP layer's slot when it has one, as the engine's cache orders them)
    const size_t row = g->kvrow, nkv = s.n_kv_heads;
    for (int a = 0; a < g->n_attn + (g->has_mtp ? 1 : 0) && positions > 0; ++a) {
        const size_t base = static_cast<size_t>(a) * s.context;
        if (kv) {
            LAUNCH_OK(cudaMemcpy(kv + (static_cast<size_t>(a) * 2 + 0) * positions * row, g->kc + base * row, positions * row, cudaMemcpyDeviceToHost));
            LAUNCH_OK(cudaMemcpy(kv + (static_cast<size_t>(a) * 2 + 1) * positions * row, g->vc + base * row, positions * row, cudaMemcpyDeviceToHost));
        }
        if (kv_scale) {
            LAUNCH_OK(cudaMemcpy(kv_scale + (static_cast<size_t>(a) * 2 + 0) * positions * nkv, g->ks + base * nkv, positions * nkv * 4, cudaMemcpyDeviceToHost));
            LAUNCH_OK(cudaMemcpy(kv_scale + (static_cast<size_t>(a) * 2 + 1) * positions * nkv, g->vs + base * nkv, positions * nkv * 4, cudaMemcpyDeviceToHost));
        }
    }
    return GCUDA_OK;
}

int gcuda_state_put(gcuda *g, const float *conv, const float *gdn, const int8_t *kv, const float *kv_scale, int pos) {
    if (!g || !g->ready || pos < 0 || pos > g->sh.context) return fail(g, GCUDA_E_ARG, "state_put");
    cudaSetDevice(g->device);
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    const gcuda_shape &s = g->sh;
    if (conv && g->conv_n) LAUNCH_OK(cudaMemcpy(g->conv, conv, g->conv_n * sizeof(float), cudaMemcpyHostToDevice));
    if (gdn && g->gdn_n) {
        std::vector<float> d(g->gdn_n);
        const int nv = s.gdn_v_heads, dv = s.gdn_v_dim, dk = s.gdn_k_dim;
        for (size_t l = 0; l < static_cast<size_t>(g->n_gdn); ++l)
            for (int h = 0; h < nv; ++h)
                for (int j = 0; j < dv; ++j)
                    for (int i = 0; i < dk; ++i)
                        d[((l * nv + h) * dv + j) * dk + i] =
                            gdn[(l * nv + h) * static_cast<size_t>(dv) * dk + static_cast<size_t>(j / 16) * dk * 16 +
                                static_cast<size_t>(i) * 16 + (j % 16)];
        LAUNCH_OK(cudaMemcpy(g->gdn, d.data(), g->gdn_n * sizeof(float), cudaMemcpyHostToDevice));
    }
    const size_t row = g->kvrow, nkv = s.n_kv_heads;
    for (int a = 0; a < g->n_attn + (g->has_mtp ? 1 : 0) && pos > 0; ++a) {
        const size_t base = static_cast<size_t>(a) * s.context;
        if (kv) {
            LAUNCH_OK(cudaMemcpy(g->kc + base * row, kv + (static_cast<size_t>(a) * 2 + 0) * pos * row, pos * row, cudaMemcpyHostToDevice));
            LAUNCH_OK(cudaMemcpy(g->vc + base * row, kv + (static_cast<size_t>(a) * 2 + 1) * pos * row, pos * row, cudaMemcpyHostToDevice));
        }
        if (kv_scale) {
            LAUNCH_OK(cudaMemcpy(g->ks + base * nkv, kv_scale + (static_cast<size_t>(a) * 2 + 0) * pos * nkv, pos * nkv * 4, cudaMemcpyHostToDevice));
            LAUNCH_OK(cudaMemcpy(g->vs + base * nkv, kv_scale + (static_cast<size_t>(a) * 2 + 1) * pos * nkv, pos * nkv * 4, cudaMemcpyHostToDevice));
        }
    }
    g->pos = pos;
    g->last_batch = 0;
    g->hid_rows = 0;
    return GCUDA_OK;
}

int gcuda_last_hidden(gcuda *g, float *out) {
    if (!g || !g->ready || !out) return fail(g, GCUDA_E_ARG, "last_hidden");
    if (g->hid_rows < 1) return fail(g, GCUDA_E_STATE, "last_hidden: no hidden row of the conversation on the device");
    cudaSetDevice(g->device);
    const size_t H = static_cast<size_t>(g->sh.hidden);
    LAUNCH_OK(cudaMemcpyAsync(out, g->hid + static_cast<size_t>(g->hid_rows - 1) * H, H * sizeof(float),
                              cudaMemcpyDeviceToHost, g->st));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    return GCUDA_OK;
}

int gcuda_put_last_hidden(gcuda *g, const float *row) {
    if (!g || !g->ready || !row) return fail(g, GCUDA_E_ARG, "put_last_hidden");
    if (g->pos < 1) return fail(g, GCUDA_E_STATE, "put_last_hidden: an empty conversation");
    cudaSetDevice(g->device);
    LAUNCH_OK(cudaMemcpyAsync(g->hid, row, static_cast<size_t>(g->sh.hidden) * sizeof(float), cudaMemcpyHostToDevice, g->st));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    g->hid_rows = 1;
    return GCUDA_OK;
}

// Tests: the device copies of the last step's intermediate rows (what: 0 x [n][H], 1 hf, 2 core_f, 3 route, 4 hid)
int gcuda_debug_read(gcuda *g, int what, void *out, size_t bytes) {
    if (!g || !g->ready) return GCUDA_E_STATE;
    cudaSetDevice(g->device);
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    const void *src = what == 0 ? static_cast<const void *>(g->x) : what == 1 ? g->hf : what == 2 ? g->core_f
                      : what == 3 ? static_cast<const void *>(g->route) : what == 4 ? g->hid : what == 5 ? g->convd
                      : what == 6 ? g->ab : what == 7 ? g->zb : g->big;
    LAUNCH_OK(cudaMemcpy(out, src, bytes, cudaMemcpyDeviceToHost));
    return GCUDA_OK;
}

// Tests / measuring: launch the step without the graph (every kernel on the stream, PDL as configured)
int gcuda_debug_step_eager(gcuda *g, const int *toks, int n, int pdl) {
    if (!g || !g->ready || n < 1 || n > g->sh.max_tokens) return GCUDA_E_ARG;
    cudaSetDevice(g->device);
    LAUNCH_OK(cudaMemcpyAsync(g->d_toks, toks, sizeof(int) * n, cudaMemcpyHostToDevice, g->st));
    LAUNCH_OK(cudaMemcpyAsync(g->d_pos, &g->pos, sizeof(int), cudaMemcpyHostToDevice, g->st));
    const bool keep = g->pdl;
    g->pdl = pdl != 0;
    const int rc = enqueue_step(g, n);
    g->pdl = keep;
    if (rc != GCUDA_OK) return rc;
    RC_OK(check_status(g));
    g->pos += n;
    g->last_batch = n;
    g->hid_rows = n;
    return GCUDA_OK;
}

// Tests: one eager step with per-layer copies (the reference's LayerTrace, engine/src/model.hpp:92-105): x, the
// router's logits and its routing per layer; the step otherwise as gcuda_verify's (position and batch advance).
int gcuda_debug_trace(gcuda *g, const int *toks, int n, float *x, float *router_logits, int *ids, float *weights,
                      float *gate, int *n_union) {
    if (!g || !g->ready || !toks || !x || n < 1 || n > g->sh.max_tokens) return GCUDA_E_ARG;
    const gcuda_shape &s = g->sh;
    if (g->pos + n > s.context) return fail(g, GCUDA_E_ARG, "trace: past the context");
    for (int i = 0; i < n; ++i)
        if (toks[i] < 0 || toks[i] >= s.vocab) return fail(g, GCUDA_E_ARG, "trace: a token id out of range");
    cudaSetDevice(g->device);
    const bool moe = !s.dense && s.n_experts > 0;
    const size_t L = static_cast<size_t>(s.n_layers), H = static_cast<size_t>(s.hidden), E1 = static_cast<size_t>(s.n_experts) + 1;
    const size_t xbytes = (L + 1) * n * H * sizeof(float), rbytes = L * n * E1 * sizeof(float);
    void *bx = nullptr, *br = nullptr, *bt = nullptr;
    if (cudaMalloc(&bx, xbytes) != cudaSuccess ||
        (moe && (cudaMalloc(&br, rbytes) != cudaSuccess || cudaMalloc(&bt, L * sizeof(RouteOut)) != cudaSuccess))) {
        cudaFree(bx);
        cudaFree(br);
        return fail(g, GCUDA_E_MEMORY, "trace: cudaMalloc");
    }
    g->tr_x = static_cast<float *>(bx);
    g->tr_rlog = static_cast<float *>(br);
    g->tr_route = static_cast<RouteOut *>(bt);
    int rc = GCUDA_OK;
    if (cudaMemcpyAsync(g->d_toks, toks, sizeof(int) * n, cudaMemcpyHostToDevice, g->st) != cudaSuccess ||
        cudaMemcpyAsync(g->d_pos, &g->pos, sizeof(int), cudaMemcpyHostToDevice, g->st) != cudaSuccess)
        rc = GCUDA_E_CUDA;
    if (rc == GCUDA_OK) rc = enqueue_step(g, n);
    if (rc == GCUDA_OK) rc = check_status(g);
    std::vector<RouteOut> ro(moe ? L : 0);
    if (rc == GCUDA_OK && (cudaMemcpy(x, bx, xbytes, cudaMemcpyDeviceToHost) != cudaSuccess ||
                           (moe && cudaMemcpy(ro.data(), bt, L * sizeof(RouteOut), cudaMemcpyDeviceToHost) != cudaSuccess) ||
                           (moe && router_logits && cudaMemcpy(router_logits, br, rbytes, cudaMemcpyDeviceToHost) != cudaSuccess)))
        rc = GCUDA_E_CUDA;
    g->tr_x = nullptr;
    g->tr_rlog = nullptr;
    g->tr_route = nullptr;
    cudaFree(bx);
    cudaFree(br);
    cudaFree(bt);
    if (rc != GCUDA_OK) return rc;
    const int K = s.top_k;
    for (size_t l = 0; l < ro.size(); ++l) {
        for (int t = 0; t < n; ++t) {
            for (int k = 0; k < K; ++k) {
                if (ids) ids[(l * n + t) * K + k] = ro[l].ids[t * K + k];
                if (weights) weights[(l * n + t) * K + k] = ro[l].w[t * K + k];
            }
            if (gate) gate[l * n + t] = ro[l].gs[t];
        }
        if (n_union) n_union[l] = ro[l].n_union;
    }
    std::memcpy(g->last_toks, toks, sizeof(int) * n);
    g->pos += n;
    g->last_batch = n;
    g->hid_rows = n;
    return GCUDA_OK;
}

// Tests / measuring: `reps` eager steps of the same n tokens at the same position (no PDL, so an event pair brackets
// each launch), the device time of each timed kind summed over the steps.
int gcuda_debug_kernel_times(gcuda *g, const int *toks, int n, int reps, float *ms, int *launches, float *step_ms,
                             int *union_sum) {
    if (!g || !g->ready || !toks || !ms || !launches || n < 1 || n > g->sh.max_tokens || reps < 1) return GCUDA_E_ARG;
    if (g->pos + n > g->sh.context) return fail(g, GCUDA_E_ARG, "kernel_times: past the context");
    cudaSetDevice(g->device);
    gcuda::KernelMarks marks;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    LAUNCH_OK(cudaEventCreate(&e0));
    LAUNCH_OK(cudaEventCreate(&e1));
    for (int k = 0; k < kKtKinds; ++k) ms[k] = 0.0f, launches[k] = 0;
    float total = 0.0f;
    int u0 = 0, u1 = 0;
    LAUNCH_OK(cudaMemcpy(&u0, &g->step->n_union_sum, sizeof(int), cudaMemcpyDeviceToHost));
    const bool keep_pdl = g->pdl;
    g->pdl = false;
    int rc = GCUDA_OK;
    for (int r = 0; r < reps && rc == GCUDA_OK; ++r) {
        marks.marks.clear();
        marks.used = 0;
        g->kt = &marks;
        if (cudaMemcpyAsync(g->d_toks, toks, sizeof(int) * n, cudaMemcpyHostToDevice, g->st) != cudaSuccess ||
            cudaMemcpyAsync(g->d_pos, &g->pos, sizeof(int), cudaMemcpyHostToDevice, g->st) != cudaSuccess ||
            cudaEventRecord(e0, g->st) != cudaSuccess)
            rc = GCUDA_E_CUDA;
        if (rc == GCUDA_OK) rc = enqueue_step(g, n);
        g->kt = nullptr;
        if (rc == GCUDA_OK && (cudaEventRecord(e1, g->st) != cudaSuccess || cudaStreamSynchronize(g->st) != cudaSuccess))
            rc = GCUDA_E_CUDA;
        if (rc != GCUDA_OK) break;
        float t = 0.0f;
        cudaEventElapsedTime(&t, e0, e1);
        total += t;
        for (const auto &m : marks.marks) {
            float d = 0.0f;
            cudaEventElapsedTime(&d, marks.pool[static_cast<size_t>(m.second)], marks.pool[static_cast<size_t>(m.second) + 1]);
            ms[m.first] += d;
            ++launches[m.first];
        }
    }
    g->pdl = keep_pdl;
    if (rc == GCUDA_OK) rc = check_status(g);
    if (rc == GCUDA_OK && cudaMemcpy(&u1, &g->step->n_union_sum, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = GCUDA_E_CUDA;
    for (cudaEvent_t e : marks.pool) cudaEventDestroy(e);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc != GCUDA_OK) return rc;
    for (int k = 0; k < kKtKinds; ++k) ms[k] /= static_cast<float>(reps), launches[k] /= reps;
    if (step_ms) *step_ms = total / static_cast<float>(reps);
    if (union_sum) *union_sum = (u1 - u0) / reps;
    g->last_batch = 0;   // (the steps ran at the same position: nothing to accept or keep)
    g->hid_rows = 0;
    return GCUDA_OK;
}

// ------------------------------------------------------------------------------------------- synthetic weights ----
namespace {
int grid_for(size_t work) { return static_cast<int>(std::min<size_t>((work + 255) / 256, 148 * 64)); }
}  // namespace

int gcuda_synth_q4(gcuda *g, int64_t rows, int64_t cols, float global, uint64_t seed) {
    if (!g || rows <= 0 || cols % 64) return fail(g, GCUDA_E_ARG, "synth_q4: cols a multiple of 64");
    cudaSetDevice(g->device);
    const size_t bytes = gcuda_op_q4_tiled_bytes(rows, cols);
    void *d = nullptr;
    cudaError_t e = cudaMalloc(&d, bytes);
    if (e != cudaSuccess) return cuda_fail(g, e, "synth_q4 cudaMalloc");
    k_synth_tiled<<<grid_for(bytes / 8), 256, 0, g->st>>>(static_cast<uint8_t *>(d), bytes, seed);
    count_launch();
    DevTensor t;
    t.d = d;
    t.bytes = bytes;
    t.rows = rows;
    t.cols = cols;
    t.global = global;
    t.kind = kQ4Tiled;
    g->tensors.push_back(t);
    return static_cast<int>(g->tensors.size()) - 1;
}

int gcuda_synth_raw(gcuda *g, size_t count, int dtype, float mean, float stdv, uint64_t seed) {
    if (!g || count == 0 || dtype < 0 || dtype > 1) return fail(g, GCUDA_E_ARG, "synth_raw");
    cudaSetDevice(g->device);
    void *d = nullptr;
    const size_t bytes = count * (dtype == 0 ? 4 : 2);
    cudaError_t e = cudaMalloc(&d, bytes);
    if (e != cudaSuccess) return cuda_fail(g, e, "synth_raw cudaMalloc");
    k_synth_values<<<grid_for(count), 256, 0, g->st>>>(d, count, dtype, mean, stdv, seed);
    count_launch();
    DevTensor t;
    t.d = d;
    t.bytes = bytes;
    t.kind = kRaw;
    g->tensors.push_back(t);
    return static_cast<int>(g->tensors.size()) - 1;
}

int gcuda_synth_embedding(gcuda *g, int64_t rows, int64_t cols, float global, uint64_t seed) {
    if (!g || rows <= 0 || cols % 16) return fail(g, GCUDA_E_ARG, "synth_embedding");
    cudaSetDevice(g->device);
    const size_t bytes = static_cast<size_t>(rows) * (cols / 16) * 9;
    void *d = nullptr;
    cudaError_t e = cudaMalloc(&d, bytes);
    if (e != cudaSuccess) return cuda_fail(g, e, "synth_embedding cudaMalloc");
    k_synth_rows<<<grid_for(bytes), 256, 0, g->st>>>(static_cast<uint8_t *>(d), rows, static_cast<int>(cols), seed);
    count_launch();
    DevTensor t;
    t.d = d;
    t.bytes = bytes;
    t.rows = rows;
    t.cols = cols;
    t.global = global;
    t.kind = kRaw;
    g->tensors.push_back(t);
    return static_cast<int>(g->tensors.size()) - 1;
}

int gcuda_synth_experts(gcuda *g, int n, int hidden, int ff, float global, uint64_t seed) {
    if (!g || n <= 0 || hidden % 64 || ff % 64) return fail(g, GCUDA_E_ARG, "synth_experts");
    cudaSetDevice(g->device);
    DevExperts X;
    X.n = n;
    X.tiled = true;
    X.stride = static_cast<size_t>(2 * ff) * (hidden / 16) * 9 + static_cast<size_t>(hidden) * (ff / 16) * 9;
    X.host_scales.assign(static_cast<size_t>(2 * n), global);
    cudaError_t e = cudaMalloc(&X.d, static_cast<size_t>(n) * X.stride);
    if (e != cudaSuccess) return cuda_fail(g, e, "synth_experts cudaMalloc");
    e = cudaMalloc(&X.scales, sizeof(float) * 2 * n);
    if (e == cudaSuccess) e = cudaMemcpy(X.scales, X.host_scales.data(), sizeof(float) * 2 * n, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(g, e, "synth_experts");
    k_synth_tiled<<<grid_for(static_cast<size_t>(n) * X.stride / 8), 256, 0, g->st>>>(X.d, static_cast<size_t>(n) * X.stride, seed);
    count_launch();
    g->experts.push_back(X);
    return static_cast<int>(g->experts.size()) - 1;
}

int gcuda_state_randomize(gcuda *g, int pos, uint64_t seed) {
    if (!g || !g->ready || pos < 0 || pos > g->sh.context) return fail(g, GCUDA_E_ARG, "state_randomize");
    cudaSetDevice(g->device);
    const gcuda_shape &s = g->sh;
    for (int a = 0; a < g->n_attn; ++a) {
        const size_t base = static_cast<size_t>(a) * s.context;
        const size_t rows = static_cast<size_t>(pos) * g->kvrow, sc = static_cast<size_t>(pos) * s.n_kv_heads;
        k_synth_kv<<<grid_for(rows), 256, 0, g->st>>>(g->kc + base * g->kvrow, rows, g->ks + base * s.n_kv_heads, sc, 0.5f, seed + 2 * a);
        k_synth_kv<<<grid_for(rows), 256, 0, g->st>>>(g->vc + base * g->kvrow, rows, g->vs + base * s.n_kv_heads, sc, 0.5f, seed + 2 * a + 1);
        count_launch(2);
    }
    if (g->conv_n) k_synth_values<<<grid_for(g->conv_n), 256, 0, g->st>>>(g->conv, g->conv_n, 0, 0.0f, 0.3f, seed ^ 0xC0);
    if (g->gdn_n) k_synth_values<<<grid_for(g->gdn_n), 256, 0, g->st>>>(g->gdn, g->gdn_n, 0, 0.0f, 0.02f, seed ^ 0xD0);
    count_launch(2);
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    g->pos = pos;
    g->last_batch = 0;
    g->hid_rows = 0;
    return GCUDA_OK;
}

// The device-resident speculative step, enqueued without waiting: the verify graph for n tokens at the device
// position, the greedy acceptance of every row (k_argmax_rows, k_argmax_finish), the decision (k_decide: kept, next,
// position += kept, toks[0] = next) and the rollback of the Gated DeltaNet states (k_rollback). The drafts
// toks[1..n-1] stay those of the first batch (gcuda_begin_device_loop); gcuda_sync_step reads the decision and the
// position back.
int gcuda_step_device(gcuda *g, int n) {
    if (!g || !g->ready || n < 2 || n > g->sh.max_tokens) return fail(g, GCUDA_E_ARG, "step_device: 2 .. max_tokens");
    cudaSetDevice(g->device);
    LAUNCH_OK(cudaGraphLaunch(g->graph[n], g->st));
    count_launch(g->graph_kernels[n]);
    // greedy: every row's argmax (the reference's Sampler at temperature 0)
    LAUNCH_OK(launch_ex(k_argmax_rows, dim3(argmax_slices(n, sm_count()), n), dim3(kArgmaxThreads), 0, g->st, false,
                        static_cast<const float *>(g->logits), g->sh.vocab, g->d_best));
    LAUNCH_OK(launch_ex(k_argmax_finish, dim3(1), dim3(32), 0, g->st, g->pdl, g->d_best, n, g->d_samples));
    LAUNCH_OK(launch_ex(k_decide, dim3(1), dim3(32), 0, g->st, g->pdl, static_cast<const int *>(g->d_samples), g->d_toks, n,
                        g->d_pos, g->step));
    LAUNCH_OK(launch_ex(k_rollback, dim3(sm_count() * 4), dim3(256), 0, g->st, g->pdl, g->conv,
                        static_cast<const float *>(g->conv_bk), g->conv_n, g->gdn, static_cast<const float *>(g->gdn_bk),
                        g->gdn_n, n, static_cast<const StepState *>(g->step)));
    return GCUDA_OK;
}

// The same step with speculative (rejection) sampling in place of the greedy rule: k_spec_reject on the verified rows
// against the draft model's rows d_draft [n-1][V] (on the device), the drafts toks[1..n-1]; Philox key = seed plus
// the handle's count of these steps times a constant (fresh uniforms every step); then the decision and the rollback.
int gcuda_step_device_reject(gcuda *g, int n, const float *d_draft, const gcuda_sampling *sp, uint64_t seed) {
    if (!g || !g->ready || n < 2 || n > g->sh.max_tokens) return fail(g, GCUDA_E_ARG, "step_device_reject: 2 .. max_tokens");
    if (!d_draft || !sp || sp->temperature <= 0.0f || sp->top_k > kMaxCand || !(sp->top_p > 0.0f && sp->top_p <= 1.0f))
        return fail(g, GCUDA_E_ARG, "step_device_reject: bad arguments");
    cudaSetDevice(g->device);
    LAUNCH_OK(cudaGraphLaunch(g->graph[n], g->st));
    count_launch(g->graph_kernels[n]);
    RejectArgs a{};
    a.target = g->logits;
    a.draft = d_draft;
    a.drafts = g->d_toks + 1;
    a.k = n - 1;
    a.V = g->sh.vocab;
    a.temperature = sp->temperature;
    a.top_p = sp->top_p;
    a.top_k = sp->top_k;
    a.seed = seed + 0x9E3779B97F4A7C15ull * g->reject_steps++;
    a.accepted = g->d_rej_step;
    a.next = g->d_rej_step + 1;
    LAUNCH_OK(launch_ex(k_spec_reject, dim3(1), dim3(kSampleThreads), 0, g->st, false, a));
    LAUNCH_OK(launch_ex(k_decide_reject, dim3(1), dim3(32), 0, g->st, g->pdl, static_cast<const int *>(g->d_rej_step),
                        static_cast<const int *>(g->d_rej_step + 1), g->d_toks, g->d_pos, g->step));
    LAUNCH_OK(launch_ex(k_rollback, dim3(sm_count() * 4), dim3(256), 0, g->st, g->pdl, g->conv,
                        static_cast<const float *>(g->conv_bk), g->conv_n, g->gdn, static_cast<const float *>(g->gdn_bk),
                        g->gdn_n, n, static_cast<const StepState *>(g->step)));
    return GCUDA_OK;
}

// Before a device loop: the position to the device, the batch's tokens (n), the counters zeroed.
int gcuda_begin_device_loop(gcuda *g, const int *toks, int n) {
    if (!g || !g->ready || !toks || n < 1 || n > g->sh.max_tokens) return fail(g, GCUDA_E_ARG, "begin_device_loop");
    cudaSetDevice(g->device);
    LAUNCH_OK(cudaMemcpyAsync(g->d_toks, toks, sizeof(int) * n, cudaMemcpyHostToDevice, g->st));
    LAUNCH_OK(cudaMemcpyAsync(g->d_pos, &g->pos, sizeof(int), cudaMemcpyHostToDevice, g->st));
    LAUNCH_OK(cudaMemsetAsync(g->step, 0, sizeof(StepState), g->st));
    LAUNCH_OK(cudaStreamSynchronize(g->st));
    return GCUDA_OK;
}

// After a device loop: the position back to the host; steps, the expert-union sum over the routed layers and the
// last kept count.
int gcuda_sync_step(gcuda *g, int *steps, int *union_sum, int *last_kept) {
    if (!g || !g->ready) return fail(g, GCUDA_E_STATE, "sync_step");
    cudaSetDevice(g->device);
    StepState ss{};
    LAUNCH_OK(cudaMemcpyAsync(&ss, g->step, sizeof(ss), cudaMemcpyDeviceToHost, g->st));
    LAUNCH_OK(cudaMemcpyAsync(&g->pos, g->d_pos, sizeof(int), cudaMemcpyDeviceToHost, g->st));
    RC_OK(check_status(g));
    if (steps) *steps = ss.steps;
    if (union_sum) *union_sum = ss.n_union_sum;
    if (last_kept) *last_kept = ss.kept;
    g->last_batch = 0;
    g->hid_rows = 0;
    return GCUDA_OK;
}

// The stream the handle enqueues on (a cudaStream_t), for callers that time it with their own events.
void *gcuda_stream(gcuda *g) { return g ? static_cast<void *>(g->st) : nullptr; }

}  // extern "C"
