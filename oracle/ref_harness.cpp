// ref_harness.cpp - TEST INFRASTRUCTURE. A C API over the reference engine's own C++ code (compiled from the
// reference checkout by oracle/Makefile into oracle/_ref/), so the Python tests can call it with ctypes:
//   - the whole verify pass:  geode::Model::open / forward_batch(all_logits) / save_state / load_state
//     (engine/src/model.hpp:161,166,239-240), with the per-layer trace hook (engine/src/model.hpp:92-105,341);
//   - the MTP drafting layer: Model::forward_mtp and the hidden rows it takes (engine/src/model.hpp:168-183);
//   - the kernels the pass is made of (engine/src/kernels.hpp): quantize_activation, matvec_rows_q_ref,
//     dequant_row, matvec_rows_bf16_multi, rmsnorm, fast_exp; route_topk (engine/src/model.hpp:30);
//   - the sampler (engine/src/sampler.hpp) and the acceptance rule of the speculation loop, restated around it
//     (engine/src/geode.cpp:327-350);
//   - the q4 block quantizer (engine/src/yue2_q4.hpp:51-53), used to pin the restated quantizer.
// Nothing here is product code: the CUDA path never links or calls it.
#include <cstdint>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "kernels.hpp"
#include "model.hpp"
#include "sampler.hpp"
#include "yue2_q4.hpp"

namespace {

struct Ref {
    geode::Model model;
    bool tracing = false;
    int hidden = 0, k = 0;
    // trace rows, [layer][token][hidden] for x, mixer, moe, out; [layer][token][k] for experts / weights
    std::vector<float> tx, tmix, tmoe, tout, tw, tgate;
    std::vector<int> tids;
    int tlayers = 0, ttokens = 0;
};

void put_err(const std::string &e, char *err, int len) {
    if (!err || len <= 0) return;
    std::strncpy(err, e.c_str(), static_cast<size_t>(len - 1));
    err[len - 1] = 0;
}

}  // namespace

extern "C" {

// draft: 1 = bind the pack's MTP layer (ModelOptions::no_draft false: forward_mtp works, the state holds the
// layer's KV), 0 = leave it unread as the verify tests do
void *ref_open2(const char *dir, int threads, int ctx, int draft, char *err, int errlen) {
    auto *r = new Ref;
    geode::ModelOptions o;
    o.compute_threads = threads;
    o.context_length = ctx;
    o.memory_budget = 0;
    o.npu = 0;
    o.mode = 1;   // RunMode::Cpu
    o.no_draft = draft == 0, o.no_vision = true, o.no_audio = true;
    std::string e;
    if (!r->model.open(dir, o, e)) {
        put_err(e, err, errlen);
        delete r;
        return nullptr;
    }
    r->hidden = r->model.config().hidden;
    r->k = r->model.config().top_k;
    return r;
}

void *ref_open(const char *dir, int threads, int ctx, char *err, int errlen) {
    return ref_open2(dir, threads, ctx, 0, err, errlen);
}

void ref_close(void *h) { delete static_cast<Ref *>(h); }

// Model::hidden(t) (engine/src/model.hpp:181): token t of the last forward_batch after the final norm (kept when the
// model has an MTP layer), hidden floats into out; -1 when the model keeps none
int ref_hidden(void *h, int t, float *out) {
    Ref *r = static_cast<Ref *>(h);
    if (!r->model.has_mtp()) return -1;
    std::memcpy(out, r->model.hidden(t), static_cast<size_t>(r->hidden) * 4);
    return 0;
}

// Model::forward_mtp (engine/src/model.cpp:4965-5039): n positions from pos, position i taking hidden row i
// (hidden: n x hidden floats) and the embedding of next[i]; logits: the last position's [vocab] (NULL: none);
// mtp_hidden (NULL: not wanted): that position's output after the layer's final norm (Model::mtp_hidden)
int ref_mtp(void *h, const int *next, const float *hidden, int n, int pos, float *logits, float *mtp_hidden, char *err,
            int errlen) {
    Ref *r = static_cast<Ref *>(h);
    std::vector<const float *> rows(static_cast<size_t>(n));
    for (int t = 0; t < n; ++t) rows[static_cast<size_t>(t)] = hidden + static_cast<size_t>(t) * r->hidden;
    std::string e;
    if (!r->model.forward_mtp(next, rows.data(), n, pos, logits, e)) {
        put_err(e, err, errlen);
        return -1;
    }
    if (logits && mtp_hidden) std::memcpy(mtp_hidden, r->model.mtp_hidden(), static_cast<size_t>(r->hidden) * 4);
    return 0;
}

int ref_position(void *h) { return static_cast<Ref *>(h)->model.position(); }

// Model::profile (engine/src/model.cpp:5041): the stage times since open, one line
void ref_profile(void *h, char *buf, int len) {
    const std::string p = static_cast<Ref *>(h)->model.profile();
    std::strncpy(buf, p.c_str(), static_cast<size_t>(len - 1));
    buf[len - 1] = 0;
}

// trace: the next forward_batch records every layer's rows for its n tokens
void ref_trace(void *h, int on, int layers, int tokens) {
    Ref *r = static_cast<Ref *>(h);
    r->tracing = on != 0;
    if (!r->tracing) {
        r->model.trace = nullptr;
        return;
    }
    const size_t H = static_cast<size_t>(r->hidden), K = static_cast<size_t>(std::max(1, r->k));
    const size_t rows = static_cast<size_t>(layers) * static_cast<size_t>(tokens);
    r->tlayers = layers, r->ttokens = tokens;
    r->tx.assign(rows * H, 0.f), r->tmix.assign(rows * H, 0.f), r->tmoe.assign(rows * H, 0.f), r->tout.assign(rows * H, 0.f);
    r->tw.assign(rows * K, 0.f), r->tids.assign(rows * K, -1), r->tgate.assign(rows, 0.f);
    r->model.trace = [r, H, K](const geode::LayerTrace &t) {
        const int tok = t.pos - (r->model.position());
        if (t.layer >= r->tlayers || tok < 0 || tok >= r->ttokens) return;
        const size_t o = static_cast<size_t>(t.layer) * r->ttokens + static_cast<size_t>(tok);
        std::memcpy(&r->tx[o * H], t.x, H * 4);
        std::memcpy(&r->tmix[o * H], t.mixer, H * 4);
        std::memcpy(&r->tmoe[o * H], t.moe, H * 4);
        std::memcpy(&r->tout[o * H], t.out, H * 4);
        if (t.experts && r->k > 0) {
            std::memcpy(&r->tids[o * K], t.experts, K * 4);
            std::memcpy(&r->tw[o * K], t.weights, K * 4);
        }
        r->tgate[o] = t.shared_gate;
    };
}

// what: 0 x, 1 mixer, 2 moe, 3 out (hidden floats); 4 expert ids (k ints); 5 weights (k floats); 6 gate (1 float)
void ref_trace_get(void *h, int what, void *out) {
    Ref *r = static_cast<Ref *>(h);
    switch (what) {
    case 0: std::memcpy(out, r->tx.data(), r->tx.size() * 4); break;
    case 1: std::memcpy(out, r->tmix.data(), r->tmix.size() * 4); break;
    case 2: std::memcpy(out, r->tmoe.data(), r->tmoe.size() * 4); break;
    case 3: std::memcpy(out, r->tout.data(), r->tout.size() * 4); break;
    case 4: std::memcpy(out, r->tids.data(), r->tids.size() * 4); break;
    case 5: std::memcpy(out, r->tw.data(), r->tw.size() * 4); break;
    case 6: std::memcpy(out, r->tgate.data(), r->tgate.size() * 4); break;
    default: break;
    }
}

int ref_forward(void *h, const int *toks, int n, float *logits, int all_logits, char *err, int errlen) {
    Ref *r = static_cast<Ref *>(h);
    std::string e;
    if (!r->model.forward_batch(toks, n, logits, all_logits != 0, e)) {
        put_err(e, err, errlen);
        return -1;
    }
    return 0;
}

int ref_save_state(void *h, const char *path, char *err, int errlen) {
    std::string e;
    if (!static_cast<Ref *>(h)->model.save_state(path, false, 0, e)) {
        put_err(e, err, errlen);
        return -1;
    }
    return 0;
}

int ref_load_state(void *h, const char *path, char *err, int errlen) {
    std::string e;
    int32_t extra = 0;
    if (!static_cast<Ref *>(h)->model.load_state(path, extra, e)) {
        put_err(e, err, errlen);
        return -1;
    }
    return 0;
}

// ---- kernels (engine/src/kernels.hpp) ----

void ref_quantize_activation(const float *x, int64_t cols, int8_t *q, float *scale, int32_t *bsum) {
    geode::QAct a;
    geode::quantize_activation(x, cols, a);
    std::memcpy(q, a.q.data(), static_cast<size_t>(cols));
    std::memcpy(scale, a.scale.data(), static_cast<size_t>(cols / 16) * 4);
    std::memcpy(bsum, a.bsum.data(), static_cast<size_t>(cols / 16) * 4);
}

// y[t][r] for n tokens: matvec_rows_q_multi over the pack's layout (type: the DType value, q4 = 6)
void ref_matvec_q(const uint8_t *data, int64_t rows, int64_t cols, float global, int type, int n, const float *xs,
                  float *ys) {
    geode::QView m{static_cast<geode::DType>(type), rows, cols, geode::row_bytes(static_cast<geode::DType>(type), cols),
                   data, global};
    std::vector<geode::QAct> acts(static_cast<size_t>(n));
    std::vector<const geode::QAct *> ap(static_cast<size_t>(n));
    std::vector<float *> yp(static_cast<size_t>(n));
    for (int t = 0; t < n; ++t) {
        geode::quantize_activation(xs + static_cast<size_t>(t) * cols, cols, acts[static_cast<size_t>(t)]);
        ap[static_cast<size_t>(t)] = &acts[static_cast<size_t>(t)];
        yp[static_cast<size_t>(t)] = ys + static_cast<size_t>(t) * rows;
    }
    geode::matvec_rows_q_multi(m, ap.data(), n, yp.data(), 0, rows);
}

// the exact path: FP32 activations times the dequantized weights (engine/src/kernels.cpp:1230-1250)
void ref_matvec_exact(const uint8_t *data, int64_t rows, int64_t cols, float global, int type, const float *x, float *y) {
    geode::QView m{static_cast<geode::DType>(type), rows, cols, geode::row_bytes(static_cast<geode::DType>(type), cols),
                   data, global};
    geode::matvec_rows(m, x, y, 0, rows);
}

void ref_dequant_row(const uint8_t *data, int64_t cols, float global, int type, float *out) {
    geode::QView m{static_cast<geode::DType>(type), 1, cols, geode::row_bytes(static_cast<geode::DType>(type), cols),
                   data, global};
    geode::dequant_row(m, 0, out);
}

void ref_matvec_bf16_multi(const uint16_t *w, int64_t rows, int64_t cols, int n, const float *xs, float *ys) {
    std::vector<const float *> xp(static_cast<size_t>(n));
    std::vector<float *> yp(static_cast<size_t>(n));
    for (int t = 0; t < n; ++t) {
        xp[static_cast<size_t>(t)] = xs + static_cast<size_t>(t) * cols;
        yp[static_cast<size_t>(t)] = ys + static_cast<size_t>(t) * rows;
    }
    geode::matvec_rows_bf16_multi(w, cols, n, xp.data(), yp.data(), 0, rows);
}

void ref_rmsnorm(const float *x, const float *w, float *out, int n, float eps, int zero_centered) {
    geode::rmsnorm(x, w, out, n, eps, zero_centered != 0);
}

float ref_fast_exp(float x) { return geode::fast_exp(x); }

void ref_route_topk(const float *logits, int E, int K, int *ids, float *weights) {
    geode::route_topk(logits, E, K, ids, weights, nullptr, 0.0f, nullptr);
}

void ref_q4_block(const float *x, float s2, uint8_t *scale_byte, uint8_t *codes) {
    geode::yue2::q4_block(x, s2, *scale_byte, codes);
}

float ref_e4m3_value(uint8_t b) { return geode::e4m3_value(b); }

// ---- the acceptance rule (engine/src/geode.cpp:327-350) around the real geode::Sampler ----
//
// rows: n rows of V logits (toks[0]'s row first); batch: the n tokens verified (batch[0] = the accepted token,
// batch[1..n-1] the drafts). Row i is sampled in order; draft i+1 stands while it equals row i's sample and is no
// stop token. Returns kept (1 + the drafts that stood); *next = the first sample that is no draft (or -1 when the
// loop stopped on a stop token that stood). samples[i] = row i's sample for the rows sampled (-1 after).
int ref_accept(const float *rows, int n, int V, const int *batch, float temperature, float top_p, int top_k,
               uint64_t seed, const int *stops, int n_stops, int *next, int *samples) {
    geode::Sampler s;
    s.seed(seed);
    geode::SamplerParams sp;
    sp.temperature = temperature;
    sp.top_p = top_p;
    sp.top_k = top_k;
    std::vector<float> row(static_cast<size_t>(V));
    auto is_stop = [&](int t) {
        for (int i = 0; i < n_stops; ++i)
            if (stops[i] == t) return true;
        return false;
    };
    for (int i = 0; i < n; ++i) samples[i] = -1;
    int kept = 1;
    *next = -1;
    for (int i = 0; i < n; ++i) {
        std::memcpy(row.data(), rows + static_cast<size_t>(i) * V, static_cast<size_t>(V) * 4);
        const int y = s.sample(row.data(), V, sp);
        samples[i] = y;
        if (i + 1 < n && y == batch[i + 1] && !is_stop(y)) {
            ++kept;
            continue;
        }
        *next = y;
        break;
    }
    return kept;
}

// ref_accept with geode_generate's presence penalty, its sample() lambda restated (engine/src/geode.cpp:234-255):
// before a row is sampled every token of seen loses the penalty; a new sample joins seen (the is_seen bitmap is
// only kept while the penalty is on). seen in/out (room for n more), *n_seen its length.
int ref_accept_seen(const float *rows, int n, int V, const int *batch, float temperature, float top_p, int top_k,
                    uint64_t seed, const int *stops, int n_stops, float penalty, int *seen, int *n_seen, int *next,
                    int *samples) {
    geode::Sampler s;
    s.seed(seed);
    geode::SamplerParams sp;
    sp.temperature = temperature;
    sp.top_p = top_p;
    sp.top_k = top_k;
    std::vector<int32_t> seen_list(seen, seen + *n_seen);
    std::vector<uint8_t> is_seen(penalty != 0.0f ? static_cast<size_t>(V) : 0, 0);
    for (int32_t t : seen_list)
        if (!is_seen.empty()) is_seen[static_cast<size_t>(t)] = 1;
    std::vector<float> row(static_cast<size_t>(V));
    const auto sample = [&](float *lg) {
        for (int32_t t : seen_list) lg[static_cast<size_t>(t)] -= penalty;
        const int32_t tok = s.sample(lg, V, sp);
        if (!is_seen.empty() && tok >= 0 && static_cast<size_t>(tok) < is_seen.size() && !is_seen[static_cast<size_t>(tok)]) {
            is_seen[static_cast<size_t>(tok)] = 1;
            seen_list.push_back(tok);
        }
        return tok;
    };
    auto is_stop = [&](int t) {
        for (int i = 0; i < n_stops; ++i)
            if (stops[i] == t) return true;
        return false;
    };
    for (int i = 0; i < n; ++i) samples[i] = -1;
    int kept = 1;
    *next = -1;
    for (int i = 0; i < n; ++i) {
        std::memcpy(row.data(), rows + static_cast<size_t>(i) * V, static_cast<size_t>(V) * 4);
        const int y = sample(row.data());
        samples[i] = y;
        if (i + 1 < n && y == batch[i + 1] && !is_stop(y)) {
            ++kept;
            continue;
        }
        *next = y;
        break;
    }
    for (size_t j = 0; j < seen_list.size(); ++j) seen[j] = seen_list[j];
    *n_seen = static_cast<int>(seen_list.size());
    return kept;
}

// the sampler's uniform stream: the first n draws uniform_real_distribution<double>(0, 1) makes from
// mt19937_64(seed) (engine/src/sampler.cpp:45 draws (0, kept); the distribution is a + (b - a) * canonical)
void ref_uniforms(uint64_t seed, int n, double *out) {
    std::mt19937_64 rng(seed);
    for (int i = 0; i < n; ++i) out[i] = std::generate_canonical<double, 53>(rng);
}

}  // extern "C"
