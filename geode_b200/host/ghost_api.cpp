// ghost_api.cpp - the C ABI of include/geode_host.h over CudaModel.
#include <cstring>
#include <string>
#include <vector>

#include "../../include/geode_host.h"
#include "cuda_model.hpp"

struct ghost_model {
    ghost::CudaModel model;
    ghost::SamplerParams params;
    ghost::Sampler sampler;
    ghost::SeenTokens seen;   // the answer's tokens for the presence penalty (from ghost_set_sampling on)
    int32_t pending = -1;   // the token passed on but not computed yet (geode.cpp's `pending`)
};

namespace {
void put(const std::string &s, char *buf, size_t len) {
    if (!buf || len == 0) return;
    std::strncpy(buf, s.c_str(), len - 1);
    buf[len - 1] = 0;
}
}  // namespace

extern "C" {

int ghost_open(const char *dir, int32_t device, int32_t context, int32_t max_tokens, ghost_model **out, char *err,
               size_t err_len) {
    if (!dir || !out) {
        put("ghost_open: bad arguments", err, err_len);
        return GHOST_E_ARG;
    }
    *out = nullptr;
    auto *m = new ghost_model;
    ghost::ModelOptions o;
    o.device = device;
    o.context = context;
    o.max_tokens = max_tokens;
    std::string e;
    if (!m->model.open(dir, o, e)) {
        put(e, err, err_len);
        delete m;
        return e.rfind("no geode.json", 0) == 0 || e.rfind("cannot", 0) == 0 ? GHOST_E_IO : GHOST_E_BACKEND;
    }
    *out = m;
    return GHOST_OK;
}

void ghost_close(ghost_model *m) { delete m; }

int32_t ghost_spec_tokens(ghost_model *m) { return m ? m->model.spec_tokens() : 0; }

int32_t ghost_position(ghost_model *m) { return m ? m->model.position() : 0; }

int ghost_verify(ghost_model *m, const int32_t *toks, int32_t n, float *logits, char *err, size_t err_len) {
    if (!m || !toks || n < 1) return GHOST_E_ARG;
    std::string e;
    if (!m->model.verify_n(toks, n, logits, e)) {
        put(e, err, err_len);
        return GHOST_E_BACKEND;
    }
    return GHOST_OK;
}

int ghost_draft(ghost_model *m, const int32_t *toks, int32_t n, int32_t pos, const float *hidden, int32_t *draft,
                float *prob, char *err, size_t err_len) {
    if (!m || !toks || !draft || n < 1) return GHOST_E_ARG;
    std::string e;
    int d = -1;
    if (!m->model.draft(toks, n, pos, hidden, d, prob, e)) {
        put(e, err, err_len);
        return GHOST_E_BACKEND;
    }
    *draft = d;
    return GHOST_OK;
}

int ghost_draft_next(ghost_model *m, int32_t tok, int32_t pos, int32_t *draft, float *prob, char *err, size_t err_len) {
    if (!m || !draft) return GHOST_E_ARG;
    std::string e;
    int d = -1;
    if (!m->model.draft_next(tok, pos, d, prob, e)) {
        put(e, err, err_len);
        return GHOST_E_BACKEND;
    }
    *draft = d;
    return GHOST_OK;
}

int ghost_reset(ghost_model *m, char *err, size_t err_len) {
    if (!m) return GHOST_E_ARG;
    std::string e;
    if (!m->model.reset(e)) {
        put(e, err, err_len);
        return GHOST_E_BACKEND;
    }
    m->pending = -1;
    return GHOST_OK;
}

int ghost_prefill(ghost_model *m, const int32_t *prompt, int32_t n, char *err, size_t err_len) {
    if (!m || !prompt || n < 1) {
        put("ghost_prefill: bad arguments", err, err_len);
        return GHOST_E_ARG;
    }
    std::string e;
    if (!m->model.prefill(prompt, n, e)) {
        put(e, err, err_len);
        return e.find("embedding of token") != std::string::npos || e.find("context is full") != std::string::npos
                   ? GHOST_E_ARG
                   : GHOST_E_BACKEND;
    }
    m->pending = -1;
    return GHOST_OK;
}

int ghost_keep(ghost_model *m, int32_t kept, char *err, size_t err_len) {
    if (!m) return GHOST_E_ARG;
    std::string e;
    if (!m->model.verify_keep(kept, e)) {
        put(e, err, err_len);
        return GHOST_E_BACKEND;
    }
    return GHOST_OK;
}

int ghost_set_sampling(ghost_model *m, const ghost_sampling *s) {
    if (!m || !s) return GHOST_E_ARG;
    m->params.temperature = s->temperature;
    m->params.top_p = s->top_p;
    m->params.top_k = s->top_k;
    m->params.presence_penalty = s->presence_penalty;
    m->sampler.seed(s->seed);
    m->seen.clear();
    return GHOST_OK;
}

int ghost_step(ghost_model *m, const int32_t *batch, int32_t n, const int32_t *stops, int32_t n_stops, int32_t *kept,
               int32_t *next, char *err, size_t err_len) {
    if (!m || !batch || n < 1 || !kept || !next) return GHOST_E_ARG;
    std::string e;
    int k = 0, nx = 0;
    if (!m->model.step(batch, n, m->params, m->sampler, m->seen, stops, n_stops, k, nx, e)) {
        put(e, err, err_len);
        return GHOST_E_BACKEND;
    }
    *kept = k;
    *next = nx;
    m->pending = nx;
    return GHOST_OK;
}

int ghost_pack_summary(const char *dir, char *out, size_t out_len, char *err, size_t err_len) {
    if (!dir || !out) return GHOST_E_ARG;
    std::string s, e;
    if (!ghost::pack_summary(dir, s, e)) {
        put(e, err, err_len);
        return GHOST_E_IO;
    }
    put(s, out, out_len);
    return GHOST_OK;
}

int ghost_state_save(ghost_model *m, const char *path, int32_t append, int32_t *out_position, char *err,
                     size_t err_len) {
    if (!m || !path || !*path) {
        put("ghost_state_save: bad arguments", err, err_len);
        return GHOST_E_ARG;
    }
    std::string e;
    int code = 0;
    if (!m->model.save_state(path, append != 0, m->pending, code, e)) {
        put(e, err, err_len);
        return code;
    }
    if (out_position) *out_position = m->model.position();
    return GHOST_OK;
}

int ghost_state_load(ghost_model *m, const char *path, int32_t *out_position, char *err, size_t err_len) {
    if (!m || !path || !*path) {
        put("ghost_state_load: bad arguments", err, err_len);
        return GHOST_E_ARG;
    }
    std::string e;
    int code = 0, extra = -1;
    const bool ok = m->model.load_state(path, extra, code, e);
    m->pending = ok ? extra : -1;
    if (out_position) *out_position = m->model.position();
    if (!ok) {
        put(e, err, err_len);
        return code;
    }
    return GHOST_OK;
}

int32_t ghost_pending(ghost_model *m) { return m ? m->pending : -1; }

namespace {
ghost::StateShapes shapes_of(const ghost_state_shapes *s) {
    ghost::StateShapes o;
    o.n_attn = s->n_attn;
    o.kv_heads = s->kv_heads;
    o.kv_row = s->kv_row;
    o.hidden = s->hidden;
    o.n_layers = s->n_layers;
    o.conv_n = s->conv_n;
    o.gdn_n = s->gdn_n;
    o.mtp = s->mtp;
    return o;
}
int state_code(ghost::StateError e) {
    return e == ghost::StateError::none     ? GHOST_OK
           : e == ghost::StateError::format ? GHOST_E_FORMAT
           : e == ghost::StateError::context ? GHOST_E_ARG
                                             : GHOST_E_IO;
}
}  // namespace

uint64_t ghost_state_fingerprint(const char *pack_dir, const ghost_state_shapes *s) {
    if (!pack_dir || !s) return 0;
    return ghost::state_fingerprint(ghost::pack_print(pack_dir), shapes_of(s));
}

int ghost_state_write(const char *path, uint64_t fingerprint, const ghost_state_shapes *s, int32_t position,
                      int32_t extra, uint64_t conv_id, const float *conv, const float *gdn, const int8_t *kv,
                      const float *kv_scale, const float *hidden, int32_t append, char *err, size_t err_len) {
    if (!path || !s) return GHOST_E_ARG;
    ghost::StateMeta m;
    m.position = position;
    m.extra = extra;
    m.conv_id = conv_id;
    std::string e;
    if (!ghost::write_state(path, fingerprint, shapes_of(s), m, conv, gdn, kv, kv_scale, hidden, append != 0, e)) {
        put(e, err, err_len);
        return e.rfind("write_state: bad", 0) == 0 ? GHOST_E_ARG : GHOST_E_IO;
    }
    return GHOST_OK;
}

int ghost_state_peek(const char *path, uint64_t fingerprint, const ghost_state_shapes *s, int32_t context,
                     int32_t *position, int32_t *extra, uint64_t *conv_id, char *err, size_t err_len) {
    if (!path || !s) return GHOST_E_ARG;
    ghost::StateMeta m;
    std::string e;
    const ghost::StateError r = ghost::peek_state(path, fingerprint, shapes_of(s), context, m, e);
    if (r != ghost::StateError::none) {
        put(e, err, err_len);
        return state_code(r);
    }
    if (position) *position = m.position;
    if (extra) *extra = m.extra;
    if (conv_id) *conv_id = m.conv_id;
    return GHOST_OK;
}

int ghost_state_read(const char *path, uint64_t fingerprint, const ghost_state_shapes *s, int32_t context, float *conv,
                     float *gdn, int8_t *kv, float *kv_scale, float *hidden, int32_t *has_hidden, char *err,
                     size_t err_len) {
    if (!path || !s) return GHOST_E_ARG;
    ghost::StateMeta m;
    std::vector<float> c, g, ks, hd;
    std::vector<int8_t> k;
    std::string e;
    const ghost::StateError r = ghost::read_state(path, fingerprint, shapes_of(s), context, m, c, g, k, ks, hd, e);
    if (r != ghost::StateError::none) {
        put(e, err, err_len);
        return state_code(r);
    }
    if ((!c.empty() && !conv) || (!g.empty() && !gdn) || (!k.empty() && (!kv || !kv_scale))) return GHOST_E_ARG;
    if (!c.empty()) std::memcpy(conv, c.data(), c.size() * sizeof(float));
    if (!g.empty()) std::memcpy(gdn, g.data(), g.size() * sizeof(float));
    if (!k.empty()) std::memcpy(kv, k.data(), k.size());
    if (!ks.empty()) std::memcpy(kv_scale, ks.data(), ks.size() * sizeof(float));
    if (has_hidden) *has_hidden = hd.empty() ? 0 : 1;
    if (!hd.empty() && hidden) std::memcpy(hidden, hd.data(), hd.size() * sizeof(float));
    return GHOST_OK;
}

}  // extern "C"
