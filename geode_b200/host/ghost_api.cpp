// ghost_api.cpp - the C ABI of include/geode_host.h over CudaModel.
#include <cstring>
#include <string>

#include "../../include/geode_host.h"
#include "cuda_model.hpp"

struct ghost_model {
    ghost::CudaModel model;
    ghost::SamplerParams params;
    ghost::Sampler sampler;
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
    m->sampler.seed(s->seed);
    return GHOST_OK;
}

int ghost_step(ghost_model *m, const int32_t *batch, int32_t n, const int32_t *stops, int32_t n_stops, int32_t *kept,
               int32_t *next, char *err, size_t err_len) {
    if (!m || !batch || n < 1 || !kept || !next) return GHOST_E_ARG;
    std::string e;
    int k = 0, nx = 0;
    if (!m->model.step(batch, n, m->params, m->sampler, stops, n_stops, k, nx, e)) {
        put(e, err, err_len);
        return GHOST_E_BACKEND;
    }
    *kept = k;
    *next = nx;
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

}  // extern "C"
