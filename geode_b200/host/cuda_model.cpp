// cuda_model.cpp - see cuda_model.hpp.
#include "cuda_model.hpp"

#include <dlfcn.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

namespace ghost {

namespace {
std::string own_dir() {
    Dl_info info{};
    if (dladdr(reinterpret_cast<void *>(&own_dir), &info) && info.dli_fname) {
        std::string p = info.dli_fname;
        const size_t s = p.rfind('/');
        if (s != std::string::npos) return p.substr(0, s);
    }
    return ".";
}
}  // namespace

bool CudaApi::load(const std::string &path, std::string &err) {
    const std::string p = path.empty() ? own_dir() + "/libgeode_cuda.so" : path;
    lib = dlopen(p.c_str(), RTLD_NOW | RTLD_LOCAL);
    if (!lib) {
        err = std::string("cannot load the CUDA backend (no CPU fallback): ") + dlerror();
        return false;
    }
    bool ok = true;
    auto sym = [&](auto &fn, const char *name) {
        fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(lib, name));
        if (!fn) {
            err = std::string("the CUDA backend lacks ") + name;
            ok = false;
        }
    };
    sym(open, "gcuda_open");
    sym(close, "gcuda_close");
    sym(last_error, "gcuda_last_error");
    sym(adopt_q4, "gcuda_adopt_q4");
    sym(adopt_raw, "gcuda_adopt_raw");
    sym(adopt_embedding, "gcuda_adopt_embedding");
    sym(adopt_experts, "gcuda_adopt_experts");
    sym(setup, "gcuda_setup");
    sym(verify, "gcuda_verify");
    sym(keep, "gcuda_keep");
    sym(position, "gcuda_position");
    sym(accept, "gcuda_accept");
    sym(state_get, "gcuda_state_get");
    sym(state_put, "gcuda_state_put");
    sym(reset, "gcuda_reset");
    sym(set_mtp, "gcuda_set_mtp");
    sym(set_draft_head, "gcuda_set_draft_head");
    sym(last_hidden, "gcuda_last_hidden");
    sym(put_last_hidden, "gcuda_put_last_hidden");
    sym(draft, "gcuda_draft");
    sym(draft_next, "gcuda_draft_next");
    return ok;
}

CudaApi::~CudaApi() {
    if (lib) dlclose(lib);
}

CudaModel::~CudaModel() {
    if (g_ && api_.close) api_.close(g_);
}

bool CudaModel::fail(const char *what, std::string &err) {
    char buf[512] = {0};
    if (g_) api_.last_error(g_, buf, sizeof buf);
    err = std::string(what) + ": " + buf;
    return false;
}

int CudaModel::position() const { return g_ ? api_.position(g_) : 0; }

bool CudaModel::open(const std::string &dir, const ModelOptions &opt, std::string &err) {
    if (opt.max_tokens < 1 || opt.max_tokens > 8) {
        err = "max_tokens: 1 .. 8";
        return false;
    }
    if (!api_.load("", err)) return false;
    if (!pack_.open(dir, err)) return false;
    char ebuf[512] = {0};
    g_ = api_.open(opt.device, ebuf, sizeof ebuf);
    if (!g_) {
        err = std::string("gcuda_open: ") + ebuf;
        return false;
    }
    const JsonRef c = pack_.config();
    const bool dense = pack_.arch() == "qwen35";
    const int L = static_cast<int>(c["num_hidden_layers"].integer());
    std::vector<gcuda_layer> layers(static_cast<size_t>(L));
    // every tensor into device memory, by the names engine/src/model.cpp:94-203 reads
    auto q4 = [&](const std::string &name, int &id) -> bool {
        TensorView t;
        if (!pack_.tensor(name, t, err)) return false;
        id = api_.adopt_q4(g_, t.data, t.rows(), t.cols(), static_cast<size_t>(t.cols() / 16) * 9, t.global);
        return id >= 0 || fail(name.c_str(), err);
    };
    auto raw = [&](const std::string &name, int &id) -> bool {
        TensorView t;
        if (!pack_.tensor(name, t, err)) return false;
        id = api_.adopt_raw(g_, t.data, t.bytes);
        return id >= 0 || fail(name.c_str(), err);
    };
    const JsonRef types = c["layer_types"];
    // one decoder layer's tensors under prefix p; l: its index for the expert table (-1: the MTP layer's)
    auto load_layer = [&](gcuda_layer &x, const std::string &p, bool attn, int l) -> bool {
        std::memset(&x, 0xFF, sizeof x);   // every id -1
        x.attn = attn ? 1 : 0;
        bool ok = raw(p + "input_layernorm.weight", x.in_norm) && raw(p + "post_attention_layernorm.weight", x.post_norm);
        if (attn) {
            ok = ok && q4(p + "self_attn.q_proj.weight", x.q) && q4(p + "self_attn.k_proj.weight", x.k) &&
                 q4(p + "self_attn.v_proj.weight", x.v) && q4(p + "self_attn.o_proj.weight", x.o) &&
                 raw(p + "self_attn.q_norm.weight", x.q_norm) && raw(p + "self_attn.k_norm.weight", x.k_norm);
        } else {
            ok = ok && q4(p + "linear_attn.in_proj_qkv.weight", x.qkv) && q4(p + "linear_attn.in_proj_z.weight", x.z) &&
                 q4(p + "linear_attn.out_proj.weight", x.out) && raw(p + "linear_attn.in_proj_a.weight", x.a) &&
                 raw(p + "linear_attn.in_proj_b.weight", x.b) && raw(p + "linear_attn.A_log", x.A_log) &&
                 raw(p + "linear_attn.dt_bias", x.dt_bias) && raw(p + "linear_attn.conv1d.weight", x.conv) &&
                 raw(p + "linear_attn.norm.weight", x.gnorm);
        }
        if (dense) {
            ok = ok && q4(p + "mlp.gate_proj.weight", x.sh_gate) && q4(p + "mlp.up_proj.weight", x.sh_up) &&
                 q4(p + "mlp.down_proj.weight", x.sh_down);
        } else {
            ok = ok && q4(p + "mlp.shared_expert.gate_proj.weight", x.sh_gate) &&
                 q4(p + "mlp.shared_expert.up_proj.weight", x.sh_up) &&
                 q4(p + "mlp.shared_expert.down_proj.weight", x.sh_down) && raw(p + "mlp.gate.weight", x.router) &&
                 raw(p + "mlp.shared_expert_gate.weight", x.shared_gate);
            if (ok) {
                ExpertTable e;
                TensorView sc;
                ok = pack_.experts(l, e, err) && pack_.tensor(p + "mlp.experts.scales", sc, err);
                if (ok) {
                    x.experts = api_.adopt_experts(g_, e.data, static_cast<int>(c["num_experts"].integer()), e.stride,
                                                   reinterpret_cast<const float *>(sc.data));
                    ok = x.experts >= 0 || fail("experts", err);
                }
            }
        }
        return ok;
    };
    for (int l = 0; l < L; ++l)
        if (!load_layer(layers[static_cast<size_t>(l)], "layers." + std::to_string(l) + ".",
                        types[static_cast<size_t>(l)].text() == "full_attention", l))
            return false;
    // the MTP drafting layer (engine/src/model.cpp:175-191), when the pack has one: on the device beside the model
    if (pack_.has("mtp.fc.weight")) {
        gcuda_layer mt;
        int fc = -1, pre_e = -1, pre_h = -1, mnorm = -1;
        if (!load_layer(mt, "mtp.layers.0.", true, -1) || !q4("mtp.fc.weight", fc) ||
            !raw("mtp.pre_fc_norm_embedding.weight", pre_e) || !raw("mtp.pre_fc_norm_hidden.weight", pre_h) ||
            !raw("mtp.norm.weight", mnorm))
            return false;
        if (api_.set_mtp(g_, fc, pre_e, pre_h, mnorm, &mt) != 0) return fail("set_mtp", err);
        has_mtp_ = true;
        // the draft head (engine/src/model.cpp:2135-2161): draft_vocab.bin's ids inside the vocabulary, padded to whole
        // tiles of 32 rows with copies of the first, and lm_head's rows of them
        std::vector<int32_t> ids;
        if (std::FILE *f = std::fopen((dir + "/draft_vocab.bin").c_str(), "rb")) {
            const int64_t V = c["vocab_size"].integer();
            int32_t id;
            while (std::fread(&id, 4, 1, f) == 1)
                if (id >= 0 && id < V) ids.push_back(id);
            std::fclose(f);
        }
        if (!ids.empty()) {
            while (ids.size() % 32) ids.push_back(ids[0]);
            TensorView lm;
            if (!pack_.tensor("lm_head.weight", lm, err)) return false;
            const size_t rb = static_cast<size_t>(lm.cols() / 16) * 9;
            std::vector<uint8_t> rows(ids.size() * rb);
            for (size_t r = 0; r < ids.size(); ++r)
                std::memcpy(rows.data() + r * rb, lm.data + static_cast<size_t>(ids[r]) * rb, rb);
            const int dh = api_.adopt_q4(g_, rows.data(), static_cast<int64_t>(ids.size()), lm.cols(), rb, lm.global);
            if (dh < 0 || api_.set_draft_head(g_, dh, ids.data(), static_cast<int>(ids.size())) != 0)
                return fail("draft head", err);
        }
    }
    TensorView et;
    if (!pack_.tensor("embed_tokens.weight", et, err)) return false;
    const int embed = api_.adopt_embedding(g_, et.data, et.rows(), et.cols(), et.global);
    if (embed < 0) return fail("embedding", err);
    int head = -1, norm = -1;
    if (!q4("lm_head.weight", head) || !raw("norm.weight", norm)) return false;
    const JsonRef rope = c["rope_parameters"];
    gcuda_shape s{};
    s.hidden = static_cast<int>(c["hidden_size"].integer());
    s.n_layers = L;
    s.vocab = static_cast<int>(c["vocab_size"].integer());
    s.eps = static_cast<float>(c["rms_norm_eps"].number(1e-6));
    s.n_heads = static_cast<int>(c["num_attention_heads"].integer());
    s.n_kv_heads = static_cast<int>(c["num_key_value_heads"].integer());
    s.head_dim = static_cast<int>(c["head_dim"].integer());
    s.rope_dim = static_cast<int>(static_cast<double>(s.head_dim) * rope["partial_rotary_factor"].number(1.0));
    s.rope_theta = static_cast<float>(rope["rope_theta"].number(10000.0));
    s.gdn_k_heads = static_cast<int>(c["linear_num_key_heads"].integer());
    s.gdn_v_heads = static_cast<int>(c["linear_num_value_heads"].integer());
    s.gdn_k_dim = static_cast<int>(c["linear_key_head_dim"].integer());
    s.gdn_v_dim = static_cast<int>(c["linear_value_head_dim"].integer());
    s.conv_kernel = static_cast<int>(c["linear_conv_kernel_dim"].integer());
    s.n_experts = static_cast<int>(c["num_experts"].integer());
    s.top_k = static_cast<int>(c["num_experts_per_tok"].integer());
    s.moe_ff = static_cast<int>(c["moe_intermediate_size"].integer());
    s.shared_ff = static_cast<int>(dense ? c["intermediate_size"].integer() : c["shared_expert_intermediate_size"].integer());
    s.dense = dense ? 1 : 0;
    s.context = opt.context > 0 ? opt.context : 4096;
    s.max_tokens = opt.max_tokens;
    if (api_.setup(g_, &s, layers.data(), embed, head, norm) != 0) return fail("setup", err);
    max_tokens_ = opt.max_tokens;
    vocab_ = s.vocab;
    context_ = s.context;
    dir_ = dir;
    // what a state of this model holds (engine/src/model.cpp:351-358: the attention layers' KV - the MTP layer's slot
    // after them when it is bound - the Gated DeltaNet layers' conv and recurrent states; with the MTP layer the last
    // hidden row too, engine/src/state.cpp:275)
    int n_attn = 0, n_gdn = 0;
    for (int l = 0; l < L; ++l) (types[static_cast<size_t>(l)].text() == "full_attention" ? n_attn : n_gdn)++;
    if (has_mtp_) ++n_attn;
    shapes_.mtp = has_mtp_ ? 1u : 0u;
    const uint64_t conv_dim = 2ull * s.gdn_k_heads * s.gdn_k_dim + static_cast<uint64_t>(s.gdn_v_heads) * s.gdn_v_dim;
    shapes_.n_attn = static_cast<uint32_t>(n_attn);
    shapes_.kv_heads = static_cast<uint32_t>(s.n_kv_heads);
    shapes_.kv_row = static_cast<uint32_t>(s.n_kv_heads * s.head_dim);
    shapes_.hidden = static_cast<uint32_t>(s.hidden);
    shapes_.n_layers = static_cast<uint32_t>(L);
    shapes_.conv_n = static_cast<uint64_t>(n_gdn) * conv_dim * static_cast<uint64_t>(std::max(0, s.conv_kernel - 1));
    shapes_.gdn_n = static_cast<uint64_t>(n_gdn) * s.gdn_v_heads * s.gdn_k_dim * s.gdn_v_dim;
    text_only_ = true;
    const JsonRef tensors = pack_.manifest()["tensors"];
    for (size_t i = 0; i < tensors.size(); ++i)
        if (tensors.key_at(i).substr(0, 7) == "vision.") text_only_ = false;   // (engine/src/vision.cpp's tensors)
    conv_id_ = new_conversation_id(this);
    return true;
}

bool CudaModel::draft(const int *toks, int n, int pos, const float *hidden, int &draft, float *prob, std::string &err) {
    if (!g_ || !has_mtp_) {
        err = "no drafting: the pack has no MTP layer";
        return false;
    }
    return api_.draft(g_, toks, n, pos, hidden, &draft, prob, nullptr) == 0 || fail("draft", err);
}

bool CudaModel::draft_next(int tok, int pos, int &draft, float *prob, std::string &err) {
    if (!g_ || !has_mtp_) {
        err = "no drafting: the pack has no MTP layer";
        return false;
    }
    return api_.draft_next(g_, tok, pos, &draft, prob, nullptr) == 0 || fail("draft_next", err);
}

uint64_t CudaModel::state_fingerprint() const { return ghost::state_fingerprint(pack_print(dir_), shapes_); }

bool CudaModel::save_state(const std::string &path, bool append, int extra, int &code, std::string &err) {
    code = 1;   // (GHOST_E_ARG)
    if (!g_) {
        err = "not open";
        return false;
    }
    if (!text_only_) {
        err = "a pack with a vision encoder: its state holds the images' positions, which this backend does not keep";
        return false;
    }
    const int pos = position();
    const StateShapes &s = shapes_;
    std::vector<float> conv(std::max<uint64_t>(1, s.conv_n)), gdn(std::max<uint64_t>(1, s.gdn_n));
    std::vector<int8_t> kv(std::max<size_t>(1, static_cast<size_t>(s.n_attn) * 2 * pos * s.kv_row));
    std::vector<float> ks(std::max<size_t>(1, static_cast<size_t>(s.n_attn) * 2 * pos * s.kv_heads));
    code = 7;   // (GHOST_E_BACKEND)
    if (api_.state_get(g_, conv.data(), gdn.data(), kv.data(), ks.data(), pos) != 0) return fail("state_get", err);
    // the last hidden row when the engine would keep one (an MTP layer, a position, a row on the device)
    std::vector<float> hid;
    if (has_mtp_ && pos > 0) {
        hid.resize(s.hidden);
        if (api_.last_hidden(g_, hid.data()) != 0) hid.clear();
    }
    StateMeta m;
    m.position = pos;
    m.extra = extra;
    m.conv_id = conv_id_;
    code = 2;   // (GHOST_E_IO)
    if (!write_state(path, state_fingerprint(), s, m, conv.data(), gdn.data(), kv.data(), ks.data(),
                     hid.empty() ? nullptr : hid.data(), append, err))
        return false;
    code = 0;
    return true;
}

bool CudaModel::load_state(const std::string &path, int &extra, int &code, std::string &err) {
    code = 1;
    if (!g_) {
        err = "not open";
        return false;
    }
    auto refuse = [&](int c) {   // the conversation empty after any failure, as the engine's
        api_.reset(g_);
        conv_id_ = new_conversation_id(this);
        last_n_ = 0;
        code = c;
        return false;
    };
    if (!text_only_) {
        err = "a pack with a vision encoder: its state holds the images' positions, which this backend does not keep";
        return refuse(3);
    }
    StateMeta m;
    std::vector<float> conv, gdn, ks, hid;
    std::vector<int8_t> kv;
    const StateError e = read_state(path, state_fingerprint(), shapes_, context_, m, conv, gdn, kv, ks, hid, err);
    if (e != StateError::none) return refuse(e == StateError::format ? 3 : e == StateError::context ? 1 : 2);
    conv.resize(std::max<size_t>(1, conv.size()));
    gdn.resize(std::max<size_t>(1, gdn.size()));
    kv.resize(std::max<size_t>(1, kv.size()));
    ks.resize(std::max<size_t>(1, ks.size()));
    if (api_.state_put(g_, conv.data(), gdn.data(), kv.data(), ks.data(), m.position) != 0 ||
        (has_mtp_ && !hid.empty() && m.position > 0 && api_.put_last_hidden(g_, hid.data()) != 0)) {
        fail("state_put", err);
        return refuse(7);
    }
    conv_id_ = m.conv_id;
    extra = m.extra;
    last_n_ = 0;
    code = 0;
    return true;
}

bool CudaModel::verify_n(const int *toks, int n, float *logits, std::string &err) {
    if (!g_) {
        err = "not open";
        return false;
    }
    if (api_.verify(g_, toks, n, logits, nullptr) != 0) return fail("verify", err);
    last_n_ = n;
    return true;
}

bool CudaModel::reset(std::string &err) {
    if (!g_) {
        err = "not open";
        return false;
    }
    if (api_.reset(g_) != 0) return fail("reset", err);
    conv_id_ = new_conversation_id(this);
    last_n_ = 0;
    return true;
}

bool CudaModel::prefill(const int *toks, int n, std::string &err) {
    if (!g_) {
        err = "not open";
        return false;
    }
    if (!toks || n < 1) {
        err = "prefill: no tokens";
        return false;
    }
    // with the MTP layer, as the engine's prompt (engine/src/geode.cpp:132-150): after each chunk the layer over the
    // previous chunk's last position and the chunk's own but its last (each fed the token after it), so its KV holds
    // every prompt position but the last; that one's row stays for the first draft (gcuda_put_last_hidden: a draft of
    // the pending token at position n - 1 with hidden NULL takes it). A failed MTP pass only ends them, as there.
    bool spec = has_mtp_;
    std::vector<float> prev;
    const int H = static_cast<int>(shapes_.hidden);
    for (int i = 0; i < n; i += max_tokens_) {
        const int k = std::min(max_tokens_, n - i), p0 = position();
        if (api_.verify(g_, toks + i, k, nullptr, nullptr) != 0) return fail("prefill", err);
        if (!spec) continue;
        int d = 0;
        if (!prev.empty() && api_.draft(g_, toks + i, 1, p0 - 1, prev.data(), &d, nullptr, nullptr) != 0) spec = false;
        if (spec && k > 1 && api_.draft(g_, toks + i + 1, k - 1, p0, nullptr, &d, nullptr, nullptr) != 0) spec = false;
        prev.resize(static_cast<size_t>(H));
        if (spec && api_.last_hidden(g_, prev.data()) != 0) spec = false;
    }
    if (spec && !prev.empty() && api_.put_last_hidden(g_, prev.data()) != 0) return fail("prefill", err);
    last_n_ = 0;   // (nothing to accept or keep: the prompt is all kept)
    return true;
}

bool CudaModel::verify_keep(int kept, std::string &err) {
    if (!g_) {
        err = "not open";
        return false;
    }
    return api_.keep(g_, kept) == 0 || fail("keep", err);
}

bool CudaModel::accept(const SamplerParams &p, Sampler &s, SeenTokens &seen, const int *stops, int n_stops, int &kept,
                       int &next, std::string &err) {
    if (!g_ || last_n_ < 1) {
        err = "accept without a verified batch";
        return false;
    }
    gcuda_sampling sp{p.temperature, p.top_p, p.top_k, p.presence_penalty};
    double u[8] = {0};
    int samples[8] = {0};
    const bool sampled = p.temperature > 0.0f;
    if (sampled) s.peek(last_n_, u);   // row i's draw is the stream's i-th from here
    int k = 0, nx = 0;
    const std::vector<int> &sl = seen.list();
    if (api_.accept(g_, &sp, sampled ? u : nullptr, stops, n_stops, sl.data(), static_cast<int>(sl.size()), &k, &nx,
                    samples) != 0)
        return fail("accept", err);
    if (sampled) s.skip(k);   // the rows sampled: kept of them (the last one gave next)
    if (p.presence_penalty != 0.0f)
        for (int i = 0; i < k; ++i) seen.add(samples[i], vocab_);   // (every sampled row, as the engine's sample())
    kept = k;
    next = nx;
    return true;
}

bool CudaModel::step(const int *batch, int n, const SamplerParams &p, Sampler &s, SeenTokens &seen, const int *stops,
                     int n_stops, int &kept, int &next, std::string &err) {
    if (p.presence_penalty != 0.0f && n > 0) seen.add(batch[0], vocab_);
    if (!verify_n(batch, n, nullptr, err) || !accept(p, s, seen, stops, n_stops, kept, next, err)) return false;
    // (every draft stood: nothing to roll back, as the engine's loop; else the states as after row kept-1)
    return kept == n || verify_keep(kept, err);
}

bool pack_summary(const std::string &dir, std::string &out, std::string &err) {
    Pack p;
    if (!p.open(dir, err)) return false;
    const JsonRef c = p.config();
    size_t n = 0, q4 = 0, bytes = 0;
    const JsonRef tensors = p.manifest()["tensors"];
    for (size_t i = 0; i < tensors.size(); ++i) {
        TensorView t;
        if (!p.tensor(std::string(tensors.key_at(i)), t, err)) return false;
        ++n;
        q4 += t.type == "q4";
        bytes += t.bytes;
    }
    size_t expert_bytes = 0;
    if (p.manifest()["experts"]["layers"].present())
        for (size_t l = 0; l < p.manifest()["experts"]["layers"].size(); ++l) {
            ExpertTable e;
            if (!p.experts(static_cast<int>(l), e, err)) return false;
            expert_bytes += e.stride * static_cast<size_t>(c["num_experts"].integer());
        }
    out = "arch=" + p.arch() + " layers=" + std::to_string(c["num_hidden_layers"].integer()) +
          " hidden=" + std::to_string(c["hidden_size"].integer()) + " vocab=" + std::to_string(c["vocab_size"].integer()) +
          " experts=" + std::to_string(c["num_experts"].integer()) + " tensors=" + std::to_string(n) +
          " q4=" + std::to_string(q4) + " bytes=" + std::to_string(bytes) + " expert_bytes=" + std::to_string(expert_bytes);
    return true;
}

}  // namespace ghost
