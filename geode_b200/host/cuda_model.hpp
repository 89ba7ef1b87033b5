// cuda_model.hpp - the host side of the CUDA backend: the engine's Model seam for the speculative verify step
// (Model::verify_n / verify_keep / can_verify / spec_tokens, engine/src/model.hpp:189-205), its Sampler's uniform
// stream (engine/src/sampler.hpp) and the acceptance rule of the speculation loop (engine/src/geode.cpp:327-350),
// over libgeode_cuda.so. The backend library is loaded at run time into a table of its C functions, as the engine
// loads its NPU backend (dlopen + dlsym, engine/src/model.cpp:2255-2320), so the engine needs no CUDA at build time.
#pragma once

#include <cstdint>
#include <random>
#include <string>
#include <vector>

#include "../../include/geode_cuda.h"
#include "pack.hpp"
#include "state_file.hpp"

namespace ghost {

// The C functions of libgeode_cuda.so this host calls.
struct CudaApi {
    void *lib = nullptr;
    decltype(&gcuda_open) open = nullptr;
    decltype(&gcuda_close) close = nullptr;
    decltype(&gcuda_last_error) last_error = nullptr;
    decltype(&gcuda_adopt_q4) adopt_q4 = nullptr;
    decltype(&gcuda_adopt_raw) adopt_raw = nullptr;
    decltype(&gcuda_adopt_embedding) adopt_embedding = nullptr;
    decltype(&gcuda_adopt_experts) adopt_experts = nullptr;
    decltype(&gcuda_setup) setup = nullptr;
    decltype(&gcuda_verify) verify = nullptr;
    decltype(&gcuda_keep) keep = nullptr;
    decltype(&gcuda_position) position = nullptr;
    decltype(&gcuda_accept) accept = nullptr;
    decltype(&gcuda_state_get) state_get = nullptr;
    decltype(&gcuda_state_put) state_put = nullptr;
    decltype(&gcuda_reset) reset = nullptr;
    decltype(&gcuda_set_mtp) set_mtp = nullptr;
    decltype(&gcuda_set_draft_head) set_draft_head = nullptr;
    decltype(&gcuda_last_hidden) last_hidden = nullptr;
    decltype(&gcuda_put_last_hidden) put_last_hidden = nullptr;
    decltype(&gcuda_draft) draft = nullptr;
    decltype(&gcuda_draft_next) draft_next = nullptr;
    // path: the library file; empty = libgeode_cuda.so beside this library
    bool load(const std::string &path, std::string &err);
    ~CudaApi();
};

struct ModelOptions {
    int device = 0;
    int context = 0;      // positions of KV cache; 0 = 4096
    int max_tokens = 5;   // the largest verify batch (1 accepted + max_tokens - 1 drafts), <= 8
};

struct SamplerParams {
    float temperature = 0.0f;        // 0 = greedy
    float top_p = 1.0f;              // 1 = off
    int top_k = 0;                   // 0 = off (1024 candidates)
    float presence_penalty = 0.0f;   // 0 = off (geode_sampling's, engine/src/geode.cpp:234-255)
};

// The answer's sampled tokens for the presence penalty (geode_generate's seen / is_seen, engine/src/geode.cpp:
// 234-255): each id once, in the order first sampled; cleared when a generation starts.
class SeenTokens {
public:
    void clear() {
        list_.clear();
        mark_.clear();
    }
    void add(int tok, int vocab) {
        if (tok < 0 || tok >= vocab) return;
        if (mark_.size() < static_cast<size_t>(vocab)) mark_.resize(static_cast<size_t>(vocab), 0);
        if (mark_[static_cast<size_t>(tok)]) return;
        mark_[static_cast<size_t>(tok)] = 1;
        list_.push_back(tok);
    }
    const std::vector<int> &list() const { return list_; }

private:
    std::vector<int> list_;
    std::vector<uint8_t> mark_;
};

// The reference sampler's random stream: std::mt19937_64 seeded once per generate call, one
// uniform_real_distribution<double>(0, 1) draw (generate_canonical<double, 53>) for each row it samples.
class Sampler {
public:
    void seed(uint64_t s) { rng_.seed(s); }
    double uniform() { return std::generate_canonical<double, 53>(rng_); }
    // the next n draws without consuming them
    void peek(int n, double *out) const {
        std::mt19937_64 copy = rng_;
        for (int i = 0; i < n; ++i) out[i] = std::generate_canonical<double, 53>(copy);
    }
    void skip(int n) {
        for (int i = 0; i < n; ++i) uniform();
    }

private:
    std::mt19937_64 rng_;
};

class CudaModel {
public:
    CudaModel() = default;
    CudaModel(const CudaModel &) = delete;
    CudaModel &operator=(const CudaModel &) = delete;
    ~CudaModel();

    bool open(const std::string &dir, const ModelOptions &opt, std::string &err);
    bool can_verify() const { return g_ != nullptr; }
    int spec_tokens() const { return max_tokens_ - 1; }   // drafts a verify batch can carry
    int position() const;
    int vocab() const { return vocab_; }

    // n tokens at positions pos .. pos+n-1 through every layer; logits [n][vocab] (or NULL); position += n
    bool verify_n(const int *toks, int n, float *logits, std::string &err);
    // Model::reset / geode_reset: the conversation empty (position 0, zero states), a new conversation id
    bool reset(std::string &err);
    // geode_prefill (engine/include/geode/geode.h:166-169): n prompt tokens appended to the conversation, no logits -
    // through the verify graphs, max_tokens positions a launch (not a tensor-core prefill: the GEMVs' weight stream
    // is read once per max_tokens tokens)
    bool prefill(const int *toks, int n, std::string &err);
    // rollback: the states as after the verified batch's row kept-1 (1 <= kept < n); position -= n - kept
    bool verify_keep(int kept, std::string &err);
    // the acceptance of the last verified batch (its rows 1.. are the drafts): kept, next (-1: a stop token stood);
    // with a presence penalty the rows are penalised for `seen`, and the rows' samples are added to it
    bool accept(const SamplerParams &p, Sampler &s, SeenTokens &seen, const int *stops, int n_stops, int &kept,
                int &next, std::string &err);
    // one speculation step: verify_n(batch), accept, verify_keep(kept) unless every draft stood. batch[0] is the
    // answer's last sampled token: with a presence penalty it joins `seen` first (a no-op after the first step,
    // whose batch[0] is the previous step's next)
    bool step(const int *batch, int n, const SamplerParams &p, Sampler &s, SeenTokens &seen, const int *stops,
              int n_stops, int &kept, int &next, std::string &err);

    // Model::draft / draft_next (engine/src/model.cpp:1295-1480) on the device's MTP layer: the MTP pass over the
    // positions pos .. pos+n-1 (toks: the tokens after them; hidden: n rows, or NULL for the last verified batch's),
    // the greedy draft from the last position and its softmax probability (prob may be NULL); draft_next: one chained
    // position from the last pass's own output row. False when the pack has no MTP layer.
    bool has_mtp() const { return has_mtp_; }
    bool draft(const int *toks, int n, int pos, const float *hidden, int &draft, float *prob, std::string &err);
    bool draft_next(int tok, int pos, int &draft, float *prob, std::string &err);

    // Model::save_state / load_state (engine/src/state.cpp:241-465) in the engine's state file: the device's KV rows
    // and recurrent states through the host (gcuda_state_get / gcuda_state_put), so a state saved by the reference
    // engine (CPU or GPU path) continues here and back. extra: the caller's token passed on but not computed yet.
    // A failed load leaves the conversation empty (position 0), as the engine's. With an MTP layer the file holds that
    // layer's KV rows and the last hidden row (a load gives the row back to the device for the next draft); packs
    // with a vision encoder are refused (their states hold the images' positions, which this backend does not keep).
    // code: 0, or GHOST_E_IO / GHOST_E_FORMAT / GHOST_E_ARG as include/geode_host.h lists them.
    bool save_state(const std::string &path, bool append, int extra, int &code, std::string &err);
    bool load_state(const std::string &path, int &extra, int &code, std::string &err);
    // the shapes the state file records and the fingerprint it carries for this pack
    const StateShapes &state_shapes() const { return shapes_; }
    uint64_t state_fingerprint() const;

private:
    bool fail(const char *what, std::string &err);
    CudaApi api_;
    Pack pack_;
    gcuda *g_ = nullptr;
    int max_tokens_ = 5, vocab_ = 0, last_n_ = 0, context_ = 0;
    std::string dir_;
    StateShapes shapes_;
    bool text_only_ = true;    // no vision encoder in the pack
    bool has_mtp_ = false;     // the MTP layer is on the device (gcuda_set_mtp)
    uint64_t conv_id_ = 0;     // the conversation (new at open and after a failed load; a loaded state's)
};

// The manifest as this host reads it, one line (tests): arch, layers, hidden, vocab, experts, tensor counts, bytes.
bool pack_summary(const std::string &dir, std::string &out, std::string &err);

}  // namespace ghost
