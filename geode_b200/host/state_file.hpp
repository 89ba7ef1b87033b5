// state_file.hpp - a conversation's state in the engine's own state file (Model::save_state / load_state,
// engine/src/state.cpp:1-17, 241-465), from and to host buffers in the layouts gcuda_state_get / gcuda_state_put
// take, so that a state saved by the reference engine (its CPU or GPU path) loads into the CUDA backend and back.
//
// The file: a 4096-byte header page (StateHeader, an FNV-1a checksum of its bytes last); at fixed_offset the fixed
// part - gen, the images' rotary positions (4 int32 each, image_cap of them), the last hidden state, the Gated
// DeltaNet conv states, their recurrent states, gen again; at kv_offset (the next 4096-byte boundary) the KV cache in
// blocks of 256 positions, each [K, V][attention layer][256][kv_row] int8 then their scales [K, V][layer][256]
// [kv_heads] f32. A whole write goes to path.tmp, renamed over path; an append (the same conversation, grown) writes
// the fixed part in place, the blocks from the one holding the last saved position on, the header last.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace ghost {

// What a state holds, as the engine's fingerprint lists it (engine/src/state.cpp:229-238): the KV element size (1:
// int8 rows with a scale a position and KV head - the only format this backend keeps), the attention layers (with
// the MTP layer's slot when there is one, engine/src/model.cpp:354), KV heads, row elements, the conv and recurrent
// state floats, the hidden size, the layers, an MTP layer, a vision encoder (never: this backend verifies text).
struct StateShapes {
    uint32_t n_attn = 0, kv_heads = 0, kv_row = 0, hidden = 0, n_layers = 0;
    uint64_t conv_n = 0, gdn_n = 0;
    uint32_t mtp = 0;
};

// The conversation around the buffers.
struct StateMeta {
    int32_t position = 0;   // the tokens computed (KV rows)
    int32_t extra = -1;     // the caller's: the token passed on but not computed yet (-1: none)
    uint64_t conv_id = 0;   // the conversation (an append goes only to its own file)
};

// FNV-1a 64 of the pack's geode.json (1 when it hashes to 0, as the engine), then of the shapes.
uint64_t pack_print(const std::string &pack_dir);
uint64_t state_fingerprint(uint64_t pack_print, const StateShapes &s);

// A new conversation's id (the engine's recipe: clocks, a counter and an address through a 64-bit mixer).
uint64_t new_conversation_id(const void *salt);

// Writes the state. kv: [n_attn][2][position][kv_row] int8, kv_scale: [n_attn][2][position][kv_heads] f32 (the
// gcuda_state_get layouts); conv, gdn: the reference's own buffers; hidden: the last position's row after the final
// norm (has_hidden, engine/src/state.cpp:275), or NULL for none. append: as the engine's (falls back to a whole write
// when the file at path is not an earlier state of this conversation in this shape).
bool write_state(const std::string &path, uint64_t fingerprint, const StateShapes &s, const StateMeta &m,
                 const float *conv, const float *gdn, const int8_t *kv, const float *kv_scale, const float *hidden,
                 bool append, std::string &err);

// The header of a state file, checked against this model (magic, version, checksum, fingerprint, shapes, the file's
// length, the fixed part's gen at both ends) and the context (position < context); fills m.
enum class StateError { none, io, format, context };
StateError peek_state(const std::string &path, uint64_t fingerprint, const StateShapes &s, int context, StateMeta &m,
                      std::string &err);
// peek_state, then the buffers (sized for m.position as write_state's); hidden: the file's last hidden row, empty
// when it has none.
StateError read_state(const std::string &path, uint64_t fingerprint, const StateShapes &s, int context, StateMeta &m,
                      std::vector<float> &conv, std::vector<float> &gdn, std::vector<int8_t> &kv,
                      std::vector<float> &kv_scale, std::vector<float> &hidden, std::string &err);

}  // namespace ghost
