// state_file.cpp - see state_file.hpp.
//
// What has to match the engine (engine/src/state.cpp) is the file's bytes: the magic, the version, the header's
// fields in their order and natural alignment, the FNV-1a checksum and fingerprint with the engine's starting value,
// the order and sizes of the fixed part's pieces, the 4096-byte page rule and the 256-position KV blocks, and the
// append rule. The code around them is this file's own: a read maps the whole file and checks every piece against
// the mapped length before it copies anything out; a write goes through stdio with an fsync between the stages whose
// order makes a save crash-safe (states, then the fixed part's closing gen, then the KV blocks, then the header).
#include "state_file.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <random>

namespace ghost {

namespace {

// ---- the format --------------------------------------------------------------------------------------------------

constexpr char kMagic[8] = {'G', 'E', 'O', 'D', 'E', 'S', 'T', 'A'};
constexpr uint32_t kFormatVersion = 1;
constexpr uint32_t kBlockPositions = 256;   // positions per KV block
constexpr uint64_t kPageBytes = 4096;       // the header's page; the KV blocks start on a page boundary
constexpr uint32_t kImageSlots = 16;        // rotary-position slots for images in a conversation that has none

struct Header {
    char magic[8];
    uint32_t version, header_size;
    uint64_t fingerprint, conv_id, gen;
    int32_t position, extra, rope_delta;
    uint32_t n_images, image_cap;
    uint32_t kv_elem, n_attn, kv_heads, kv_row, hidden, has_hidden, block;
    uint64_t conv_n, gdn_n;
    uint64_t fixed_offset, fixed_bytes, kv_offset, block_bytes;
    uint64_t checksum;   // FNV-1a of every byte before it
};
static_assert(sizeof(Header) == 144 && offsetof(Header, position) == 40 && offsetof(Header, conv_n) == 88 &&
                  offsetof(Header, checksum) == 136,
              "the header's bytes are the engine's");

// FNV-1a 64 from the engine's starting value 1469598103934665603 (it differs from the published offset basis,
// 14695981039346656037, by a dropped digit; files carry the engine's value, so this one is kept).
struct Fnv {
    uint64_t h = 1469598103934665603ull;
    Fnv &add(const void *data, size_t n) {
        const auto *p = static_cast<const uint8_t *>(data);
        for (const uint8_t *e = p + n; p != e; ++p) h = (h ^ *p) * 1099511628211ull;
        return *this;
    }
};

uint64_t checksum_of(const Header &h) { return Fnv().add(&h, offsetof(Header, checksum)).h; }

uint64_t round_up(uint64_t x, uint64_t to) { return (x + to - 1) / to * to; }

// The fixed part, piece by piece from fixed_offset: gen, the images' rotary positions (4 int32 per slot), the last
// hidden row, the conv states, the recurrent states, gen again. The KV blocks follow at the next page boundary.
struct Pieces {
    uint64_t gen_lead = 0, images = 0, hidden = 0, conv = 0, recurrent = 0, gen_trail = 0, end = 0, kv = 0;
};
Pieces pieces_of(const Header &h) {
    Pieces p;
    uint64_t cursor = h.fixed_offset;
    auto take = [&cursor](uint64_t bytes) {
        const uint64_t at = cursor;
        cursor += bytes;
        return at;
    };
    p.gen_lead = take(sizeof(uint64_t));
    p.images = take(uint64_t{h.image_cap} * 4 * sizeof(int32_t));
    p.hidden = take(uint64_t{h.hidden} * sizeof(float));
    p.conv = take(h.conv_n * sizeof(float));
    p.recurrent = take(h.gdn_n * sizeof(float));
    p.gen_trail = take(sizeof(uint64_t));
    p.end = cursor;
    p.kv = round_up(cursor, kPageBytes);
    return p;
}

// A block: [K, V][attention layer][kBlockPositions][kv_row] int8, then [K, V][layer][kBlockPositions][kv_heads] f32.
uint64_t block_size(const StateShapes &s, uint64_t positions) {
    return 2 * uint64_t{s.n_attn} * positions * (uint64_t{s.kv_row} + uint64_t{s.kv_heads} * sizeof(float));
}

// Visits the (K|V, layer) segments of block b (of `per_block` positions) for a conversation of `positions`
// positions: for each, the segment's index in the block's order (K|V major, then layer), the index of the same rows'
// run in the callers' arrays ([layer][K|V][positions]), the first position and how many the block holds.
template <typename Fn>
void for_each_segment(const StateShapes &s, size_t per_block, size_t positions, size_t b, Fn &&fn) {
    const size_t p0 = b * per_block, run = std::min<size_t>(positions, p0 + per_block) - p0;
    for (size_t half = 0; half < 2; ++half)
        for (size_t layer = 0; layer < s.n_attn; ++layer)
            fn(half * s.n_attn + layer, layer * 2 + half, p0, run);
}

// ---- reading -----------------------------------------------------------------------------------------------------

// A whole file mapped read-only (empty when it cannot be opened or mapped).
class MappedFile {
public:
    explicit MappedFile(const std::string &path) {
        const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
        if (fd < 0) return;
        opened_ = true;
        struct stat st {};
        if (fstat(fd, &st) == 0 && st.st_size > 0) {
            void *p = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_SHARED, fd, 0);
            if (p != MAP_FAILED) {
                base_ = static_cast<const uint8_t *>(p);
                size_ = static_cast<uint64_t>(st.st_size);
            }
        }
        ::close(fd);
    }
    ~MappedFile() {
        if (base_) munmap(const_cast<uint8_t *>(base_), size_);
    }
    MappedFile(const MappedFile &) = delete;
    MappedFile &operator=(const MappedFile &) = delete;

    bool opened() const { return opened_; }
    uint64_t size() const { return size_; }
    // bytes [at, at + n) if the file holds them
    const uint8_t *span(uint64_t at, uint64_t n) const {
        return base_ && at <= size_ && n <= size_ - at ? base_ + at : nullptr;
    }

private:
    bool opened_ = false;
    const uint8_t *base_ = nullptr;
    uint64_t size_ = 0;
};

// The header of a mapped file when it is one of this format: false, and why, otherwise.
bool header_in(const MappedFile &f, Header &h, std::string &why) {
    const uint8_t *p = f.span(0, sizeof(Header));
    if (!p) {
        why = "the file is shorter than a state file's header";
        return false;
    }
    std::memcpy(&h, p, sizeof h);
    if (std::memcmp(h.magic, kMagic, sizeof kMagic) != 0) {
        why = "the file is not a state file (its magic differs)";
        return false;
    }
    if (h.version != kFormatVersion || h.header_size != sizeof(Header)) {
        why = "the state file has format version " + std::to_string(h.version) + "; this reader takes version " +
              std::to_string(kFormatVersion);
        return false;
    }
    if (checksum_of(h) != h.checksum) {
        why = "the state file's header fails its checksum";
        return false;
    }
    return true;
}

// The header checked against this model and context, then the file's pieces against the header and the file's
// length; the mapped file stays open for the caller's copies.
StateError validate(const MappedFile &f, const std::string &path, uint64_t fingerprint, const StateShapes &s,
                    int context, Header &h, std::string &err) {
    if (!f.opened()) {
        err = "cannot open " + path;
        return StateError::io;
    }
    if (!header_in(f, h, err)) return StateError::format;
    const bool same_model = h.fingerprint == fingerprint && h.kv_elem == 1 && h.n_attn == s.n_attn &&
                            h.kv_heads == s.kv_heads && h.kv_row == s.kv_row && h.hidden == s.hidden &&
                            h.conv_n == s.conv_n && h.gdn_n == s.gdn_n && h.block != 0;
    if (!same_model) {
        err = "the state file belongs to a different model (or a different KV cache format)";
        return StateError::format;
    }
    if (h.position < 0 || h.position >= context) {
        err = "the state file holds " + std::to_string(h.position) + " positions; this context has room for " +
              std::to_string(context);
        return StateError::context;
    }
    const Pieces p = pieces_of(h);
    const uint64_t blocks = (uint64_t(h.position) + h.block - 1) / h.block;
    const bool whole = p.end - h.fixed_offset == h.fixed_bytes && p.kv == h.kv_offset && h.n_images <= h.image_cap &&
                       h.block_bytes == block_size(s, h.block) && f.span(h.kv_offset, blocks * h.block_bytes) &&
                       f.span(h.fixed_offset, h.fixed_bytes);
    if (!whole) {
        err = "the state file is truncated or its pieces do not add up";
        return StateError::io;
    }
    uint64_t lead = 0, trail = 0;
    std::memcpy(&lead, f.span(p.gen_lead, sizeof lead), sizeof lead);
    std::memcpy(&trail, f.span(p.gen_trail, sizeof trail), sizeof trail);
    if (lead != h.gen || trail != h.gen) {
        err = "the state file was left half-written (a save did not finish)";
        return StateError::io;
    }
    if (h.n_images > 0) {   // a conversation with images needs the vision encoder this backend does not run
        err = "the state file holds images, which this text-only model cannot resume";
        return StateError::format;
    }
    return StateError::none;
}

// ---- writing -----------------------------------------------------------------------------------------------------

// stdio at byte offsets, with fsync for the points whose order matters.
class Writer {
public:
    Writer(const std::string &path, bool fresh) : f_(std::fopen(path.c_str(), fresh ? "wb" : "r+b")) {}
    ~Writer() { close(); }
    Writer(const Writer &) = delete;
    Writer &operator=(const Writer &) = delete;

    bool ok() const { return f_ != nullptr && good_; }
    Writer &put(uint64_t at, const void *data, size_t n) {
        if (ok() && n > 0)
            good_ = fseeko(f_, static_cast<off_t>(at), SEEK_SET) == 0 && std::fwrite(data, 1, n, f_) == n;
        return *this;
    }
    Writer &durable() {
        if (ok()) good_ = std::fflush(f_) == 0 && ::fsync(fileno(f_)) == 0;
        return *this;
    }
    bool close() {
        if (!f_) return good_;
        good_ = std::fclose(f_) == 0 && good_;
        f_ = nullptr;
        return good_;
    }

private:
    std::FILE *f_;
    bool good_ = true;
};

}  // namespace

uint64_t pack_print(const std::string &pack_dir) {
    std::ifstream in(pack_dir + "/geode.json", std::ios::binary);
    const std::string bytes((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
    const uint64_t h = Fnv().add(bytes.data(), bytes.size()).h;
    return h ? h : 1;   // (0 would read as "not computed yet" in the engine)
}

uint64_t state_fingerprint(uint64_t print, const StateShapes &s) {
    // the engine's list, in its order: version, KV element bytes (1: int8), attention layers, KV heads, row elements,
    // conv floats, recurrent floats, hidden, layers, an MTP layer (0 / 1), a vision encoder (0)
    const uint64_t shapes[] = {kFormatVersion, 1u, s.n_attn, s.kv_heads, s.kv_row, s.conv_n, s.gdn_n, s.hidden,
                               s.n_layers, s.mtp ? 1u : 0u, 0u};
    Fnv f;
    f.h = print;
    return f.add(shapes, sizeof shapes).h;
}

uint64_t new_conversation_id(const void *salt) {
    // 64 bits from the system's entropy source, with the caller's address folded in so that two ids drawn in one
    // process differ even if that source repeats
    std::random_device rd;
    const uint64_t r = (uint64_t{rd()} << 32) ^ uint64_t{rd()};
    return r ^ (reinterpret_cast<uintptr_t>(salt) * 0xD6E8FEB86659FD93ull);
}

bool write_state(const std::string &path, uint64_t fingerprint, const StateShapes &s, const StateMeta &m,
                 const float *conv, const float *gdn, const int8_t *kv, const float *kv_scale, const float *hidden,
                 bool append, std::string &err) {
    const bool missing = (m.position > 0 && s.n_attn > 0 && (!kv || !kv_scale)) || (s.conv_n && !conv) ||
                         (s.gdn_n && !gdn);
    if (m.position < 0 || missing) {
        err = "write_state: a negative position or a missing buffer";
        return false;
    }
    Header h{};
    std::memcpy(h.magic, kMagic, sizeof kMagic);
    h.version = kFormatVersion;
    h.header_size = sizeof(Header);
    h.fingerprint = fingerprint;
    h.conv_id = m.conv_id;
    h.gen = 1;
    h.position = m.position;
    h.extra = m.extra;
    h.image_cap = kImageSlots;
    h.kv_elem = 1;
    h.n_attn = s.n_attn;
    h.kv_heads = s.kv_heads;
    h.kv_row = s.kv_row;
    h.hidden = s.hidden;
    h.has_hidden = hidden ? 1 : 0;
    h.block = kBlockPositions;
    h.conv_n = s.conv_n;
    h.gdn_n = s.gdn_n;
    h.fixed_offset = kPageBytes;
    h.block_bytes = block_size(s, kBlockPositions);

    // An append needs the file to hold an earlier save of this same conversation and shape; it then rewrites the
    // fixed part in place and the KV blocks from the one holding the earlier save's last position.
    size_t first_block = 0;
    bool in_place = false;
    if (append) {
        MappedFile old_file(path);
        Header old{};
        std::string why;
        if (header_in(old_file, old, why) && old.fingerprint == h.fingerprint && old.conv_id == h.conv_id &&
            old.position <= h.position && old.image_cap >= h.n_images && old.block == h.block &&
            old.block_bytes == h.block_bytes && old.fixed_offset == h.fixed_offset) {
            in_place = true;
            h.image_cap = old.image_cap;
            h.gen = old.gen + 1;
            first_block = static_cast<size_t>(std::max(0, old.position - 1)) / kBlockPositions;
        }
    }
    const Pieces p = pieces_of(h);
    h.fixed_bytes = p.end - h.fixed_offset;
    h.kv_offset = p.kv;
    h.checksum = checksum_of(h);

    const std::string target = in_place ? path : path + ".tmp";
    Writer w(target, !in_place);
    auto give_up = [&](const std::string &stage) {
        w.close();
        if (!in_place) std::remove(target.c_str());
        err = "writing " + target + " failed at " + stage;
        return false;
    };
    if (!w.ok()) return give_up("open");

    // 1. the fixed part up to the states (gen, empty image slots, the hidden row or zeros), the states, then - once
    //    those are on disk - the closing gen, so a reader sees both gens equal only after a finished state write
    std::vector<uint8_t> lead(static_cast<size_t>(p.conv - p.gen_lead), 0);
    std::memcpy(lead.data(), &h.gen, sizeof h.gen);
    if (hidden) std::memcpy(lead.data() + (p.hidden - p.gen_lead), hidden, size_t{s.hidden} * sizeof(float));
    w.put(p.gen_lead, lead.data(), lead.size())
        .put(p.conv, conv, s.conv_n * sizeof(float))
        .put(p.recurrent, gdn, s.gdn_n * sizeof(float))
        .durable()
        .put(p.gen_trail, &h.gen, sizeof h.gen);
    if (!w.ok()) return give_up("the states");

    // 2. the KV blocks (the callers' [layer][K|V][position] runs regrouped per block), a few MiB at a time
    const size_t P = static_cast<size_t>(m.position), blocks = (P + kBlockPositions - 1) / kBlockPositions;
    if (s.n_attn > 0 && blocks > first_block) {
        const size_t bb = static_cast<size_t>(h.block_bytes), row = s.kv_row, heads = s.kv_heads;
        const size_t scale_at = 2 * size_t{s.n_attn} * kBlockPositions * row;
        const size_t batch = std::max<size_t>(1, (size_t{16} << 20) / bb);
        std::vector<uint8_t> buf;
        for (size_t b0 = first_block; b0 < blocks; b0 += batch) {
            const size_t nb = std::min(batch, blocks - b0);
            buf.assign(nb * bb, 0);
            for (size_t b = b0; b < b0 + nb; ++b) {
                uint8_t *blk = buf.data() + (b - b0) * bb;
                for_each_segment(s, kBlockPositions, P, b, [&](size_t seg, size_t src, size_t p0, size_t run) {
                    std::memcpy(blk + seg * kBlockPositions * row, kv + (src * P + p0) * row, run * row);
                    std::memcpy(blk + scale_at + seg * kBlockPositions * heads * sizeof(float),
                                kv_scale + (src * P + p0) * heads, run * heads * sizeof(float));
                });
            }
            w.put(h.kv_offset + b0 * bb, buf.data(), buf.size());
            if (!w.ok()) return give_up("the KV cache");
        }
    }

    // 3. the header, once everything it describes is on disk
    w.durable().put(0, &h, sizeof h).durable();
    if (!w.ok() || !w.close()) return give_up("the header");
    if (!in_place && std::rename(target.c_str(), path.c_str()) != 0) {
        std::remove(target.c_str());
        err = "renaming " + target + " to " + path + " failed";
        return false;
    }
    return true;
}

StateError peek_state(const std::string &path, uint64_t fingerprint, const StateShapes &s, int context, StateMeta &m,
                      std::string &err) {
    const MappedFile f(path);
    Header h{};
    const StateError e = validate(f, path, fingerprint, s, context, h, err);
    if (e == StateError::none) m = StateMeta{h.position, h.extra, h.conv_id};
    return e;
}

StateError read_state(const std::string &path, uint64_t fingerprint, const StateShapes &s, int context, StateMeta &m,
                      std::vector<float> &conv, std::vector<float> &gdn, std::vector<int8_t> &kv,
                      std::vector<float> &kv_scale, std::vector<float> &hidden, std::string &err) {
    const MappedFile f(path);
    Header h{};
    const StateError e = validate(f, path, fingerprint, s, context, h, err);
    if (e != StateError::none) return e;
    const Pieces p = pieces_of(h);
    const size_t P = static_cast<size_t>(h.position), row = s.kv_row, heads = s.kv_heads;
    conv.resize(s.conv_n);
    gdn.resize(s.gdn_n);
    std::memcpy(conv.data(), f.span(p.conv, s.conv_n * sizeof(float)), s.conv_n * sizeof(float));
    std::memcpy(gdn.data(), f.span(p.recurrent, s.gdn_n * sizeof(float)), s.gdn_n * sizeof(float));
    hidden.clear();
    if (h.has_hidden) {
        hidden.resize(s.hidden);
        std::memcpy(hidden.data(), f.span(p.hidden, size_t{s.hidden} * sizeof(float)), size_t{s.hidden} * sizeof(float));
    }
    kv.assign(size_t{s.n_attn} * 2 * P * row, 0);
    kv_scale.assign(size_t{s.n_attn} * 2 * P * heads, 0.0f);
    const size_t B = h.block, blocks = (P + B - 1) / B, bb = static_cast<size_t>(h.block_bytes);
    const size_t scale_at = 2 * size_t{s.n_attn} * B * row;
    for (size_t b = 0; b < blocks && s.n_attn > 0; ++b) {
        const uint8_t *blk = f.span(h.kv_offset + b * bb, bb);   // (validate checked that every block is there)
        for_each_segment(s, B, P, b, [&](size_t seg, size_t dst, size_t p0, size_t run) {
            std::memcpy(kv.data() + (dst * P + p0) * row, blk + seg * B * row, run * row);
            std::memcpy(kv_scale.data() + (dst * P + p0) * heads, blk + scale_at + seg * B * heads * sizeof(float),
                        run * heads * sizeof(float));
        });
    }
    m = StateMeta{h.position, h.extra, h.conv_id};
    return StateError::none;
}

}  // namespace ghost
