// state_file.cpp - see state_file.hpp.
#include "state_file.hpp"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>

namespace ghost {

namespace {

constexpr char kMagic[8] = {'G', 'E', 'O', 'D', 'E', 'S', 'T', 'A'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kBlock = 256;      // positions in a KV block of the file (engine/src/state.cpp:46)
constexpr uint64_t kPage = 4096;      // the header's page; the KV blocks start on a page boundary
constexpr uint32_t kImageCap = 16;    // image slots of a conversation without images (engine/src/state.cpp:282)
constexpr size_t kIoBytes = 16u << 20;

// The header's fields in the engine's order (engine/src/state.cpp:50-63); the file holds the machine's own layout
// (little-endian, natural alignment), so the offsets are pinned here.
struct Header {
    char magic[8];
    uint32_t version, header_size;
    uint64_t fingerprint, conv_id, gen;
    int32_t position, extra, rope_delta;
    uint32_t n_images, image_cap;
    uint32_t kv_elem, n_attn, kv_heads, kv_row, hidden, has_hidden, block;
    uint64_t conv_n, gdn_n;
    uint64_t fixed_offset, fixed_bytes, kv_offset, block_bytes;
    uint64_t checksum;
};
static_assert(sizeof(Header) == 144 && offsetof(Header, position) == 40 && offsetof(Header, conv_n) == 88 &&
                  offsetof(Header, checksum) == 136,
              "the engine's header layout");

// FNV-1a, 64-bit, from the engine's starting value: 1469598103934665603 (engine/src/state.cpp:66). That is not the
// published FNV offset basis (14695981039346656037, one digit longer); the files carry the engine's, so it is kept.
constexpr uint64_t kFnvStart = 1469598103934665603ull;
constexpr uint64_t kFnvPrime = 1099511628211ull;
uint64_t fnv(const void *data, size_t n, uint64_t h = kFnvStart) {
    const auto *p = static_cast<const uint8_t *>(data);
    for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * kFnvPrime;
    return h;
}
uint64_t header_sum(const Header &h) { return fnv(&h, offsetof(Header, checksum)); }

uint64_t page_up(uint64_t x) { return (x + kPage - 1) / kPage * kPage; }

// where the fixed part's pieces lie
struct Layout {
    uint64_t images, hidden, conv, gdn, trail, fixed_bytes, kv_offset;
};
Layout layout_of(const Header &h) {
    Layout L{};
    L.images = h.fixed_offset + sizeof(uint64_t);
    L.hidden = L.images + static_cast<uint64_t>(h.image_cap) * 4 * sizeof(int32_t);
    L.conv = L.hidden + static_cast<uint64_t>(h.hidden) * sizeof(float);
    L.gdn = L.conv + h.conv_n * sizeof(float);
    L.trail = L.gdn + h.gdn_n * sizeof(float);
    L.fixed_bytes = L.trail + sizeof(uint64_t) - h.fixed_offset;
    L.kv_offset = page_up(h.fixed_offset + L.fixed_bytes);
    return L;
}

uint64_t block_bytes(const StateShapes &s, uint64_t block) {
    return 2 * static_cast<uint64_t>(s.n_attn) * block * (s.kv_row + static_cast<uint64_t>(s.kv_heads) * sizeof(float));
}

// A file read and written at offsets.
class File {
public:
    ~File() { close(); }
    bool open(const std::string &path, bool write, bool create) {
        int flags = O_CLOEXEC | (write ? O_RDWR : O_RDONLY);
        if (create) flags |= O_CREAT | O_TRUNC;
        fd_ = ::open(path.c_str(), flags, 0600);
        return fd_ >= 0;
    }
    void close() {
        if (fd_ >= 0) ::close(fd_);
        fd_ = -1;
    }
    uint64_t size() const {
        struct stat st {};
        return fstat(fd_, &st) == 0 && st.st_size > 0 ? static_cast<uint64_t>(st.st_size) : 0;
    }
    bool write(uint64_t off, const void *data, size_t n) {
        const auto *p = static_cast<const uint8_t *>(data);
        while (n > 0) {
            const ssize_t w = ::pwrite(fd_, p, std::min<size_t>(n, 1u << 30), static_cast<off_t>(off));
            if (w <= 0) return false;
            p += w;
            off += static_cast<uint64_t>(w);
            n -= static_cast<size_t>(w);
        }
        return true;
    }
    bool read(uint64_t off, void *data, size_t n) {
        auto *p = static_cast<uint8_t *>(data);
        while (n > 0) {
            const ssize_t r = ::pread(fd_, p, std::min<size_t>(n, 1u << 30), static_cast<off_t>(off));
            if (r <= 0) return false;
            p += r;
            off += static_cast<uint64_t>(r);
            n -= static_cast<size_t>(r);
        }
        return true;
    }
    bool sync() { return ::fsync(fd_) == 0; }

private:
    int fd_ = -1;
};

// the header at the start of f, if it is one of this format (else err)
bool header_of(File &f, Header &h, std::string &err) {
    if (!f.read(0, &h, sizeof h)) {
        err = "not a saved conversation (too short)";
        return false;
    }
    if (std::memcmp(h.magic, kMagic, sizeof kMagic) != 0) {
        err = "not a saved conversation";
        return false;
    }
    if (h.version != kVersion || h.header_size != sizeof(Header)) {
        err = "a saved conversation of another version (" + std::to_string(h.version) + ")";
        return false;
    }
    if (h.checksum != header_sum(h)) {
        err = "the saved conversation's header is damaged";
        return false;
    }
    return true;
}

}  // namespace

uint64_t pack_print(const std::string &pack_dir) {
    uint64_t h = fnv(nullptr, 0);
    if (std::FILE *f = std::fopen((pack_dir + "/geode.json").c_str(), "rb")) {
        std::vector<char> buf(1 << 16);
        size_t n;
        while ((n = std::fread(buf.data(), 1, buf.size(), f)) > 0) h = fnv(buf.data(), n, h);
        std::fclose(f);
    }
    return h ? h : 1;
}

uint64_t state_fingerprint(uint64_t print, const StateShapes &s) {
    // the engine's list (engine/src/state.cpp:234-237): version, KV element bytes (1: int8), attention layers, KV
    // heads, row elements, conv floats, recurrent floats, hidden, layers, an MTP layer (0), a vision encoder (0)
    const uint64_t shapes[] = {kVersion, 1u, s.n_attn, s.kv_heads, s.kv_row, s.conv_n, s.gdn_n, s.hidden, s.n_layers,
                               0u, 0u};
    return fnv(shapes, sizeof shapes, print);
}

uint64_t new_conversation_id(const void *salt) {
    static std::atomic<uint64_t> counter{0};
    const uint64_t a = static_cast<uint64_t>(std::chrono::steady_clock::now().time_since_epoch().count());
    const uint64_t b = static_cast<uint64_t>(std::chrono::system_clock::now().time_since_epoch().count());
    uint64_t x = a ^ ((b << 17) | (b >> 47)) ^ (++counter * 0x9E3779B97F4A7C15ull) ^ reinterpret_cast<uintptr_t>(salt);
    // splitmix64's finaliser (Steele, Lea, Flood 2014)
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

bool write_state(const std::string &path, uint64_t fingerprint, const StateShapes &s, const StateMeta &m,
                 const float *conv, const float *gdn, const int8_t *kv, const float *kv_scale, bool append,
                 std::string &err) {
    if (m.position < 0 || (m.position > 0 && s.n_attn > 0 && (!kv || !kv_scale)) || (s.conv_n && !conv) ||
        (s.gdn_n && !gdn)) {
        err = "write_state: bad arguments";
        return false;
    }
    Header h{};
    std::memcpy(h.magic, kMagic, sizeof kMagic);
    h.version = kVersion;
    h.header_size = sizeof(Header);
    h.fingerprint = fingerprint;
    h.conv_id = m.conv_id;
    h.gen = 1;
    h.position = m.position;
    h.extra = m.extra;
    h.image_cap = kImageCap;
    h.kv_elem = 1;
    h.n_attn = s.n_attn;
    h.kv_heads = s.kv_heads;
    h.kv_row = s.kv_row;
    h.hidden = s.hidden;
    h.block = kBlock;
    h.conv_n = s.conv_n;
    h.gdn_n = s.gdn_n;
    h.fixed_offset = kPage;
    h.block_bytes = block_bytes(s, kBlock);
    // an append: the file holds an earlier state of this conversation in this shape - written in place from the
    // block that holds its last position (engine/src/state.cpp:290-306)
    int first_block = 0;
    bool in_place = false;
    if (append) {
        File f;
        Header old{};
        std::string e;
        if (f.open(path, false, false) && header_of(f, old, e) && old.fingerprint == h.fingerprint &&
            old.conv_id == h.conv_id && old.position <= h.position && old.image_cap >= h.n_images &&
            old.block == h.block && old.block_bytes == h.block_bytes && old.fixed_offset == h.fixed_offset) {
            h.image_cap = old.image_cap;
            h.gen = old.gen + 1;
            first_block = std::max(0, old.position - 1) / static_cast<int>(kBlock);
            in_place = true;
        }
    }
    const Layout L = layout_of(h);
    h.fixed_bytes = L.fixed_bytes;
    h.kv_offset = L.kv_offset;
    h.checksum = header_sum(h);

    const std::string target = in_place ? path : path + ".tmp";
    File f;
    if (!f.open(target, true, !in_place)) {
        err = "cannot write " + target;
        return false;
    }
    auto fail = [&](const char *what) {
        f.close();
        if (!in_place) std::remove(target.c_str());
        err = std::string("cannot write the conversation's ") + what + " to " + target;
        return false;
    };
    // the fixed part: gen, the (empty) image slots and hidden state, the states; gen again once they are down
    {
        std::vector<uint8_t> head(static_cast<size_t>(L.conv - h.fixed_offset), 0);
        std::memcpy(head.data(), &h.gen, sizeof h.gen);
        if (!f.write(h.fixed_offset, head.data(), head.size()) || !f.write(L.conv, conv, s.conv_n * sizeof(float)) ||
            !f.write(L.gdn, gdn, s.gdn_n * sizeof(float)) || !f.sync() || !f.write(L.trail, &h.gen, sizeof h.gen))
            return fail("states");
    }
    // the KV rows, re-blocked: ours [layer][K|V][position][row] -> the file's [K|V][layer][block position][row]
    const int blocks = (m.position + static_cast<int>(kBlock) - 1) / static_cast<int>(kBlock);
    if (blocks > first_block && s.n_attn > 0) {
        const size_t bb = static_cast<size_t>(h.block_bytes), row = s.kv_row, heads = s.kv_heads;
        const int per = static_cast<int>(std::max<size_t>(1, kIoBytes / bb));
        std::vector<uint8_t> buf(static_cast<size_t>(std::min(per, blocks - first_block)) * bb);
        for (int b0 = first_block; b0 < blocks; b0 += per) {
            const int nb = std::min(per, blocks - b0);
            std::fill(buf.begin(), buf.begin() + static_cast<ptrdiff_t>(static_cast<size_t>(nb) * bb), uint8_t{0});
            for (int b = b0; b < b0 + nb; ++b) {
                uint8_t *blk = buf.data() + static_cast<size_t>(b - b0) * bb;
                uint8_t *scales = blk + 2 * static_cast<size_t>(s.n_attn) * kBlock * row;
                const int p0 = b * static_cast<int>(kBlock), p1 = std::min(m.position, p0 + static_cast<int>(kBlock));
                for (int v = 0; v < 2; ++v)
                    for (uint32_t l = 0; l < s.n_attn; ++l) {
                        const size_t seg = (static_cast<size_t>(v) * s.n_attn + l) * kBlock;
                        const size_t src = (static_cast<size_t>(l) * 2 + static_cast<size_t>(v)) * static_cast<size_t>(m.position);
                        const size_t run = static_cast<size_t>(p1 - p0);
                        std::memcpy(blk + seg * row, kv + (src + static_cast<size_t>(p0)) * row, run * row);
                        std::memcpy(scales + seg * heads * sizeof(float), kv_scale + (src + static_cast<size_t>(p0)) * heads,
                                    run * heads * sizeof(float));
                    }
            }
            if (!f.write(h.kv_offset + static_cast<uint64_t>(b0) * h.block_bytes, buf.data(), static_cast<size_t>(nb) * bb))
                return fail("KV cache");
        }
    }
    // the header last, once what it names is down
    if (!f.sync() || !f.write(0, &h, sizeof h) || !f.sync()) return fail("header");
    f.close();
    if (!in_place && std::rename(target.c_str(), path.c_str()) != 0) {
        std::remove(target.c_str());
        err = "cannot move " + target + " to " + path;
        return false;
    }
    return true;
}

namespace {

// the header checked against this model and context; the file's layout checked against the header
StateError check(File &f, const std::string &path, uint64_t fingerprint, const StateShapes &s, int context, Header &h,
                 std::string &err) {
    if (!f.open(path, false, false)) {
        err = "cannot open " + path;
        return StateError::io;
    }
    if (!header_of(f, h, err)) return StateError::format;
    if (h.fingerprint != fingerprint || h.kv_elem != 1 || h.n_attn != s.n_attn || h.kv_heads != s.kv_heads ||
        h.kv_row != s.kv_row || h.hidden != s.hidden || h.conv_n != s.conv_n || h.gdn_n != s.gdn_n || h.block == 0) {
        err = "the conversation was saved by another model or another KV cache format";
        return StateError::format;
    }
    if (h.position < 0 || h.position >= context) {
        err = "the saved conversation (" + std::to_string(h.position) + " tokens) is longer than this context (" +
              std::to_string(context) + ")";
        return StateError::context;
    }
    const Layout L = layout_of(h);
    const uint64_t blocks = (static_cast<uint64_t>(h.position) + h.block - 1) / h.block;
    if (L.fixed_bytes != h.fixed_bytes || L.kv_offset != h.kv_offset || h.n_images > h.image_cap ||
        h.block_bytes != block_bytes(s, h.block) || f.size() < h.kv_offset + blocks * h.block_bytes) {
        err = "the saved conversation is cut short";
        return StateError::io;
    }
    uint64_t lead = 0, trail = 0;
    if (!f.read(h.fixed_offset, &lead, sizeof lead) || !f.read(L.trail, &trail, sizeof trail) || lead != h.gen ||
        trail != h.gen) {
        err = "the saved conversation is incomplete (its save was interrupted)";
        return StateError::io;
    }
    if (h.n_images > 0) {   // (this backend verifies text: a conversation with images is another model's)
        err = "the conversation was saved by another model (it holds images)";
        return StateError::format;
    }
    return StateError::none;
}

}  // namespace

StateError peek_state(const std::string &path, uint64_t fingerprint, const StateShapes &s, int context, StateMeta &m,
                      std::string &err) {
    File f;
    Header h{};
    const StateError e = check(f, path, fingerprint, s, context, h, err);
    if (e != StateError::none) return e;
    m.position = h.position;
    m.extra = h.extra;
    m.conv_id = h.conv_id;
    return StateError::none;
}

StateError read_state(const std::string &path, uint64_t fingerprint, const StateShapes &s, int context, StateMeta &m,
                      std::vector<float> &conv, std::vector<float> &gdn, std::vector<int8_t> &kv,
                      std::vector<float> &kv_scale, std::string &err) {
    File f;
    Header h{};
    const StateError e = check(f, path, fingerprint, s, context, h, err);
    if (e != StateError::none) return e;
    const Layout L = layout_of(h);
    const size_t P = static_cast<size_t>(h.position), row = s.kv_row, heads = s.kv_heads;
    conv.assign(s.conv_n, 0.0f);
    gdn.assign(s.gdn_n, 0.0f);
    kv.assign(static_cast<size_t>(s.n_attn) * 2 * P * row, 0);
    kv_scale.assign(static_cast<size_t>(s.n_attn) * 2 * P * heads, 0.0f);
    if (!f.read(L.conv, conv.data(), s.conv_n * sizeof(float)) || !f.read(L.gdn, gdn.data(), s.gdn_n * sizeof(float))) {
        err = "cannot read the states";
        return StateError::io;
    }
    const int B = static_cast<int>(h.block);
    const int blocks = (h.position + B - 1) / B;
    if (blocks > 0 && s.n_attn > 0) {
        const size_t bb = static_cast<size_t>(h.block_bytes);
        const int per = static_cast<int>(std::max<size_t>(1, kIoBytes / bb));
        std::vector<uint8_t> buf(static_cast<size_t>(std::min(per, blocks)) * bb);
        for (int b0 = 0; b0 < blocks; b0 += per) {
            const int nb = std::min(per, blocks - b0);
            if (!f.read(h.kv_offset + static_cast<uint64_t>(b0) * h.block_bytes, buf.data(), static_cast<size_t>(nb) * bb)) {
                err = "cannot read the KV cache";
                return StateError::io;
            }
            for (int b = b0; b < b0 + nb; ++b) {
                const uint8_t *blk = buf.data() + static_cast<size_t>(b - b0) * bb;
                const uint8_t *scales = blk + 2 * static_cast<size_t>(s.n_attn) * static_cast<size_t>(B) * row;
                const int p0 = b * B, p1 = std::min(h.position, p0 + B);
                for (int v = 0; v < 2; ++v)
                    for (uint32_t l = 0; l < s.n_attn; ++l) {
                        const size_t seg = (static_cast<size_t>(v) * s.n_attn + l) * static_cast<size_t>(B);
                        const size_t dst = (static_cast<size_t>(l) * 2 + static_cast<size_t>(v)) * P;
                        const size_t run = static_cast<size_t>(p1 - p0);
                        std::memcpy(kv.data() + (dst + static_cast<size_t>(p0)) * row, blk + seg * row, run * row);
                        std::memcpy(kv_scale.data() + (dst + static_cast<size_t>(p0)) * heads,
                                    scales + seg * heads * sizeof(float), run * heads * sizeof(float));
                    }
            }
        }
    }
    m.position = h.position;
    m.extra = h.extra;
    m.conv_id = h.conv_id;
    return StateError::none;
}

}  // namespace ghost
