// json.cpp - see json.hpp.
#include "json.hpp"

#include <algorithm>
#include <charconv>

namespace ghost {

namespace {

enum class Tok { End, MapOpen, MapClose, ListOpen, ListClose, Colon, Comma, Text, Number, True, False, Null, Bad };

// Splits the text into tokens. Text tokens are decoded into the pool as they are scanned; Number tokens are checked
// against the JSON number grammar and converted with from_chars.
class Scanner {
public:
    Scanner(std::string_view src, std::string &pool) : src_(src), pool_(pool) {}

    Tok next() {
        while (pos_ < src_.size() && is_space(src_[pos_])) ++pos_;
        start_ = pos_;
        if (pos_ >= src_.size()) return Tok::End;
        const char c = src_[pos_];
        switch (c) {
        case '{': ++pos_; return Tok::MapOpen;
        case '}': ++pos_; return Tok::MapClose;
        case '[': ++pos_; return Tok::ListOpen;
        case ']': ++pos_; return Tok::ListClose;
        case ':': ++pos_; return Tok::Colon;
        case ',': ++pos_; return Tok::Comma;
        case '"': return scan_text() ? Tok::Text : Tok::Bad;
        case 't': return word("true") ? Tok::True : Tok::Bad;
        case 'f': return word("false") ? Tok::False : Tok::Bad;
        case 'n': return word("null") ? Tok::Null : Tok::Bad;
        default: break;
        }
        if (c == '-' || (c >= '0' && c <= '9')) return scan_number() ? Tok::Number : Tok::Bad;
        problem_ = "unexpected character";
        return Tok::Bad;
    }

    size_t start() const { return start_; }
    size_t pos() const { return pos_; }
    const char *problem() const { return problem_; }
    double number() const { return number_; }
    uint32_t text_at() const { return text_at_; }
    uint32_t text_len() const { return text_len_; }

private:
    static bool is_space(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
    static bool is_digit(char c) { return c >= '0' && c <= '9'; }
    char at(size_t i) const { return i < src_.size() ? src_[i] : '\0'; }

    bool word(std::string_view w) {
        if (src_.substr(pos_, w.size()) != w) {
            problem_ = "unknown word";
            return false;
        }
        pos_ += w.size();
        return true;
    }

    bool scan_number() {
        size_t i = pos_;
        if (at(i) == '-') ++i;
        if (at(i) == '0') {
            ++i;
        } else if (is_digit(at(i))) {
            while (is_digit(at(i))) ++i;
        } else {
            problem_ = "a number without digits";
            return false;
        }
        if (at(i) == '.') {
            ++i;
            if (!is_digit(at(i))) {
                problem_ = "a number without digits after its point";
                return false;
            }
            while (is_digit(at(i))) ++i;
        }
        if (at(i) == 'e' || at(i) == 'E') {
            ++i;
            if (at(i) == '+' || at(i) == '-') ++i;
            if (!is_digit(at(i))) {
                problem_ = "a number without exponent digits";
                return false;
            }
            while (is_digit(at(i))) ++i;
        }
        const char *first = src_.data() + pos_, *last = src_.data() + i;
        const auto r = std::from_chars(first, last, number_);
        if (r.ec != std::errc() || r.ptr != last) {
            problem_ = "a number out of range";
            return false;
        }
        pos_ = i;
        return true;
    }

    // four hex digits at pos_ (moved past them)
    bool hex_unit(uint32_t &u) {
        if (pos_ + 4 > src_.size()) return false;
        u = 0;
        for (size_t k = 0; k < 4; ++k) {
            const char c = src_[pos_ + k];
            const int d = is_digit(c) ? c - '0' : (c >= 'a' && c <= 'f') ? c - 'a' + 10 : (c >= 'A' && c <= 'F') ? c - 'A' + 10 : -1;
            if (d < 0) return false;
            u = u * 16 + static_cast<uint32_t>(d);
        }
        pos_ += 4;
        return true;
    }

    void put_code_point(uint32_t cp) {
        // UTF-8: the lead byte carries the length (0, 110, 1110, 11110 prefixes), then 6 bits per continuation byte
        const int extra = cp < 0x80 ? 0 : cp < 0x800 ? 1 : cp < 0x10000 ? 2 : 3;
        static const uint8_t lead[4] = {0x00, 0xC0, 0xE0, 0xF0};
        pool_.push_back(static_cast<char>(lead[extra] | (cp >> (6 * extra))));
        for (int k = extra - 1; k >= 0; --k) pool_.push_back(static_cast<char>(0x80 | ((cp >> (6 * k)) & 0x3F)));
    }

    bool scan_text() {
        ++pos_;   // the opening quote
        text_at_ = static_cast<uint32_t>(pool_.size());
        for (;;) {
            if (pos_ >= src_.size()) {
                problem_ = "a string without its closing quote";
                return false;
            }
            const unsigned char c = static_cast<unsigned char>(src_[pos_++]);
            if (c == '"') break;
            if (c < 0x20) {
                problem_ = "a control character inside a string";
                return false;
            }
            if (c != '\\') {
                pool_.push_back(static_cast<char>(c));
                continue;
            }
            const char e = at(pos_++);
            static const char from[] = "\"\\/bfnrt", to[] = "\"\\/\b\f\n\r\t";
            if (const char *hit = e ? std::char_traits<char>::find(from, 8, e) : nullptr) {
                pool_.push_back(to[hit - from]);
                continue;
            }
            if (e != 'u') {
                problem_ = "an unknown escape";
                return false;
            }
            uint32_t u = 0;
            if (!hex_unit(u)) {
                problem_ = "a \\u escape without four hex digits";
                return false;
            }
            if (u >= 0xD800 && u < 0xDC00) {   // a high surrogate: its low half must follow as another \u escape
                uint32_t lo = 0;
                if (at(pos_) != '\\' || at(pos_ + 1) != 'u' || (pos_ += 2, !hex_unit(lo)) || lo < 0xDC00 || lo >= 0xE000) {
                    problem_ = "a surrogate pair cut in half";
                    return false;
                }
                u = 0x10000 + ((u - 0xD800) << 10) + (lo - 0xDC00);
            } else if (u >= 0xDC00 && u < 0xE000) {
                problem_ = "a lone low surrogate";
                return false;
            }
            put_code_point(u);
        }
        text_len_ = static_cast<uint32_t>(pool_.size() - text_at_);
        return true;
    }

    std::string_view src_;
    std::string &pool_;
    size_t pos_ = 0, start_ = 0;
    const char *problem_ = "";
    double number_ = 0.0;
    uint32_t text_at_ = 0, text_len_ = 0;
};

}  // namespace

bool JsonDoc::load(std::string_view text, std::string &err) {
    nodes_.clear();
    slots_.clear();
    pool_.clear();
    constexpr size_t kMaxDepth = 512;

    // What the innermost open container waits for next.
    enum class Want { FirstItem, Item, CommaOrClose, Key, Colon };
    struct Open {
        int32_t node;
        bool map;
        size_t first;   // its first entry in `pending`
        Want want;
        uint32_t key_at, key_len;
    };
    std::vector<Open> open;
    std::vector<Slot> pending;   // the open containers' finished children, innermost last
    bool done = false;
    Scanner sc(text, pool_);

    auto fail = [&](const std::string &what, size_t at) {
        nodes_.clear();
        slots_.clear();
        pool_.clear();
        err = what + " (byte " + std::to_string(at) + ")";
        return false;
    };
    // a finished value goes to its container (or is the document)
    auto finish = [&](int32_t node) {
        if (open.empty()) {
            done = true;
            return;
        }
        Open &o = open.back();
        pending.push_back(Slot{node, o.key_at, o.key_len});
        o.want = Want::CommaOrClose;
    };
    auto close = [&]() {
        const Open o = open.back();
        open.pop_back();
        Node &n = nodes_[static_cast<size_t>(o.node)];
        n.at = static_cast<uint32_t>(slots_.size());
        n.count = static_cast<uint32_t>(pending.size() - o.first);
        slots_.insert(slots_.end(), pending.begin() + static_cast<std::ptrdiff_t>(o.first), pending.end());
        pending.resize(o.first);
        if (o.map)
            std::stable_sort(slots_.begin() + n.at, slots_.end(),
                             [this](const Slot &a, const Slot &b) { return key_of(a) < key_of(b); });
        finish(o.node);
    };

    for (;;) {
        const Tok t = sc.next();
        if (t == Tok::Bad) return fail(sc.problem(), sc.start());
        if (done) {
            if (t != Tok::End) return fail("text after the document", sc.start());
            return true;
        }
        if (t == Tok::End) return fail(open.empty() ? "an empty document" : "the document ends inside a container", sc.start());
        const Want want = open.empty() ? Want::Item : open.back().want;

        if (want == Want::Key) {
            if (t != Tok::Text) return fail("a member name expected", sc.start());
            open.back().key_at = sc.text_at();
            open.back().key_len = sc.text_len();
            open.back().want = Want::Colon;
            continue;
        }
        if (want == Want::Colon) {
            if (t != Tok::Colon) return fail("':' expected after a member name", sc.start());
            open.back().want = Want::Item;
            continue;
        }
        if (want == Want::CommaOrClose) {
            const bool map = open.back().map;
            if (t == Tok::Comma) {
                open.back().want = map ? Want::Key : Want::Item;
            } else if (t == (map ? Tok::MapClose : Tok::ListClose)) {
                close();
            } else {
                return fail(map ? "',' or '}' expected" : "',' or ']' expected", sc.start());
            }
            continue;
        }
        // FirstItem / Item: a value (FirstItem also takes the container's close; a map's first entry is a key)
        if (want == Want::FirstItem) {
            const bool map = open.back().map;
            if (t == (map ? Tok::MapClose : Tok::ListClose)) {
                close();
                continue;
            }
            if (map) {
                open.back().want = Want::Key;
                if (t != Tok::Text) return fail("a member name expected", sc.start());
                open.back().key_at = sc.text_at();
                open.back().key_len = sc.text_len();
                open.back().want = Want::Colon;
                continue;
            }
        }
        Node n;
        const int32_t id = static_cast<int32_t>(nodes_.size());
        switch (t) {
        case Tok::MapOpen:
        case Tok::ListOpen:
            if (open.size() >= kMaxDepth) return fail("containers nested too deeply", sc.start());
            n.type = t == Tok::MapOpen ? JsonRef::Type::Map : JsonRef::Type::List;
            nodes_.push_back(n);
            open.push_back(Open{id, t == Tok::MapOpen, pending.size(), Want::FirstItem, 0, 0});
            continue;
        case Tok::Text:
            n.type = JsonRef::Type::Text;
            n.at = sc.text_at();
            n.count = sc.text_len();
            break;
        case Tok::Number:
            n.type = JsonRef::Type::Number;
            n.value = sc.number();
            break;
        case Tok::True:
        case Tok::False:
            n.type = JsonRef::Type::Bool;
            n.flag = t == Tok::True;
            break;
        case Tok::Null: n.type = JsonRef::Type::Null; break;
        default: return fail("a value expected", sc.start());
        }
        nodes_.push_back(n);
        finish(id);
    }
}

JsonRef::Type JsonRef::type() const {
    return doc_ && node_ >= 0 ? doc_->nodes_[static_cast<size_t>(node_)].type : Type::Missing;
}

size_t JsonRef::size() const {
    const Type t = type();
    return t == Type::List || t == Type::Map ? doc_->nodes_[static_cast<size_t>(node_)].count : 0;
}

JsonRef JsonRef::value_at(size_t i) const {
    if (i >= size()) return JsonRef();
    const auto &n = doc_->nodes_[static_cast<size_t>(node_)];
    return JsonRef(doc_, doc_->slots_[n.at + i].node);
}

JsonRef JsonRef::operator[](size_t i) const { return is_list() ? value_at(i) : JsonRef(); }

std::string_view JsonRef::key_at(size_t i) const {
    if (!is_map() || i >= size()) return std::string_view();
    return doc_->key_of(doc_->slots_[doc_->nodes_[static_cast<size_t>(node_)].at + i]);
}

JsonRef JsonRef::operator[](std::string_view key) const {
    if (!is_map()) return JsonRef();
    const auto &n = doc_->nodes_[static_cast<size_t>(node_)];
    const auto first = doc_->slots_.begin() + n.at, last = first + n.count;
    // the last member of that name: the end of its equal run in the stably sorted slots
    const auto hit = std::upper_bound(first, last, key, [this](std::string_view k, const JsonDoc::Slot &s) {
        return k < doc_->key_of(s);
    });
    if (hit == first || doc_->key_of(*(hit - 1)) != key) return JsonRef();
    return JsonRef(doc_, (hit - 1)->node);
}

double JsonRef::number(double fallback) const {
    return type() == Type::Number ? doc_->nodes_[static_cast<size_t>(node_)].value : fallback;
}

long long JsonRef::integer(long long fallback) const {
    return type() == Type::Number ? static_cast<long long>(doc_->nodes_[static_cast<size_t>(node_)].value) : fallback;
}

bool JsonRef::boolean(bool fallback) const {
    return type() == Type::Bool ? doc_->nodes_[static_cast<size_t>(node_)].flag : fallback;
}

std::string JsonRef::text(const std::string &fallback) const {
    if (type() != Type::Text) return fallback;
    const auto &n = doc_->nodes_[static_cast<size_t>(node_)];
    return doc_->pool_.substr(n.at, n.count);
}

}  // namespace ghost
