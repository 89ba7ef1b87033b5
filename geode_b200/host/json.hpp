// json.hpp - the geode-pack manifest (geode.json) as a read-only document.
//
// Design: the text is scanned once by a token-level state machine (no recursion), and every value becomes one entry
// of a flat node table in document order. A container's node names a contiguous run of child slots; an object's
// slots also carry their keys and are kept sorted by key after parsing, so a member lookup is a binary search.
// Decoded string bytes (escapes resolved, \uXXXX and surrogate pairs as UTF-8) live in one pool. JsonRef is a small
// view (document, node) that callers pass by value; looking up what is not there gives a "missing" view whose
// accessors return their fallbacks, so chains like doc.root()["config"]["hidden_size"].integer() need no checks.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <string_view>
#include <vector>

namespace ghost {

class JsonDoc;

class JsonRef {
public:
    enum class Type : uint8_t { Missing, Null, Bool, Number, Text, List, Map };

    JsonRef() = default;
    Type type() const;
    bool present() const { return type() != Type::Missing; }
    bool is_list() const { return type() == Type::List; }
    bool is_map() const { return type() == Type::Map; }

    JsonRef operator[](std::string_view key) const;   // a Map's member (the last one of that name), else missing
    JsonRef operator[](size_t i) const;               // a List's item, else missing
    size_t size() const;                              // items of a List, members of a Map, else 0
    std::string_view key_at(size_t i) const;          // a Map's i-th key in sorted order
    JsonRef value_at(size_t i) const;                 // its value (a List's i-th item for a List)

    double number(double fallback = 0.0) const;
    long long integer(long long fallback = 0) const;   // a Number truncated toward zero
    bool boolean(bool fallback = false) const;
    std::string text(const std::string &fallback = std::string()) const;

    class Iter;   // a List's items (or a Map's values in key order)
    Iter begin() const;
    Iter end() const;

private:
    friend class JsonDoc;
    friend class Iter;
    JsonRef(const JsonDoc *d, int32_t n) : doc_(d), node_(n) {}
    const JsonDoc *doc_ = nullptr;
    int32_t node_ = -1;
};

class JsonRef::Iter {
public:
    Iter(const JsonDoc *d, int32_t n, size_t i) : doc_(d), node_(n), i_(i) {}
    JsonRef operator*() const { return JsonRef(doc_, node_).value_at(i_); }
    Iter &operator++() {
        ++i_;
        return *this;
    }
    bool operator!=(const Iter &o) const { return i_ != o.i_; }

private:
    const JsonDoc *doc_;
    int32_t node_;
    size_t i_;
};
inline JsonRef::Iter JsonRef::begin() const { return Iter(doc_, node_, 0); }
inline JsonRef::Iter JsonRef::end() const { return Iter(doc_, node_, size()); }

class JsonDoc {
public:
    // Parses text; false (the document left empty) with a message naming the byte offset on malformed input.
    bool load(std::string_view text, std::string &err);
    JsonRef root() const { return nodes_.empty() ? JsonRef() : JsonRef(this, 0); }

private:
    friend class JsonRef;
    struct Node {
        JsonRef::Type type = JsonRef::Type::Null;
        bool flag = false;     // Bool
        double value = 0.0;    // Number
        uint32_t at = 0;       // Text: offset into pool_; List / Map: first slot
        uint32_t count = 0;    // Text: bytes; List / Map: slots
    };
    struct Slot {
        int32_t node = -1;
        uint32_t key_at = 0, key_len = 0;   // Map members only
    };
    std::string_view key_of(const Slot &s) const { return std::string_view(pool_).substr(s.key_at, s.key_len); }

    std::vector<Node> nodes_;
    std::vector<Slot> slots_;
    std::string pool_;
};

}  // namespace ghost
