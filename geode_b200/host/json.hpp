// json.hpp - a small JSON reader for the geode-pack manifest (geode.json): objects, arrays, strings (with \uXXXX
// escapes kept as UTF-8), numbers (as double), true / false / null. Errors carry the byte offset.
#pragma once

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace ghost {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Json> arr;
    std::map<std::string, Json> obj;

    bool has(const std::string &k) const { return kind == Object && obj.count(k) != 0; }
    const Json &operator[](const std::string &k) const;   // a Null value when absent
    const Json &operator[](size_t i) const { return arr.at(i); }
    double number(double dflt = 0.0) const { return kind == Number ? num : dflt; }
    long long integer(long long dflt = 0) const { return kind == Number ? static_cast<long long>(num) : dflt; }
    const std::string &string() const { return str; }
    size_t size() const { return kind == Array ? arr.size() : kind == Object ? obj.size() : 0; }
};

// Parses text into out; false (and a message in err) on malformed input.
bool parse_json(const std::string &text, Json &out, std::string &err);

}  // namespace ghost
