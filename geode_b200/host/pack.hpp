// pack.hpp - the geode-pack reader of the host side: geode.json (the manifest: files, config, tensor table, expert
// table; engine/src/pack.cpp:52-111, 155-210, 254-291) and the data files, memory-mapped read-only.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "json.hpp"

namespace ghost {

struct TensorView {
    const uint8_t *data = nullptr;
    std::string type;              // "q4", "f32", "bf16"
    std::vector<int64_t> shape;
    float global = 1.0f;           // q4: the per-tensor f32 scale
    size_t bytes = 0;
    int64_t rows() const { return shape.empty() ? 0 : shape[0]; }
    int64_t cols() const {         // the product of the other dims
        int64_t c = 1;
        for (size_t i = 1; i < shape.size(); ++i) c *= shape[i];
        return c;
    }
};

struct ExpertTable {
    const uint8_t *data = nullptr;   // expert e's block at data + e * stride
    size_t stride = 0;
};

class Pack {
public:
    Pack() = default;
    Pack(const Pack &) = delete;
    Pack &operator=(const Pack &) = delete;
    ~Pack();

    bool open(const std::string &dir, std::string &err);
    JsonRef manifest() const { return m_.root(); }
    JsonRef config() const { return m_.root()["config"]; }
    std::string arch() const { return m_.root()["arch"].text(); }
    bool has(const std::string &name) const { return m_.root()["tensors"][name].present(); }
    // false (and err) when the tensor is missing or its bytes run past its file
    bool tensor(const std::string &name, TensorView &out, std::string &err) const;
    // a MoE layer's routed experts (layer -1: the MTP layer's)
    bool experts(int layer, ExpertTable &out, std::string &err) const;

private:
    struct Mapped {
        const uint8_t *data = nullptr;
        size_t size = 0;
    };
    JsonDoc m_;
    std::map<std::string, Mapped> files_;
};

}  // namespace ghost
