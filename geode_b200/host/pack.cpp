// pack.cpp - see pack.hpp.
#include "pack.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <fstream>
#include <sstream>

namespace ghost {

Pack::~Pack() {
    for (auto &f : files_)
        if (f.second.data) munmap(const_cast<uint8_t *>(f.second.data), f.second.size);
}

bool Pack::open(const std::string &dir, std::string &err) {
    std::ifstream in(dir + "/geode.json");
    if (!in) {
        err = "no geode.json in " + dir;
        return false;
    }
    std::stringstream ss;
    ss << in.rdbuf();
    std::string jerr;
    if (!m_.load(ss.str(), jerr)) {
        err = "geode.json: " + jerr;
        return false;
    }
    const JsonRef files = manifest()["files"];
    if (!files.is_list()) {
        err = "geode.json: no file list";
        return false;
    }
    for (const JsonRef f : files) {
        const std::string name = f["name"].text();
        const std::string path = dir + "/" + name;
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) {
            err = "cannot open " + path;
            return false;
        }
        struct stat st{};
        if (fstat(fd, &st) != 0) {
            ::close(fd);
            err = "cannot stat " + path;
            return false;
        }
        Mapped mp;
        mp.size = static_cast<size_t>(st.st_size);
        if (mp.size) {
            void *p = mmap(nullptr, mp.size, PROT_READ, MAP_PRIVATE, fd, 0);
            if (p == MAP_FAILED) {
                ::close(fd);
                err = "cannot map " + path;
                return false;
            }
            mp.data = static_cast<const uint8_t *>(p);
        }
        ::close(fd);
        files_[name] = mp;
    }
    return true;
}

bool Pack::tensor(const std::string &name, TensorView &out, std::string &err) const {
    const JsonRef t = manifest()["tensors"][name];
    if (!t.is_map()) {
        err = "tensor " + name + " is not in the pack";
        return false;
    }
    const auto f = files_.find(t["file"].text());
    if (f == files_.end()) {
        err = "tensor " + name + ": unknown file " + t["file"].text();
        return false;
    }
    out = TensorView();
    out.type = t["type"].text();
    for (const JsonRef d : t["shape"]) out.shape.push_back(d.integer());
    out.global = static_cast<float>(t["global"].number(1.0));
    int64_t n = 1;
    for (int64_t d : out.shape) n *= d;
    if (out.type == "f32") out.bytes = static_cast<size_t>(n) * 4;
    else if (out.type == "bf16") out.bytes = static_cast<size_t>(n) * 2;
    else if (out.type == "q4") out.bytes = static_cast<size_t>(out.rows()) * static_cast<size_t>(out.cols() / 16) * 9;
    else {
        err = "tensor " + name + ": type " + out.type + " is not read by this backend";
        return false;
    }
    const size_t off = static_cast<size_t>(t["offset"].integer());
    if (off + out.bytes > f->second.size) {
        err = "tensor " + name + " runs past its file";
        return false;
    }
    out.data = f->second.data + off;
    return true;
}

bool Pack::experts(int layer, ExpertTable &out, std::string &err) const {
    const JsonRef ls = manifest()["experts"]["layers"];
    const std::string what = layer < 0 ? std::string("the MTP layer") : "layer " + std::to_string(layer);
    // layer -1: the MTP layer's table, the manifest's "mtp": {"experts": ...} (engine/src/pack.cpp:300-305)
    const JsonRef e = layer < 0 ? manifest()["mtp"]["experts"]
                                : (ls.is_list() && static_cast<size_t>(layer) < ls.size() ? ls[static_cast<size_t>(layer)]
                                                                                          : JsonRef());
    if (!e.is_map()) {
        err = "no expert table for " + what;
        return false;
    }
    const auto f = files_.find(e["file"].text());
    if (f == files_.end()) {
        err = "experts of " + what + ": unknown file";
        return false;
    }
    out.stride = static_cast<size_t>(e["stride"].integer());
    const size_t off = static_cast<size_t>(e["offset"].integer());
    const size_t n = static_cast<size_t>(config()["num_experts"].integer());
    if (off + n * out.stride > f->second.size) {
        err = "experts of " + what + " run past their file";
        return false;
    }
    out.data = f->second.data + off;
    return true;
}

}  // namespace ghost
