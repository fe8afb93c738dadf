// MIT2 weight-bundle reader of the B200 GPT library (host side).
//
// Accepts the container the reference reads in vendor/metal-runtime/
// bundle.cpp:176-293 (directory form): manifest.json with format "MIT2",
// version 1, a non-zero alignment, endianness "little" and a tensors array of
// {name, shape, dtype, offset, nbytes}; weights.bin starting with "MIT2" +
// u32 version + u32 alignment; every tensor aligned and inside the file; no
// duplicate names.  The tensor-size rule of src/weights.cpp:17-27 (f32/u32 only,
// nbytes == product(shape) * 4) is applied by check_sizes().
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace itts {

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json* get(const char* k) const {
        for (auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

class JsonReader {
public:
    explicit JsonReader(const std::string& s) : s_(s) {}
    Json parse() {
        Json v = value();
        skip();
        if (p_ != s_.size()) bad("trailing data");
        return v;
    }

private:
    const std::string& s_;
    size_t p_ = 0;
    [[noreturn]] void bad(const char* why) { throw std::runtime_error(std::string("invalid manifest.json: ") + why); }
    void skip() {
        while (p_ < s_.size() && std::isspace(static_cast<unsigned char>(s_[p_]))) ++p_;
    }
    bool eat(char c) {
        skip();
        if (p_ < s_.size() && s_[p_] == c) {
            ++p_;
            return true;
        }
        return false;
    }
    std::string text() {
        if (!eat('"')) bad("expected string");
        std::string out;
        while (p_ < s_.size() && s_[p_] != '"') {
            char c = s_[p_++];
            if (c == '\\' && p_ < s_.size()) {
                const char e = s_[p_++];
                c = e == 'n' ? '\n' : e == 't' ? '\t' : e == 'r' ? '\r' : e;
            }
            out.push_back(c);
        }
        if (p_ >= s_.size()) bad("unterminated string");
        ++p_;
        return out;
    }
    Json value() {
        skip();
        if (p_ >= s_.size()) bad("unexpected end");
        Json v;
        const char c = s_[p_];
        if (c == '{') {
            ++p_;
            v.kind = Json::Obj;
            if (eat('}')) return v;
            do {
                std::string k = text();
                if (!eat(':')) bad("expected ':'");
                v.obj.emplace_back(std::move(k), value());
            } while (eat(','));
            if (!eat('}')) bad("expected '}'");
        } else if (c == '[') {
            ++p_;
            v.kind = Json::Arr;
            if (eat(']')) return v;
            do v.arr.push_back(value());
            while (eat(','));
            if (!eat(']')) bad("expected ']'");
        } else if (c == '"') {
            v.kind = Json::Str;
            v.str = text();
        } else if (s_.compare(p_, 4, "true") == 0) {
            v.kind = Json::Bool;
            v.num = 1;
            p_ += 4;
        } else if (s_.compare(p_, 5, "false") == 0) {
            v.kind = Json::Bool;
            p_ += 5;
        } else if (s_.compare(p_, 4, "null") == 0) {
            p_ += 4;
        } else {
            const size_t st = p_;
            while (p_ < s_.size() && (std::isdigit(static_cast<unsigned char>(s_[p_])) || std::strchr("+-.eE", s_[p_])))
                ++p_;
            if (st == p_) bad("unexpected character");
            v.kind = Json::Num;
            v.num = std::stod(s_.substr(st, p_ - st));
        }
        return v;
    }
};

struct TensorInfo {
    std::string name, dtype;
    std::vector<int64_t> shape;
    uint64_t offset = 0, nbytes = 0;
};

class Mit2Bundle {
public:
    explicit Mit2Bundle(const std::string& dir) {
        std::ifstream f(dir + "/manifest.json");
        if (!f) throw std::runtime_error("failed to open " + dir + "/manifest.json");
        std::stringstream ss;
        ss << f.rdbuf();
        manifest_text_ = ss.str();
        const Json m = JsonReader(manifest_text_).parse();
        if (m.kind != Json::Obj) throw std::runtime_error("invalid manifest.json: not an object");
        const Json* fmt = m.get("format");
        if (!fmt || fmt->kind != Json::Str || fmt->str != "MIT2")
            throw std::runtime_error("unsupported bundle format: " + (fmt ? fmt->str : std::string()));
        const Json* ver = m.get("version");
        const Json* al = m.get("alignment");
        if (!ver || ver->kind != Json::Num) throw std::runtime_error("missing numeric key version");
        if (!al || al->kind != Json::Num) throw std::runtime_error("missing numeric key alignment");
        if (ver->num != 1) throw std::runtime_error("unsupported bundle version");
        alignment_ = static_cast<uint64_t>(al->num);
        if (!alignment_) throw std::runtime_error("bundle alignment must be non-zero");
        const Json* en = m.get("endianness");
        if (!en || en->str != "little") throw std::runtime_error("unsupported bundle endianness");
        if (const Json* t = m.get("target")) target_ = t->str;
        std::string wf = "weights.bin";
        if (const Json* w = m.get("weights_file"))
            if (!w->str.empty()) wf = w->str;
        fd_ = ::open((dir + "/" + wf).c_str(), O_RDONLY);
        if (fd_ < 0) throw std::runtime_error("failed to open mapped file: " + dir + "/" + wf);
        struct stat st {};
        if (fstat(fd_, &st) != 0) throw std::runtime_error("failed to stat mapped file");
        size_ = static_cast<size_t>(st.st_size);
        if (size_ < 12) throw std::runtime_error("weights file is too small for MIT2 header");
        void* p = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (p == MAP_FAILED) throw std::runtime_error("failed to mmap weights file");
        data_ = static_cast<const uint8_t*>(p);
        if (std::memcmp(data_, "MIT2", 4) != 0) throw std::runtime_error("weights file has invalid MIT2 magic");
        uint32_t fv, fa;
        std::memcpy(&fv, data_ + 4, 4);
        std::memcpy(&fa, data_ + 8, 4);
        if (fv != 1) throw std::runtime_error("weights header version mismatch");
        if (fa != alignment_) throw std::runtime_error("weights header alignment mismatch");
        const Json* ts = m.get("tensors");
        if (!ts || ts->kind != Json::Arr) throw std::runtime_error("manifest missing tensors");
        for (const Json& o : ts->arr) {
            TensorInfo t;
            const Json *n = o.get("name"), *d = o.get("dtype"), *sh = o.get("shape"), *of = o.get("offset"),
                       *nb = o.get("nbytes");
            if (!n || n->str.empty()) throw std::runtime_error("tensor record has empty name");
            if (!sh || sh->kind != Json::Arr) throw std::runtime_error("missing tensor shape");
            if (!of || !nb) throw std::runtime_error("missing numeric key offset/nbytes");
            t.name = n->str;
            t.dtype = d ? d->str : std::string();
            for (const Json& x : sh->arr) t.shape.push_back(static_cast<int64_t>(x.num));
            t.offset = static_cast<uint64_t>(of->num);
            t.nbytes = static_cast<uint64_t>(nb->num);
            if (by_name_.count(t.name)) throw std::runtime_error("duplicate tensor in manifest: " + t.name);
            if (t.offset % alignment_) throw std::runtime_error("tensor offset is not bundle-aligned: " + t.name);
            if (!t.nbytes) throw std::runtime_error("tensor has zero bytes: " + t.name);
            if (t.offset + t.nbytes > size_) throw std::runtime_error("tensor extends beyond weights file: " + t.name);
            by_name_[t.name] = tensors_.size();
            tensors_.push_back(std::move(t));
        }
    }
    ~Mit2Bundle() {
        if (data_) munmap(const_cast<uint8_t*>(data_), size_);
        if (fd_ >= 0) ::close(fd_);
    }
    Mit2Bundle(const Mit2Bundle&) = delete;
    Mit2Bundle& operator=(const Mit2Bundle&) = delete;

    const std::string& target() const { return target_; }
    const std::vector<TensorInfo>& tensors() const { return tensors_; }
    const TensorInfo* find(const std::string& n) const {
        auto it = by_name_.find(n);
        return it == by_name_.end() ? nullptr : &tensors_[it->second];
    }
    const TensorInfo& info(const std::string& n) const {
        const TensorInfo* t = find(n);
        if (!t) throw std::runtime_error("Missing tensor: " + n);
        return *t;
    }
    const uint8_t* data(const TensorInfo& t) const { return data_ + t.offset; }
    // src/weights.cpp:17-27
    void check_sizes() const {
        for (const auto& t : tensors_) {
            if (t.dtype != "f32" && t.dtype != "u32") throw std::runtime_error("Initial native backend requires f32/u32: " + t.name);
            uint64_t count = 1;
            for (auto n : t.shape) {
                if (n <= 0) throw std::runtime_error("Invalid shape: " + t.name);
                count *= static_cast<uint64_t>(n);
            }
            if (count * 4 != t.nbytes) throw std::runtime_error("Tensor size does not match shape: " + t.name);
        }
    }

private:
    std::string manifest_text_, target_;
    int fd_ = -1;
    size_t size_ = 0;
    const uint8_t* data_ = nullptr;
    uint64_t alignment_ = 0;
    std::vector<TensorInfo> tensors_;
    std::map<std::string, size_t> by_name_;
};

}  // namespace itts
