// ORACLE / TEST INFRASTRUCTURE — never linked into the product library.
//
// Minimal reader of the MIT2 bundle container used by the oracle port.  It
// follows the rules of the reference parser (vendor/metal-runtime/bundle.cpp:
// 176-293): manifest keys format/version/alignment/endianness, a tensors array
// of {name, shape, dtype, offset, nbytes}, a "MIT2" + u32 version + u32
// alignment header in weights.bin, aligned offsets, and tensors inside the file.
#pragma once

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace orc {

struct JsonValue {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    std::string raw_num, str;
    std::vector<JsonValue> arr;
    std::map<std::string, JsonValue> obj;
    const JsonValue* get(const std::string& k) const {
        auto it = obj.find(k);
        return it == obj.end() ? nullptr : &it->second;
    }
};

class JsonParser {
public:
    explicit JsonParser(const std::string& s) : s_(s) {}
    JsonValue parse() {
        JsonValue v = value();
        ws();
        if (i_ != s_.size()) fail("trailing characters");
        return v;
    }

private:
    const std::string& s_;
    size_t i_ = 0;
    [[noreturn]] void fail(const char* m) { throw std::runtime_error(std::string("manifest json: ") + m); }
    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    JsonValue value() {
        ws();
        if (i_ >= s_.size()) fail("unexpected end");
        const char c = s_[i_];
        JsonValue v;
        if (c == '{') {
            v.kind = JsonValue::Obj;
            ++i_;
            ws();
            if (i_ < s_.size() && s_[i_] == '}') { ++i_; return v; }
            for (;;) {
                ws();
                std::string k = string();
                ws();
                if (i_ >= s_.size() || s_[i_] != ':') fail("expected ':'");
                ++i_;
                v.obj[k] = value();
                ws();
                if (i_ < s_.size() && s_[i_] == ',') { ++i_; continue; }
                if (i_ < s_.size() && s_[i_] == '}') { ++i_; return v; }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = JsonValue::Arr;
            ++i_;
            ws();
            if (i_ < s_.size() && s_[i_] == ']') { ++i_; return v; }
            for (;;) {
                v.arr.push_back(value());
                ws();
                if (i_ < s_.size() && s_[i_] == ',') { ++i_; continue; }
                if (i_ < s_.size() && s_[i_] == ']') { ++i_; return v; }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"') { v.kind = JsonValue::Str; v.str = string(); return v; }
        if (!s_.compare(i_, 4, "true")) { v.kind = JsonValue::Bool; v.b = true; i_ += 4; return v; }
        if (!s_.compare(i_, 5, "false")) { v.kind = JsonValue::Bool; i_ += 5; return v; }
        if (!s_.compare(i_, 4, "null")) { i_ += 4; return v; }
        const size_t st = i_;
        while (i_ < s_.size() && (std::isdigit(static_cast<unsigned char>(s_[i_])) || s_[i_] == '-' ||
                                  s_[i_] == '+' || s_[i_] == '.' || s_[i_] == 'e' || s_[i_] == 'E'))
            ++i_;
        if (st == i_) fail("bad token");
        v.kind = JsonValue::Num;
        v.raw_num = s_.substr(st, i_ - st);
        v.num = std::stod(v.raw_num);
        return v;
    }
    std::string string() {
        if (i_ >= s_.size() || s_[i_] != '"') fail("expected string");
        ++i_;
        std::string out;
        while (i_ < s_.size() && s_[i_] != '"') {
            if (s_[i_] == '\\' && i_ + 1 < s_.size()) {
                const char e = s_[++i_];
                out += e == 'n' ? '\n' : e == 't' ? '\t' : e;
                ++i_;
            } else {
                out += s_[i_++];
            }
        }
        if (i_ >= s_.size()) fail("unterminated string");
        ++i_;
        return out;
    }
};

struct Tensor {
    std::string name, dtype;
    std::vector<int64_t> shape;
    uint64_t offset = 0, nbytes = 0;
};

class Bundle {
public:
    explicit Bundle(const std::string& dir) {
        std::ifstream f(dir + "/manifest.json");
        if (!f) throw std::runtime_error("failed to open " + dir + "/manifest.json");
        std::stringstream ss;
        ss << f.rdbuf();
        const std::string text = ss.str();
        const JsonValue m = JsonParser(text).parse();
        auto str = [&](const char* k) { auto* v = m.get(k); return v && v->kind == JsonValue::Str ? v->str : std::string(); };
        auto num = [&](const char* k) -> uint64_t {
            auto* v = m.get(k);
            if (!v || v->kind != JsonValue::Num) throw std::runtime_error(std::string("missing numeric key ") + k);
            return static_cast<uint64_t>(v->num);
        };
        if (str("format") != "MIT2") throw std::runtime_error("unsupported bundle format");
        if (num("version") != 1) throw std::runtime_error("unsupported bundle version");
        alignment_ = num("alignment");
        if (!alignment_) throw std::runtime_error("bundle alignment must be non-zero");
        if (str("endianness") != "little") throw std::runtime_error("unsupported bundle endianness");
        target_ = str("target");
        std::string wf = str("weights_file");
        if (wf.empty()) wf = "weights.bin";
        fd_ = ::open((dir + "/" + wf).c_str(), O_RDONLY);
        if (fd_ < 0) throw std::runtime_error("failed to open weights file");
        struct stat st {};
        if (fstat(fd_, &st)) throw std::runtime_error("failed to stat weights file");
        size_ = static_cast<size_t>(st.st_size);
        data_ = static_cast<const uint8_t*>(mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0));
        if (data_ == MAP_FAILED) { data_ = nullptr; throw std::runtime_error("mmap failed"); }
        if (size_ < 12 || std::memcmp(data_, "MIT2", 4)) throw std::runtime_error("weights file has invalid MIT2 magic");
        uint32_t ver, al;
        std::memcpy(&ver, data_ + 4, 4);
        std::memcpy(&al, data_ + 8, 4);
        if (ver != 1 || al != alignment_) throw std::runtime_error("weights header mismatch");
        const JsonValue* ts = m.get("tensors");
        if (!ts || ts->kind != JsonValue::Arr) throw std::runtime_error("manifest missing tensors");
        for (const auto& o : ts->arr) {
            Tensor t;
            auto* n = o.get("name");
            auto* d = o.get("dtype");
            auto* sh = o.get("shape");
            auto* of = o.get("offset");
            auto* nb = o.get("nbytes");
            if (!n || !d || !sh || !of || !nb) throw std::runtime_error("incomplete tensor record");
            t.name = n->str;
            t.dtype = d->str;
            for (auto& x : sh->arr) t.shape.push_back(static_cast<int64_t>(x.num));
            t.offset = static_cast<uint64_t>(of->num);
            t.nbytes = static_cast<uint64_t>(nb->num);
            if (t.name.empty() || by_name_.count(t.name)) throw std::runtime_error("bad tensor name: " + t.name);
            if (t.offset % alignment_ || !t.nbytes || t.offset + t.nbytes > size_)
                throw std::runtime_error("bad tensor extent: " + t.name);
            by_name_[t.name] = tensors_.size();
            tensors_.push_back(t);
        }
    }
    ~Bundle() {
        if (data_) munmap(const_cast<uint8_t*>(data_), size_);
        if (fd_ >= 0) ::close(fd_);
    }
    Bundle(const Bundle&) = delete;
    Bundle& operator=(const Bundle&) = delete;
    const Tensor* find(const std::string& n) const {
        auto it = by_name_.find(n);
        return it == by_name_.end() ? nullptr : &tensors_[it->second];
    }
    const Tensor& info(const std::string& n) const {
        const Tensor* t = find(n);
        if (!t) throw std::runtime_error("Missing tensor: " + n);
        return *t;
    }
    const float* f32(const std::string& n) const {
        const Tensor& t = info(n);
        if (t.dtype != "f32") throw std::runtime_error("Expected float32: " + n);
        return reinterpret_cast<const float*>(data_ + t.offset);
    }
    const std::string& target() const { return target_; }

private:
    int fd_ = -1;
    size_t size_ = 0;
    const uint8_t* data_ = nullptr;
    uint64_t alignment_ = 0;
    std::string target_;
    std::vector<Tensor> tensors_;
    std::map<std::string, size_t> by_name_;
};

}  // namespace orc
