// qtts_safetensors.h -- the reader of a .safetensors file (host code): the
// role of mormot2-ai's TSafeTensorsFile as TQwenTalker.Create uses it
// (talker.pas:299-332: Tensor(name) -> dtype, shape, data of the mapped
// file).  The format (huggingface/safetensors, published): a little-endian
// u64 N, N bytes of a JSON object {name: {"dtype", "shape", "data_offsets":
// [begin, end)}, "__metadata__": {...}}, then the data; offsets count from
// the end of the header.  The file is mapped read-only, so that a tensor is
// a pointer into the mapping, as the reference reads its BF16 rows in place.
#pragma once
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace qtts_st {

struct Tensor {
    std::string name, dtype;  // dtype as the file names it ("BF16", "F32", ...)
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;
};

// bytes of one element of a safetensors dtype, 0 when unknown
inline int dtype_size(const std::string &d) {
    if (d == "F64" || d == "I64" || d == "U64") return 8;
    if (d == "F32" || d == "I32" || d == "U32") return 4;
    if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
    if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
    return 0;
}

// A JSON reader for the header: objects, arrays, strings, numbers, true /
// false / null.  Tensor entries are collected; everything else is skipped.
class Header {
  public:
    Header(const char *p, const char *e) : p_(p), e_(e) {}
    bool parse(std::vector<Tensor> &out, std::string &err) {
        ws();
        if (!eat('{')) return fail(err, "the header is not a JSON object");
        ws();
        if (eat('}')) return done(err);
        for (;;) {
            std::string key;
            ws();
            if (!str(key)) return fail(err, "bad key");
            ws();
            if (!eat(':')) return fail(err, "':' expected");
            ws();
            if (key == "__metadata__") {
                if (!skip()) return fail(err, "bad __metadata__");
            } else {
                Tensor t;
                t.name = key;
                if (!tensor(t)) return fail(err, "bad entry for tensor " + key);
                out.push_back(std::move(t));
            }
            ws();
            if (eat(',')) continue;
            if (eat('}')) return done(err);
            return fail(err, "',' or '}' expected");
        }
    }

  private:
    const char *p_, *e_;
    bool fail(std::string &err, const std::string &m) {
        err = m;
        return false;
    }
    bool done(std::string &err) {
        ws();
        return p_ == e_ ? true : fail(err, "data after the header object");
    }
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool eat(char c) {
        if (p_ < e_ && *p_ == c) {
            ++p_;
            return true;
        }
        return false;
    }
    static int hexv(char c) {
        if (c >= '0' && c <= '9') return c - '0';
        if (c >= 'a' && c <= 'f') return c - 'a' + 10;
        if (c >= 'A' && c <= 'F') return c - 'A' + 10;
        return -1;
    }
    bool str(std::string &s) {
        if (!eat('"')) return false;
        s.clear();
        while (p_ < e_) {
            char c = *p_++;
            if (c == '"') return true;
            if (static_cast<unsigned char>(c) < 0x20) return false;
            if (c != '\\') {
                s.push_back(c);
                continue;
            }
            if (p_ >= e_) return false;
            c = *p_++;
            switch (c) {
                case '"': case '\\': case '/': s.push_back(c); break;
                case 'b': s.push_back('\b'); break;
                case 'f': s.push_back('\f'); break;
                case 'n': s.push_back('\n'); break;
                case 'r': s.push_back('\r'); break;
                case 't': s.push_back('\t'); break;
                case 'u': {
                    if (e_ - p_ < 4) return false;
                    unsigned u = 0;
                    for (int i = 0; i < 4; ++i) {
                        const int h = hexv(p_[i]);
                        if (h < 0) return false;
                        u = u * 16 + static_cast<unsigned>(h);
                    }
                    p_ += 4;
                    // UTF-8 of a code point of the basic plane (names are ASCII in practice)
                    if (u < 0x80) {
                        s.push_back(static_cast<char>(u));
                    } else if (u < 0x800) {
                        s.push_back(static_cast<char>(0xC0 | (u >> 6)));
                        s.push_back(static_cast<char>(0x80 | (u & 0x3F)));
                    } else {
                        s.push_back(static_cast<char>(0xE0 | (u >> 12)));
                        s.push_back(static_cast<char>(0x80 | ((u >> 6) & 0x3F)));
                        s.push_back(static_cast<char>(0x80 | (u & 0x3F)));
                    }
                    break;
                }
                default: return false;
            }
        }
        return false;
    }
    // a non-negative integer (shapes and offsets)
    bool uint(uint64_t &v) {
        if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
        v = 0;
        while (p_ < e_ && *p_ >= '0' && *p_ <= '9') {
            const uint64_t d = static_cast<uint64_t>(*p_++ - '0');
            if (v > (UINT64_MAX - d) / 10) return false;
            v = v * 10 + d;
        }
        return true;
    }
    bool uints(std::vector<uint64_t> &v) {
        if (!eat('[')) return false;
        ws();
        if (eat(']')) return true;
        for (;;) {
            uint64_t x;
            ws();
            if (!uint(x)) return false;
            v.push_back(x);
            ws();
            if (eat(',')) continue;
            return eat(']');
        }
    }
    bool tensor(Tensor &t) {
        if (!eat('{')) return false;
        bool have_d = false, have_s = false, have_o = false;
        ws();
        if (eat('}')) return false;
        for (;;) {
            std::string k;
            ws();
            if (!str(k)) return false;
            ws();
            if (!eat(':')) return false;
            ws();
            if (k == "dtype") {
                if (!str(t.dtype)) return false;
                have_d = true;
            } else if (k == "shape") {
                std::vector<uint64_t> s;
                if (!uints(s)) return false;
                for (uint64_t x : s) {
                    if (x > (1ull << 40)) return false;
                    t.shape.push_back(static_cast<int64_t>(x));
                }
                have_s = true;
            } else if (k == "data_offsets") {
                std::vector<uint64_t> o;
                if (!uints(o) || o.size() != 2) return false;
                t.begin = o[0];
                t.end = o[1];
                have_o = true;
            } else if (!skip()) {
                return false;
            }
            ws();
            if (eat(',')) continue;
            if (!eat('}')) return false;
            return have_d && have_s && have_o;
        }
    }
    // any JSON value, skipped (bounded nesting)
    bool skip(int depth = 0) {
        ws();
        if (depth > 64 || p_ >= e_) return false;
        if (*p_ == '"') {
            std::string s;
            return str(s);
        }
        if (*p_ == '{' || *p_ == '[') {
            const char close = *p_ == '{' ? '}' : ']';
            const bool obj = *p_ == '{';
            ++p_;
            ws();
            if (eat(close)) return true;
            for (;;) {
                ws();
                if (obj) {
                    std::string k;
                    if (!str(k)) return false;
                    ws();
                    if (!eat(':')) return false;
                }
                if (!skip(depth + 1)) return false;
                ws();
                if (eat(',')) continue;
                return eat(close);
            }
        }
        // number, true, false, null
        const char *b = p_;
        while (p_ < e_ && *p_ && (std::strchr("+-.eE0123456789", *p_) || (*p_ >= 'a' && *p_ <= 'z'))) ++p_;
        return p_ > b;
    }
};

struct File {
    int fd = -1;
    void *map = nullptr;
    size_t size = 0;
    const uint8_t *data = nullptr;  // the first byte after the header
    size_t data_size = 0;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> index;

    ~File() { close(); }
    void close() {
        if (map && map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) ::close(fd);
        map = nullptr;
        fd = -1;
    }
    // maps `path` and reads its header; false with err on any inconsistency
    // (size, JSON, dtype, offsets outside the data, bytes != shape x dtype)
    bool open(const char *path, std::string &err) {
        fd = ::open(path, O_RDONLY | O_CLOEXEC);
        if (fd < 0) {
            err = std::string("cannot open ") + path;
            return false;
        }
        struct stat st;
        if (fstat(fd, &st) != 0 || st.st_size < 8) {
            err = "not a safetensors file (shorter than 8 bytes)";
            return false;
        }
        size = static_cast<size_t>(st.st_size);
        map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (map == MAP_FAILED) {
            map = nullptr;
            err = "mmap failed";
            return false;
        }
        const uint8_t *b = static_cast<const uint8_t *>(map);
        uint64_t n = 0;
        for (int i = 7; i >= 0; --i) n = (n << 8) | b[i];
        if (n > size - 8 || n > (100ull << 20)) {
            err = "header size " + std::to_string(n) + " beyond the file";
            return false;
        }
        Header h(reinterpret_cast<const char *>(b + 8), reinterpret_cast<const char *>(b + 8 + n));
        if (!h.parse(tensors, err)) return false;
        data = b + 8 + n;
        data_size = size - 8 - n;
        for (size_t i = 0; i < tensors.size(); ++i) {
            const Tensor &t = tensors[i];
            const int es = dtype_size(t.dtype);
            if (es == 0) {
                err = "tensor " + t.name + ": unknown dtype " + t.dtype;
                return false;
            }
            uint64_t count = 1;
            for (int64_t d : t.shape) {
                if (d != 0 && count > UINT64_MAX / static_cast<uint64_t>(d)) {
                    err = "tensor " + t.name + ": shape overflows";
                    return false;
                }
                count *= static_cast<uint64_t>(d);
            }
            if (t.begin > t.end || t.end > data_size || t.end - t.begin != count * static_cast<uint64_t>(es)) {
                err = "tensor " + t.name + ": data_offsets do not match its shape or the file";
                return false;
            }
            if (!index.emplace(t.name, i).second) {
                err = "tensor " + t.name + " appears twice";
                return false;
            }
        }
        return true;
    }
    const Tensor *find(const std::string &name) const {
        auto it = index.find(name);
        return it == index.end() ? nullptr : &tensors[it->second];
    }
    uint64_t count(const Tensor &t) const {
        uint64_t c = 1;
        for (int64_t d : t.shape) c *= static_cast<uint64_t>(d);
        return c;
    }
};

}  // namespace qtts_st
