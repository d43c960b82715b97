// container.h - host-side reader of floyd's Moonlight model directory:
// config.json plus *.safetensors shards (moonlight_model.c:41-110, st.h).
//
// The container written by floyd's converter (tools/convert_moonlight.py)
// holds, per 2-D weight, either F32 data (embedding, lm-head, MoE router) or
// U8 packed values `name` plus one fp32 scale per output row `name.qs`
// (int8: O*I bytes; int4: O*ceil(I/2) bytes, q+8 with the even element in
// the low nibble).  1-D tensors (norms, e_score_correction_bias) are F32.
//
// Only what the loader needs is parsed: a small JSON reader (objects,
// arrays, strings, numbers, booleans, null) and the safetensors header (an
// 8-byte little-endian length, then a JSON object of
// {name: {dtype, shape, data_offsets}}).
#pragma once

#include <dirent.h>
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace fc_container {

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json *get(const char *key) const {
        if (kind != Obj) return nullptr;
        for (auto &kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JsonParser {
public:
    JsonParser(const char *p, const char *end) : p_(p), end_(end) {}

    bool parse(Json &out) {
        if (!value(out, 0)) return false;
        ws();
        return p_ == end_;
    }

private:
    const char *p_, *end_;

    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }
    bool lit(const char *s) {
        size_t n = strlen(s);
        if ((size_t)(end_ - p_) < n || memcmp(p_, s, n)) return false;
        p_ += n;
        return true;
    }
    static void put_utf8(std::string &s, uint32_t c) {
        if (c < 0x80) {
            s += (char)c;
        } else if (c < 0x800) {
            s += (char)(0xC0 | (c >> 6));
            s += (char)(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            s += (char)(0xE0 | (c >> 12));
            s += (char)(0x80 | ((c >> 6) & 0x3F));
            s += (char)(0x80 | (c & 0x3F));
        } else {
            s += (char)(0xF0 | (c >> 18));
            s += (char)(0x80 | ((c >> 12) & 0x3F));
            s += (char)(0x80 | ((c >> 6) & 0x3F));
            s += (char)(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t &v) {
        if (end_ - p_ < 4) return false;
        v = 0;
        for (int i = 0; i < 4; ++i) {
            char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else return false;
        }
        return true;
    }
    bool string(std::string &s) {
        if (p_ >= end_ || *p_ != '"') return false;
        ++p_;
        while (p_ < end_ && *p_ != '"') {
            char c = *p_++;
            if (c != '\\') {
                s += c;
                continue;
            }
            if (p_ >= end_) return false;
            char e = *p_++;
            switch (e) {
                case '"': s += '"'; break;
                case '\\': s += '\\'; break;
                case '/': s += '/'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'n': s += '\n'; break;
                case 'r': s += '\r'; break;
                case 't': s += '\t'; break;
                case 'u': {
                    uint32_t c1;
                    if (!hex4(c1)) return false;
                    if (c1 >= 0xD800 && c1 < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        p_ += 2;
                        uint32_t c2;
                        if (!hex4(c2)) return false;
                        c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
                    }
                    put_utf8(s, c1);
                    break;
                }
                default: return false;
            }
        }
        if (p_ >= end_) return false;
        ++p_;
        return true;
    }
    bool value(Json &v, int depth) {
        if (depth > 64) return false;
        ws();
        if (p_ >= end_) return false;
        char c = *p_;
        if (c == '{') {
            ++p_;
            v.kind = Json::Obj;
            ws();
            if (p_ < end_ && *p_ == '}') { ++p_; return true; }
            for (;;) {
                ws();
                std::string key;
                if (!string(key)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return false;
                ++p_;
                Json child;
                if (!value(child, depth + 1)) return false;
                v.obj.emplace_back(std::move(key), std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') { ++p_; continue; }
                if (p_ < end_ && *p_ == '}') { ++p_; return true; }
                return false;
            }
        }
        if (c == '[') {
            ++p_;
            v.kind = Json::Arr;
            ws();
            if (p_ < end_ && *p_ == ']') { ++p_; return true; }
            for (;;) {
                Json child;
                if (!value(child, depth + 1)) return false;
                v.arr.push_back(std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') { ++p_; continue; }
                if (p_ < end_ && *p_ == ']') { ++p_; return true; }
                return false;
            }
        }
        if (c == '"') {
            v.kind = Json::Str;
            return string(v.str);
        }
        if (lit("true")) { v.kind = Json::Bool; v.b = true; return true; }
        if (lit("false")) { v.kind = Json::Bool; v.b = false; return true; }
        if (lit("null")) { v.kind = Json::Null; return true; }
        // number
        std::string num;
        while (p_ < end_ && (isdigit((unsigned char)*p_) || *p_ == '-' || *p_ == '+' || *p_ == '.' ||
                             *p_ == 'e' || *p_ == 'E'))
            num += *p_++;
        if (num.empty()) return false;
        char *stop = nullptr;
        v.num = strtod(num.c_str(), &stop);
        if (!stop || *stop) return false;
        v.kind = Json::Num;
        return true;
    }
};

inline bool read_file(const std::string &path, std::string &out) {
    int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) return false;
    off_t len = lseek(fd, 0, SEEK_END);
    if (len < 0 || lseek(fd, 0, SEEK_SET) != 0) {
        close(fd);
        return false;
    }
    out.resize((size_t)len);
    size_t got = 0;
    while (got < (size_t)len) {
        ssize_t r = read(fd, &out[got], (size_t)len - got);
        if (r <= 0) break;
        got += (size_t)r;
    }
    close(fd);
    return got == (size_t)len;
}

// safetensors dtypes this loader understands.
enum Dtype { DT_F32, DT_F16, DT_BF16, DT_U8, DT_I8, DT_I32, DT_I64, DT_OTHER };

inline Dtype dtype_of(const std::string &s) {
    if (s == "F32") return DT_F32;
    if (s == "F16") return DT_F16;
    if (s == "BF16") return DT_BF16;
    if (s == "U8") return DT_U8;
    if (s == "I8") return DT_I8;
    if (s == "I32") return DT_I32;
    if (s == "I64") return DT_I64;
    return DT_OTHER;
}

struct Tensor {
    int file = -1;        // index into Index::fds
    Dtype dtype = DT_OTHER;
    std::vector<int64_t> shape;
    uint64_t offset = 0;  // absolute byte offset in the file
    uint64_t bytes = 0;
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t d : shape) n *= d;
        return n;
    }
};

// Every *.safetensors file of a directory, by tensor name.
class Index {
public:
    ~Index() {
        for (int fd : fds)
            if (fd >= 0) close(fd);
    }

    bool open_dir(const std::string &dir, std::string &err) {
        DIR *d = opendir(dir.c_str());
        if (!d) {
            err = "cannot open directory " + dir;
            return false;
        }
        std::vector<std::string> files;
        while (dirent *e = readdir(d)) {
            std::string n = e->d_name;
            if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files.push_back(n);
        }
        closedir(d);
        std::sort(files.begin(), files.end());
        for (auto &f : files)
            if (!add_file(dir + "/" + f, err)) return false;
        return true;
    }

    const Tensor *find(const std::string &name) const {
        auto it = tensors.find(name);
        return it == tensors.end() ? nullptr : &it->second;
    }

    bool read(const Tensor &t, void *dst) const {
        uint8_t *p = reinterpret_cast<uint8_t *>(dst);
        uint64_t got = 0;
        while (got < t.bytes) {
            ssize_t r = pread(fds[t.file], p + got, (size_t)(t.bytes - got), (off_t)(t.offset + got));
            if (r <= 0) return false;
            got += (uint64_t)r;
        }
        return true;
    }

    // Reads a float tensor (F32, F16 or BF16 on disk) as fp32.
    bool read_f32(const Tensor &t, std::vector<float> &out) const {
        const int64_t n = t.numel();
        out.resize((size_t)n);
        if (t.dtype == DT_F32) return t.bytes == (uint64_t)n * 4 && read(t, out.data());
        if (t.dtype != DT_F16 && t.dtype != DT_BF16) return false;
        if (t.bytes != (uint64_t)n * 2) return false;
        std::vector<uint16_t> raw((size_t)n);
        if (!read(t, raw.data())) return false;
        for (int64_t i = 0; i < n; ++i) {
            uint32_t bits;
            if (t.dtype == DT_BF16) {
                bits = (uint32_t)raw[i] << 16;
            } else {  // IEEE half -> float
                uint32_t h = raw[i], sign = (h & 0x8000u) << 16, ex = (h >> 10) & 31, man = h & 1023;
                if (ex == 0) {
                    if (man == 0) {
                        bits = sign;
                    } else {  // subnormal
                        int e = -1;
                        do { man <<= 1; ++e; } while (!(man & 1024));
                        bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 1023) << 13);
                    }
                } else if (ex == 31) {
                    bits = sign | 0x7F800000u | (man << 13);
                } else {
                    bits = sign | ((ex + 112) << 23) | (man << 13);
                }
            }
            memcpy(&out[i], &bits, 4);
        }
        return true;
    }

    std::map<std::string, Tensor> tensors;
    std::vector<int> fds;
    uint64_t total_bytes = 0;

private:
    bool add_file(const std::string &path, std::string &err) {
        int fd = open(path.c_str(), O_RDONLY);
        if (fd < 0) {
            err = "cannot open " + path;
            return false;
        }
        fds.push_back(fd);
        const int file = (int)fds.size() - 1;
        uint8_t lenb[8];
        if (pread(fd, lenb, 8, 0) != 8) {
            err = "short safetensors header in " + path;
            return false;
        }
        uint64_t hlen = 0;
        for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | lenb[i];
        if (hlen == 0 || hlen > ((uint64_t)1 << 30)) {
            err = "invalid safetensors header length in " + path;
            return false;
        }
        std::string header((size_t)hlen, '\0');
        if (pread(fd, &header[0], (size_t)hlen, 8) != (ssize_t)hlen) {
            err = "short safetensors header in " + path;
            return false;
        }
        Json root;
        JsonParser jp(header.data(), header.data() + header.size());
        if (!jp.parse(root) || root.kind != Json::Obj) {
            err = "invalid safetensors header JSON in " + path;
            return false;
        }
        const uint64_t base = 8 + hlen;
        for (auto &kv : root.obj) {
            if (kv.first == "__metadata__") continue;
            const Json &e = kv.second;
            const Json *dt = e.get("dtype"), *sh = e.get("shape"), *off = e.get("data_offsets");
            if (!dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr || !off ||
                off->kind != Json::Arr || off->arr.size() != 2) {
                err = "malformed entry " + kv.first + " in " + path;
                return false;
            }
            Tensor t;
            t.file = file;
            t.dtype = dtype_of(dt->str);
            for (auto &d : sh->arr) t.shape.push_back((int64_t)d.num);
            t.offset = base + (uint64_t)off->arr[0].num;
            t.bytes = (uint64_t)off->arr[1].num - (uint64_t)off->arr[0].num;
            total_bytes += t.bytes;
            tensors[kv.first] = std::move(t);
        }
        return true;
    }
};

}  // namespace fc_container
