// Header reader for the safetensors format; the checks and messages follow
// src/formats/safetensors.rs (read_with, :161-257; SafeTensorsError, :30-68).
// The JSON is parsed strictly (RFC 8259: no comments or trailing commas,
// UTF-8 strings, paired \u surrogates, at most 128 levels of nesting) into a
// small tree whose objects are sorted maps with the last duplicate key kept:
// the reference's serde_json map without order preservation.
#include "safetensors.h"

#include <cerrno>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

namespace krt {
namespace {

struct JVal {
    enum Type { NUL, BOOL, NUM, STR, ARR, OBJ } t = NUL;
    bool u64ok = false;  // a non-negative integer literal that fits u64 (serde_json's as_u64)
    uint64_t u = 0;
    std::string s;
    std::vector<JVal> a;
    std::map<std::string, JVal> o;
};

class Parser {
  public:
    Parser(const unsigned char *p, size_t n) : p_(p), n_(n) {}

    bool parse(JVal *out, std::string *err) {
        ws();
        if (!value(out, 0)) {
            *err = err_;
            return false;
        }
        ws();
        if (i_ != n_) {
            *err = "trailing characters at byte " + std::to_string(i_);
            return false;
        }
        return true;
    }

  private:
    const unsigned char *p_;
    size_t n_, i_ = 0;
    std::string err_;

    bool fail(const char *what) {
        if (err_.empty()) err_ = std::string(what) + " at byte " + std::to_string(i_);
        return false;
    }
    void ws() {
        while (i_ < n_ && (p_[i_] == ' ' || p_[i_] == '\t' || p_[i_] == '\n' || p_[i_] == '\r')) ++i_;
    }
    bool lit(const char *w) {
        const size_t k = std::strlen(w);
        if (n_ - i_ < k || std::memcmp(p_ + i_, w, k) != 0) return fail("expected value");
        i_ += k;
        return true;
    }

    bool value(JVal *v, int depth) {
        if (depth > 128) return fail("recursion limit exceeded");
        if (i_ >= n_) return fail("EOF while parsing a value");
        const unsigned char c = p_[i_];
        if (c == '{') return object(v, depth);
        if (c == '[') return array(v, depth);
        if (c == '"') {
            v->t = JVal::STR;
            return string(&v->s);
        }
        if (c == 't') {
            v->t = JVal::BOOL;
            return lit("true");
        }
        if (c == 'f') {
            v->t = JVal::BOOL;
            return lit("false");
        }
        if (c == 'n') {
            v->t = JVal::NUL;
            return lit("null");
        }
        if (c == '-' || (c >= '0' && c <= '9')) return number(v);
        return fail("expected value");
    }

    bool number(JVal *v) {
        v->t = JVal::NUM;
        const size_t s0 = i_;
        bool neg = false, integral = true;
        if (p_[i_] == '-') {
            neg = true;
            ++i_;
        }
        if (i_ >= n_ || p_[i_] < '0' || p_[i_] > '9') return fail("invalid number");
        if (p_[i_] == '0') {
            ++i_;
        } else {
            while (i_ < n_ && p_[i_] >= '0' && p_[i_] <= '9') ++i_;
        }
        const size_t int_end = i_;
        if (i_ < n_ && p_[i_] == '.') {
            integral = false;
            ++i_;
            if (i_ >= n_ || p_[i_] < '0' || p_[i_] > '9') return fail("invalid number");
            while (i_ < n_ && p_[i_] >= '0' && p_[i_] <= '9') ++i_;
        }
        if (i_ < n_ && (p_[i_] == 'e' || p_[i_] == 'E')) {
            integral = false;
            ++i_;
            if (i_ < n_ && (p_[i_] == '+' || p_[i_] == '-')) ++i_;
            if (i_ >= n_ || p_[i_] < '0' || p_[i_] > '9') return fail("invalid number");
            while (i_ < n_ && p_[i_] >= '0' && p_[i_] <= '9') ++i_;
        }
        if (integral && !neg) {
            uint64_t x = 0;
            bool fits = true;
            for (size_t k = s0; k < int_end; ++k) {
                const uint64_t d = (uint64_t)(p_[k] - '0');
                if (x > (UINT64_MAX - d) / 10) {
                    fits = false;
                    break;
                }
                x = x * 10 + d;
            }
            v->u64ok = fits;
            v->u = fits ? x : 0;
        }
        return true;
    }

    static void put_utf8(std::string *s, uint32_t cp) {
        if (cp < 0x80) {
            s->push_back((char)cp);
        } else if (cp < 0x800) {
            s->push_back((char)(0xc0 | (cp >> 6)));
            s->push_back((char)(0x80 | (cp & 0x3f)));
        } else if (cp < 0x10000) {
            s->push_back((char)(0xe0 | (cp >> 12)));
            s->push_back((char)(0x80 | ((cp >> 6) & 0x3f)));
            s->push_back((char)(0x80 | (cp & 0x3f)));
        } else {
            s->push_back((char)(0xf0 | (cp >> 18)));
            s->push_back((char)(0x80 | ((cp >> 12) & 0x3f)));
            s->push_back((char)(0x80 | ((cp >> 6) & 0x3f)));
            s->push_back((char)(0x80 | (cp & 0x3f)));
        }
    }

    bool hex4(uint32_t *out) {
        if (n_ - i_ < 4) return fail("EOF while parsing a string");
        uint32_t x = 0;
        for (int k = 0; k < 4; ++k) {
            const unsigned char c = p_[i_ + k];
            uint32_t d;
            if (c >= '0' && c <= '9') d = c - '0';
            else if (c >= 'a' && c <= 'f') d = c - 'a' + 10;
            else if (c >= 'A' && c <= 'F') d = c - 'A' + 10;
            else return fail("invalid escape");
            x = x * 16 + d;
        }
        i_ += 4;
        *out = x;
        return true;
    }

    // One UTF-8 sequence starting at p_[i_] (well formed, shortest form, no
    // surrogates), appended to s.
    bool utf8(std::string *s) {
        const unsigned char c = p_[i_];
        int k;
        uint32_t cp, lo;
        if (c < 0x80) {
            s->push_back((char)c);
            ++i_;
            return true;
        } else if ((c & 0xe0) == 0xc0) {
            k = 1, cp = c & 0x1f, lo = 0x80;
        } else if ((c & 0xf0) == 0xe0) {
            k = 2, cp = c & 0x0f, lo = 0x800;
        } else if ((c & 0xf8) == 0xf0) {
            k = 3, cp = c & 0x07, lo = 0x10000;
        } else {
            return fail("invalid unicode code point");
        }
        if (n_ - i_ <= (size_t)k) return fail("EOF while parsing a string");
        for (int j = 1; j <= k; ++j) {
            const unsigned char d = p_[i_ + j];
            if ((d & 0xc0) != 0x80) return fail("invalid unicode code point");
            cp = (cp << 6) | (d & 0x3f);
        }
        if (cp < lo || cp > 0x10ffff || (cp >= 0xd800 && cp <= 0xdfff)) return fail("invalid unicode code point");
        s->append(reinterpret_cast<const char *>(p_ + i_), (size_t)k + 1);
        i_ += (size_t)k + 1;
        return true;
    }

    bool string(std::string *s) {
        ++i_;  // opening quote
        while (true) {
            if (i_ >= n_) return fail("EOF while parsing a string");
            const unsigned char c = p_[i_];
            if (c == '"') {
                ++i_;
                return true;
            }
            if (c < 0x20) return fail("control character while parsing a string");
            if (c != '\\') {
                if (!utf8(s)) return false;
                continue;
            }
            ++i_;
            if (i_ >= n_) return fail("EOF while parsing a string");
            const unsigned char e = p_[i_++];
            switch (e) {
            case '"': s->push_back('"'); break;
            case '\\': s->push_back('\\'); break;
            case '/': s->push_back('/'); break;
            case 'b': s->push_back('\b'); break;
            case 'f': s->push_back('\f'); break;
            case 'n': s->push_back('\n'); break;
            case 'r': s->push_back('\r'); break;
            case 't': s->push_back('\t'); break;
            case 'u': {
                uint32_t cp;
                if (!hex4(&cp)) return false;
                if (cp >= 0xdc00 && cp <= 0xdfff) return fail("lone trailing surrogate in hex escape");
                if (cp >= 0xd800 && cp <= 0xdbff) {
                    if (n_ - i_ < 2 || p_[i_] != '\\' || p_[i_ + 1] != 'u')
                        return fail("lone leading surrogate in hex escape");
                    i_ += 2;
                    uint32_t lo;
                    if (!hex4(&lo)) return false;
                    if (lo < 0xdc00 || lo > 0xdfff) return fail("lone leading surrogate in hex escape");
                    cp = 0x10000 + ((cp - 0xd800) << 10) + (lo - 0xdc00);
                }
                put_utf8(s, cp);
                break;
            }
            default: return fail("invalid escape");
            }
        }
    }

    bool array(JVal *v, int depth) {
        v->t = JVal::ARR;
        ++i_;
        ws();
        if (i_ < n_ && p_[i_] == ']') {
            ++i_;
            return true;
        }
        while (true) {
            v->a.emplace_back();
            ws();
            if (!value(&v->a.back(), depth + 1)) return false;
            ws();
            if (i_ >= n_) return fail("EOF while parsing a list");
            if (p_[i_] == ',') {
                ++i_;
                continue;
            }
            if (p_[i_] == ']') {
                ++i_;
                return true;
            }
            return fail("expected `,` or `]`");
        }
    }

    bool object(JVal *v, int depth) {
        v->t = JVal::OBJ;
        ++i_;
        ws();
        if (i_ < n_ && p_[i_] == '}') {
            ++i_;
            return true;
        }
        while (true) {
            ws();
            if (i_ >= n_) return fail("EOF while parsing an object");
            if (p_[i_] != '"') return fail("key must be a string");
            std::string key;
            if (!string(&key)) return false;
            ws();
            if (i_ >= n_ || p_[i_] != ':') return fail("expected `:`");
            ++i_;
            ws();
            JVal val;
            if (!value(&val, depth + 1)) return false;
            v->o[key] = std::move(val);  // a later duplicate replaces the earlier
            ws();
            if (i_ >= n_) return fail("EOF while parsing an object");
            if (p_[i_] == ',') {
                ++i_;
                continue;
            }
            if (p_[i_] == '}') {
                ++i_;
                return true;
            }
            return fail("expected `,` or `}`");
        }
    }
};

// Rust's `{:?}` of a string: quoted, with \", \\ and control characters escaped.
std::string debug_str(const std::string &s) {
    std::string o = "\"";
    for (unsigned char c : s) {
        if (c == '"') o += "\\\"";
        else if (c == '\\') o += "\\\\";
        else if (c == '\n') o += "\\n";
        else if (c == '\r') o += "\\r";
        else if (c == '\t') o += "\\t";
        else if (c < 0x20) {
            char b[16];
            std::snprintf(b, sizeof b, "\\u{%x}", c);
            o += b;
        } else o.push_back((char)c);
    }
    return o + "\"";
}

std::string too_short(uint64_t file_len, uint64_t needed) {
    return "file of " + std::to_string(file_len) + " bytes is too short for a " + std::to_string(needed) +
           "-byte header";
}

}  // namespace

std::string st_parse(const unsigned char *prefix, size_t prefix_len, uint64_t file_len, StHeader *out) {
    if (file_len < 8 || prefix_len < 8) return too_short(file_len, 8);
    uint64_t header_len = 0;
    for (int k = 7; k >= 0; --k) header_len = (header_len << 8) | prefix[k];
    if (header_len > file_len - 8) {
        // 8 + header_len, saturating as the reference's checked_add fails
        const uint64_t needed = header_len > UINT64_MAX - 8 ? UINT64_MAX : 8 + header_len;
        return too_short(file_len, needed);
    }
    if (prefix_len < 8 + header_len) return "i/o error: short read of the header";
    JVal root;
    std::string jerr;
    Parser ps(prefix + 8, (size_t)header_len);
    if (!ps.parse(&root, &jerr)) return "invalid header JSON: " + jerr;
    if (root.t != JVal::OBJ) return "invalid header: top level is not an object";
    out->data_offset = 8 + header_len;
    out->data_len = file_len - out->data_offset;
    out->tensors.clear();
    for (const auto &kv : root.o) {
        const std::string &name = kv.first;
        if (name == "__metadata__") continue;
        const JVal &spec = kv.second;
        const std::string q = debug_str(name);
        if (spec.t != JVal::OBJ) return "invalid header: tensor " + q + " is not an object";
        auto it = spec.o.find("dtype");
        if (it == spec.o.end() || it->second.t != JVal::STR) return "invalid header: tensor " + q + " has no dtype";
        StTensor t{};
        const std::string &dt = it->second.s;
        uint64_t width;
        if (dt == "F32") t.dtype = ST_F32, width = 4;
        else if (dt == "BF16") t.dtype = ST_BF16, width = 2;
        else if (dt == "F16") t.dtype = ST_F16, width = 2;
        else return "unsupported dtype " + debug_str(dt) + " (F32, BF16 and F16 are read)";
        it = spec.o.find("shape");
        if (it == spec.o.end() || it->second.t != JVal::ARR)
            return "invalid header: tensor " + q + " has no shape array";
        for (const JVal &d : it->second.a) {
            if (d.t != JVal::NUM || !d.u64ok) return "invalid header: tensor " + q + " has a non-integer shape";
            t.shape.push_back(d.u);
        }
        it = spec.o.find("data_offsets");
        if (it == spec.o.end() || it->second.t != JVal::ARR)
            return "invalid header: tensor " + q + " has no data_offsets";
        const std::vector<JVal> &off = it->second.a;
        if (off.size() < 2 || off[0].t != JVal::NUM || !off[0].u64ok || off[1].t != JVal::NUM || !off[1].u64ok)
            return "invalid header: tensor " + q + " needs two integer data_offsets";
        t.start = off[0].u;
        t.end = off[1].u;
        // numel and its byte size with overflow checks (safetensors.rs:240-247)
        bool ok = true;
        uint64_t numel = 1;
        for (uint64_t d : t.shape) {
            if (d != 0 && numel > UINT64_MAX / d) {
                ok = false;
                break;
            }
            numel *= d;
        }
        if (ok && numel > UINT64_MAX / width) ok = false;
        if (t.start > t.end || t.end > out->data_len || !ok || t.end - t.start != numel * width)
            return "tensor " + q + " has byte range " + std::to_string(t.start) + ".." + std::to_string(t.end) +
                   " that does not match its shape";
        out->tensors[name] = std::move(t);
    }
    return "";
}

std::string st_read_header(const char *path, StHeader *out) {
    if (!path) return "i/o error: null path";
    const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return std::string("i/o error: ") + std::strerror(errno);
    struct stat st;
    if (::fstat(fd, &st) != 0) {
        const std::string e = std::string("i/o error: ") + std::strerror(errno);
        ::close(fd);
        return e;
    }
    const uint64_t file_len = (uint64_t)st.st_size;
    std::vector<unsigned char> buf(8);
    size_t have = 0;
    auto read_to = [&](size_t want) -> bool {
        buf.resize(want);
        while (have < want) {
            const ssize_t r = ::pread(fd, buf.data() + have, want - have, (off_t)have);
            if (r < 0 && errno == EINTR) continue;
            if (r <= 0) return false;
            have += (size_t)r;
        }
        return true;
    };
    std::string err;
    if (file_len < 8 || !read_to(8)) {
        err = too_short(file_len, 8);
    } else {
        uint64_t header_len = 0;
        for (int k = 7; k >= 0; --k) header_len = (header_len << 8) | buf[k];
        // a header longer than the file fails in st_parse without reading it
        if (header_len <= file_len - 8 && !read_to((size_t)(8 + header_len)))
            err = "i/o error: short read of the header";
        if (err.empty()) err = st_parse(buf.data(), have, file_len, out);
    }
    ::close(fd);
    return err;
}

}  // namespace krt
