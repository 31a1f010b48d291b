/* folder.cpp -- the projector folder read, checked and held resident in HBM (include/ridgefill_folder.h).
 *
 * Reading follows the reference's loader (arch/ridgefill_folder.h:246-293): the manifest, the files it lists
 * mapped read-only and hashed (SHA-256, FIPS 180-4, one thread a file), the safetensors tensors named; checking
 * follows arch/ridgefill_projector.h:84-129. The upload replaces the reference's host block + one-slot ring
 * (arch/ridgefill_projector.h:282-336) by one device block holding everything at once; int8 maps go through the
 * GEMM row's own layout / relayout hooks (the contract arch/ridgefill_int8.h:86-130 relies on).
 */
#include "ridgefill.h"
#include "ridgefill_folder.h"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

namespace {

/* ================================================================== JSON (RFC 8259) */

/* A parsed JSON value. Objects keep their members in document order; a key twice in one object is malformed. */
struct JValue {
    enum Type { Null, Bool, Number, String, Array, Object } type = Null;
    bool flag = false;
    double number = 0.0;
    std::string string;
    std::vector<JValue> items;
    std::vector<std::pair<std::string, JValue>> members;
};

const JValue* member(const JValue* v, const char* key) {
    if (!v || v->type != JValue::Object) return nullptr;
    for (const auto& m : v->members)
        if (m.first == key) return &m.second;
    return nullptr;
}

std::string as_string(const JValue* v, const char* dflt = "") { return v && v->type == JValue::String ? v->string : dflt; }

bool as_int(const JValue* v, int64_t* out) {
    if (!v || v->type != JValue::Number || !(v->number >= -9.0e15 && v->number <= 9.0e15)) return false;
    const int64_t i = (int64_t)v->number;
    if ((double)i != v->number) return false;
    *out = i;
    return true;
}

class JsonReader {
public:
    JsonReader(const char* text, size_t n) : p_(text), end_(text + n) {}

    bool document(JValue* out) {
        if (!value(out, 0)) return false;
        skip();
        return p_ == end_;
    }

private:
    const char* p_;
    const char* end_;

    void skip() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }

    bool literal(const char* word) {
        const size_t n = std::strlen(word);
        if ((size_t)(end_ - p_) < n || std::memcmp(p_, word, n) != 0) return false;
        p_ += n;
        return true;
    }

    static void utf8(uint32_t c, std::string* s) {
        if (c < 0x80) {
            s->push_back((char)c);
        } else if (c < 0x800) {
            s->push_back((char)(0xC0 | (c >> 6)));
            s->push_back((char)(0x80 | (c & 0x3F)));
        } else if (c < 0x10000) {
            s->push_back((char)(0xE0 | (c >> 12)));
            s->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
            s->push_back((char)(0x80 | (c & 0x3F)));
        } else {
            s->push_back((char)(0xF0 | (c >> 18)));
            s->push_back((char)(0x80 | ((c >> 12) & 0x3F)));
            s->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
            s->push_back((char)(0x80 | (c & 0x3F)));
        }
    }

    bool hex4(uint32_t* out) {
        if (end_ - p_ < 4) return false;
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else return false;
        }
        *out = v;
        return true;
    }

    bool string(std::string* out) {
        if (p_ >= end_ || *p_ != '"') return false;
        ++p_;
        while (p_ < end_) {
            const unsigned char c = (unsigned char)*p_++;
            if (c == '"') return true;
            if (c < 0x20) return false;
            if (c != '\\') {
                out->push_back((char)c);
                continue;
            }
            if (p_ >= end_) return false;
            const char e = *p_++;
            switch (e) {
            case '"': out->push_back('"'); break;
            case '\\': out->push_back('\\'); break;
            case '/': out->push_back('/'); break;
            case 'b': out->push_back('\b'); break;
            case 'f': out->push_back('\f'); break;
            case 'n': out->push_back('\n'); break;
            case 'r': out->push_back('\r'); break;
            case 't': out->push_back('\t'); break;
            case 'u': {
                uint32_t u = 0;
                if (!hex4(&u)) return false;
                if (u >= 0xD800 && u < 0xDC00) {   /* a high surrogate: its low half must follow */
                    uint32_t lo = 0;
                    if (!literal("\\u") || !hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                    u = 0x10000 + ((u - 0xD800) << 10) + (lo - 0xDC00);
                } else if (u >= 0xDC00 && u < 0xE000) {
                    return false;
                }
                utf8(u, out);
                break;
            }
            default: return false;
            }
        }
        return false;
    }

    bool number(double* out) {
        const char* s = p_;
        if (p_ < end_ && *p_ == '-') ++p_;
        if (p_ >= end_) return false;
        if (*p_ == '0') {
            ++p_;
        } else if (*p_ >= '1' && *p_ <= '9') {
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        } else {
            return false;
        }
        if (p_ < end_ && *p_ == '.') {
            ++p_;
            if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
            ++p_;
            if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ >= end_ || !(*p_ >= '0' && *p_ <= '9')) return false;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        const std::string text(s, p_);
        *out = std::strtod(text.c_str(), nullptr);
        return true;
    }

    bool value(JValue* v, int depth) {
        if (depth > 64) return false;
        skip();
        if (p_ >= end_) return false;
        switch (*p_) {
        case '{': {
            ++p_;
            v->type = JValue::Object;
            skip();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            for (;;) {
                skip();
                std::string key;
                if (!string(&key)) return false;
                for (const auto& m : v->members)
                    if (m.first == key) return false;
                skip();
                if (p_ >= end_ || *p_ != ':') return false;
                ++p_;
                v->members.emplace_back(std::move(key), JValue{});
                if (!value(&v->members.back().second, depth + 1)) return false;
                skip();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        case '[': {
            ++p_;
            v->type = JValue::Array;
            skip();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            for (;;) {
                v->items.emplace_back();
                if (!value(&v->items.back(), depth + 1)) return false;
                skip();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        case '"':
            v->type = JValue::String;
            return string(&v->string);
        case 't':
            v->type = JValue::Bool;
            v->flag = true;
            return literal("true");
        case 'f':
            v->type = JValue::Bool;
            return literal("false");
        case 'n':
            return literal("null");
        default:
            v->type = JValue::Number;
            return number(&v->number);
        }
    }
};

/* ================================================================== SHA-256 (FIPS 180-4) */

/* The round constants and initial hash words, derived as the standard defines them: the first 32 bits of the
 * fractional parts of the cube roots of the first 64 primes, and of the square roots of the first 8, by exact
 * integer roots (floor(cbrt(p * 2^96)) and floor(sqrt(p * 2^64)), whose low 32 bits are those fractions). */
struct ShaConstants {
    uint32_t k[64];
    uint32_t h0[8];
    ShaConstants() {
        int primes[64], n = 0;
        for (int c = 2; n < 64; ++c) {
            bool prime = true;
            for (int d = 2; d * d <= c; ++d)
                if (c % d == 0) prime = false;
            if (prime) primes[n++] = c;
        }
        for (int i = 0; i < 64; ++i) k[i] = (uint32_t)root((unsigned __int128)primes[i] << 96, 3);
        for (int i = 0; i < 8; ++i) h0[i] = (uint32_t)root((unsigned __int128)primes[i] << 64, 2);
    }
    static uint64_t root(unsigned __int128 x, int degree) {   /* floor(x^(1/degree)) for x < 2^105 */
        uint64_t lo = 0, hi = (uint64_t)1 << 36;
        while (lo < hi) {
            const uint64_t mid = lo + (hi - lo + 1) / 2;
            unsigned __int128 p = mid;
            for (int i = 1; i < degree; ++i) p *= mid;
            if (p <= x) lo = mid;
            else hi = mid - 1;
        }
        return lo;
    }
};

const ShaConstants& sha_constants() {
    static const ShaConstants c;
    return c;
}

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void sha_compress(uint32_t h[8], const uint8_t* block, const uint32_t* k) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
        w[i] = (uint32_t)block[4 * i] << 24 | (uint32_t)block[4 * i + 1] << 16 | (uint32_t)block[4 * i + 2] << 8 |
               (uint32_t)block[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
        const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
        const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[i] + w[i];
        const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
        hh = g;
        g = f;
        f = e;
        e = d + t1;
        d = c;
        c = b;
        b = a;
        a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

std::string sha256_hex(const uint8_t* data, size_t n) {
    const ShaConstants& c = sha_constants();
    uint32_t h[8];
    std::memcpy(h, c.h0, sizeof h);
    size_t at = 0;
    for (; at + 64 <= n; at += 64) sha_compress(h, data + at, c.k);
    uint8_t last[128] = {};
    const size_t rest = n - at, blocks = rest + 9 <= 64 ? 1 : 2;
    if (rest) std::memcpy(last, data + at, rest);
    last[rest] = 0x80;
    const uint64_t bits = (uint64_t)n * 8;
    for (int i = 0; i < 8; ++i) last[blocks * 64 - 1 - i] = (uint8_t)(bits >> (8 * i));
    for (size_t b = 0; b < blocks; ++b) sha_compress(h, last + 64 * b, c.k);
    char hex[65];
    for (int i = 0; i < 8; ++i) std::snprintf(hex + 8 * i, 9, "%08x", h[i]);
    return std::string(hex, 64);
}

/* ================================================================== the folder */

struct HostTensor {
    const uint8_t* data = nullptr;
    uint32_t dtype = 0;
    std::vector<int64_t> shape;
    int64_t bytes = 0;
};

struct Mapping {
    const uint8_t* data = nullptr;
    size_t size = 0;
};

uint32_t st_dtype(const std::string& s) {   /* the dtypes the folder's writer uses */
    if (s == "BF16") return RAD_BF16;
    if (s == "F32") return RAD_F32;
    if (s == "F16") return RAD_F16;
    if (s == "I8") return RAD_I8;
    if (s == "I32") return RAD_I32;
    return 0;
}

void say(char* why, size_t n, const char* fmt, ...) {
    if (!why || n == 0) return;
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(why, n, fmt, ap);
    va_end(ap);
}

bool shaped(const HostTensor* t, uint32_t dtype, std::initializer_list<int64_t> shape) {
    return t && t->dtype == dtype && t->shape == std::vector<int64_t>(shape);
}

}  // namespace

struct RidgeFillFolder {
    std::string dir;
    JValue manifest;
    std::vector<Mapping> maps;
    std::map<std::string, HostTensor> tensors;
    int64_t file_bytes = 0;

    ~RidgeFillFolder() {
        for (const Mapping& m : maps)
            if (m.data) munmap((void*)m.data, m.size);
    }

    const HostTensor* find(const std::string& name) const {
        const auto it = tensors.find(name);
        return it == tensors.end() ? nullptr : &it->second;
    }
};

namespace {

/* One safetensors file's tensors into f->tensors: an 8-byte little-endian header length, the JSON header, the
 * data section; every tensor's [begin, end) inside the data section and equal to its shape times its dtype. */
bool read_tensors(const std::string& name, const Mapping& m, RidgeFillFolder* f, char* why, size_t nw) {
    uint64_t hlen = 0;
    if (m.size < 8) {
        say(why, nw, "%s is shorter than a safetensors header", name.c_str());
        return false;
    }
    std::memcpy(&hlen, m.data, 8);
    JValue h;
    if (hlen > m.size - 8 || !JsonReader((const char*)m.data + 8, (size_t)hlen).document(&h) || h.type != JValue::Object) {
        say(why, nw, "%s: its safetensors header does not parse", name.c_str());
        return false;
    }
    const uint64_t data_bytes = m.size - 8 - hlen;
    for (const auto& kv : h.members) {
        if (kv.first == "__metadata__") continue;
        HostTensor t;
        t.dtype = st_dtype(as_string(member(&kv.second, "dtype")));
        const JValue* shape = member(&kv.second, "shape");
        const JValue* off = member(&kv.second, "data_offsets");
        bool ok = t.dtype != 0 && shape && shape->type == JValue::Array && off && off->type == JValue::Array &&
                  off->items.size() == 2;
        int64_t numel = 1;
        for (size_t i = 0; ok && i < shape->items.size(); ++i) {
            int64_t d = 0;
            ok = as_int(&shape->items[i], &d) && d >= 0 && d < ((int64_t)1 << 40);
            t.shape.push_back(d);
            numel *= d;
            ok = ok && numel < ((int64_t)1 << 48);
        }
        int64_t lo = 0, hi = 0;
        ok = ok && as_int(&off->items[0], &lo) && as_int(&off->items[1], &hi) && lo >= 0 && lo <= hi &&
             (uint64_t)hi <= data_bytes;
        t.bytes = ok ? rad_dtype_bytes(t.dtype, numel) : -1;
        if (!ok || hi - lo != t.bytes) {
            say(why, nw, "%s: tensor '%s' has an unknown dtype or its bytes do not match its shape", name.c_str(),
                kv.first.c_str());
            return false;
        }
        t.data = m.data + 8 + hlen + lo;
        if (!f->tensors.emplace(kv.first, std::move(t)).second) {
            say(why, nw, "tensor '%s' is in two files", kv.first.c_str());
            return false;
        }
    }
    return true;
}

Mapping map_file(const std::string& path) {
    Mapping m;
    const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return m;
    struct stat st {};
    if (fstat(fd, &st) == 0 && S_ISREG(st.st_mode) && st.st_size > 0) {
        void* p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (p != MAP_FAILED) {
            m.data = (const uint8_t*)p;
            m.size = (size_t)st.st_size;
        }
    }
    close(fd);
    return m;
}

/* Whether late layer `li` keeps no correction (a full-attention layer). */
bool full_layer(const RidgeFillFolder* f, const RidgeFillModelGeom* m, int64_t li) {
    if (m->full) return m->full[li] != 0;
    const JValue* layers = member(&f->manifest, "layers");
    return as_string(member(layers, std::to_string(li).c_str())) == "full_attn";
}

const char* const kTables[] = { "score", "score_none", "score_all" };

}  // namespace

extern "C" int ridgefill_folder_open(const char* dir, RidgeFillFolder** out, char* why, size_t nw) {
    if (!dir || !out) return RAD_E_INVAL;
    *out = nullptr;
    std::unique_ptr<RidgeFillFolder> f(new RidgeFillFolder);
    f->dir = dir;
    const std::string mpath = f->dir + "/ridgefill.json";
    const Mapping mm = map_file(mpath);
    bool ok = mm.data && JsonReader((const char*)mm.data, mm.size).document(&f->manifest) &&
              f->manifest.type == JValue::Object;
    if (mm.data) munmap((void*)mm.data, mm.size);
    int64_t format = 0;
    if (!ok || !as_int(member(&f->manifest, "format"), &format) || format != 1) {
        say(why, nw, "%s does not parse as a format-1 projector manifest", mpath.c_str());
        return RAD_E_INVAL;
    }
    const JValue* files = member(&f->manifest, "files");
    if (!files || files->type != JValue::Object || files->members.empty()) {
        say(why, nw, "%s lists no files", mpath.c_str());
        return RAD_E_INVAL;
    }
    const size_t n = files->members.size();
    for (size_t i = 0; i < n; ++i) {
        const std::string& name = files->members[i].first;
        /* a bare file name: the manifest cannot reach outside its folder */
        const Mapping m = name.find('/') == std::string::npos && name != "." && name != ".."
                              ? map_file(f->dir + "/" + name) : Mapping{};
        if (!m.data) {
            say(why, nw, "the manifest lists %s, which is missing or unreadable in %s", name.c_str(), dir);
            return RAD_E_INVAL;
        }
        f->maps.push_back(m);
        f->file_bytes += (int64_t)m.size;
    }
    std::vector<std::string> got(n);
    {
        std::vector<std::thread> pool;
        for (size_t i = 0; i < n; ++i)
            pool.emplace_back([&, i] { got[i] = sha256_hex(f->maps[i].data, f->maps[i].size); });
        for (std::thread& t : pool) t.join();
    }
    for (size_t i = 0; i < n; ++i) {
        const std::string& name = files->members[i].first;
        const std::string want = as_string(&files->members[i].second);
        if (got[i] != want) {
            say(why, nw, "%s is corrupt or not the file the manifest names (sha256 %s, the manifest says %s)",
                name.c_str(), got[i].c_str(), want.c_str());
            return RAD_E_INVAL;
        }
        const bool st = name.size() > 12 && name.compare(name.size() - 12, 12, ".safetensors") == 0;
        if (st && !read_tensors(name, f->maps[i], f.get(), why, nw)) return RAD_E_INVAL;
    }
    *out = f.release();
    return RAD_OK;
}

extern "C" void ridgefill_folder_close(RidgeFillFolder* f) { delete f; }

extern "C" int64_t ridgefill_folder_tensor_count(const RidgeFillFolder* f) { return f ? (int64_t)f->tensors.size() : 0; }

extern "C" int64_t ridgefill_folder_file_bytes(const RidgeFillFolder* f) { return f ? f->file_bytes : 0; }

extern "C" int ridgefill_folder_tensor(const RidgeFillFolder* f, const char* name, RadTensor* out) {
    const HostTensor* t = f && name ? f->find(name) : nullptr;
    if (!t || !out || t->shape.size() > RAD_MAX_RANK) return RAD_E_INVAL;
    *out = RadTensor{};
    out->dtype = t->dtype;
    out->rank = (uint32_t)t->shape.size();
    for (size_t i = 0; i < t->shape.size(); ++i) out->shape[i] = t->shape[i];
    rad_tensor_pack(out);
    out->data = (void*)t->data;
    return RAD_OK;
}

extern "C" int ridgefill_folder_check(const RidgeFillFolder* f, const RidgeFillModelGeom* m, int64_t* split_out,
                                      int* int8_out, char* why, size_t nw) {
    if (!f || !m) return RAD_E_INVAL;
    const int64_t n = m->n_embd, wide = m->wide;
    int64_t S = -1;
    as_int(member(&f->manifest, "split"), &S);
    if (S < m->split_lo || S >= m->n_layer) {
        say(why, nw, "its split %lld is not a late layer of this model (layers %lld..%lld)", (long long)S,
            (long long)m->split_lo, (long long)m->n_layer - 1);
        return RAD_E_INVAL;
    }
    const JValue* proj = member(&f->manifest, "projector");
    const std::string dtype = as_string(member(proj, "dtype"), "bf16");
    if (dtype != "bf16" && dtype != "i8") {
        say(why, nw, "its projector dtype '%s' is neither bf16 nor i8", dtype.c_str());
        return RAD_E_INVAL;
    }
    const bool int8 = dtype == "i8";
    int held = 0, want = 0;
    for (int64_t li = S; li < m->n_layer; ++li) {
        const std::string p = "proj." + std::to_string(li);
        const bool map_ok = int8 ? wide % 128 == 0 && shaped(f->find(p + ".codes"), RAD_I8, { n, wide }) &&
                                       shaped(f->find(p + ".scale"), RAD_BF16, { n, wide / 128 })
                                 : shaped(f->find(p + ".weight"), RAD_BF16, { n, wide });
        if (!map_ok || !shaped(f->find(p + ".bias"), RAD_BF16, { n })) {
            if (int8)
                say(why, nw, "%s.codes i8 [%lld, %lld] / .scale bf16 [%lld, %lld / 128] / .bias bf16 is missing or misshapen",
                    p.c_str(), (long long)n, (long long)wide, (long long)n, (long long)wide);
            else
                say(why, nw, "%s.weight [%lld, %lld] / .bias bf16 is missing or misshapen", p.c_str(), (long long)n,
                    (long long)wide);
            return RAD_E_INVAL;
        }
        if (full_layer(f, m, li)) continue;
        ++want;
        held += shaped(f->find("st." + std::to_string(li)), RAD_F32, { m->st_heads, m->st_sd0, m->st_sd1 });
    }
    if (held && held != want) {
        say(why, nw, "the correction covers %d of the %d delta-net layers from the split up; it is all of them or none",
            held, want);
        return RAD_E_INVAL;
    }
    if (member(&f->manifest, "final") &&
        (!shaped(f->find("final.weight"), RAD_BF16, { wide, wide }) || !shaped(f->find("final.bias"), RAD_BF16, { wide }))) {
        say(why, nw, "its final map is not final.weight bf16 [%lld, %lld] + final.bias [%lld]", (long long)wide,
            (long long)wide, (long long)wide);
        return RAD_E_INVAL;
    }
    for (const char* s : kTables)
        if (f->find(s) && !shaped(f->find(s), RAD_F32, { m->n_vocab })) {
            say(why, nw, "the row table '%s' is not f32 [%lld]", s, (long long)m->n_vocab);
            return RAD_E_INVAL;
        }
    if (split_out) *split_out = S;
    if (int8_out) *int8_out = int8;
    return RAD_OK;
}

/* ================================================================== the resident block */

struct RidgeFillResident {
    void* block = nullptr;
    int device = 0;   /* the device the block was allocated on */
    int64_t bytes = 0;
    int64_t n_embd = 0, wide = 0, split = 0, n_layer = 0, heads = 0, sd0 = 0, sd1 = 0, n_vocab = 0;
    bool int8 = false;
    std::vector<int64_t> w_at, scale_at, bias_at, st_at;   /* per layer; -1 where nothing was uploaded */
    std::map<std::string, int64_t> table_at;
    int64_t final_w_at = -1, final_b_at = -1;

    ~RidgeFillResident() {
        if (!block) return;
        int cur = 0;
        const bool switched = cudaGetDevice(&cur) == cudaSuccess && cur != device && cudaSetDevice(device) == cudaSuccess;
        cudaFree(block);
        if (switched) cudaSetDevice(cur);
    }

    void* at(int64_t off) const { return (char*)block + off; }
};

namespace {

RadTensor device_view(void* data, uint32_t dtype, std::initializer_list<int64_t> shape) {
    RadTensor t{};
    t.dtype = dtype;
    for (int64_t d : shape) t.shape[t.rank++] = d;
    rad_tensor_pack(&t);
    t.data = data;
    return t;
}

/* One piece of the upload: `bytes` from `src` (a mapping, or `owned`) to offset `at` of the block. */
struct Piece {
    const void* src = nullptr;
    int64_t bytes = 0;
    int64_t at = 0;
    std::vector<uint8_t> owned;
};

int64_t place(std::vector<Piece>& plan, int64_t* end, const void* src, int64_t bytes) {
    const int64_t at = (*end + 255) / 256 * 256;
    Piece p;
    p.src = src;
    p.bytes = bytes;
    p.at = at;
    plan.push_back(std::move(p));
    *end = at + bytes;
    return at;
}

}  // namespace

extern "C" int ridgefill_folder_upload(const RidgeFillFolder* f, const RidgeFillModelGeom* m, int64_t head_first,
                                       int64_t n_heads, RadStream s, RidgeFillResident** out, char* why, size_t nw) {
    if (!f || !m || !out) return RAD_E_INVAL;
    *out = nullptr;
    int64_t S = 0;
    int int8 = 0;
    int rc = ridgefill_folder_check(f, m, &S, &int8, why, nw);
    if (rc != RAD_OK) return rc;
    const int64_t n = m->n_embd, wide = m->wide, L = m->n_layer;
    if (n_heads < 0) {
        head_first = 0;
        n_heads = m->st_heads;
    }
    if (head_first < 0 || n_heads < 0 || head_first + n_heads > m->st_heads) {
        say(why, nw, "heads [%lld, %lld) are outside the correction's %lld", (long long)head_first,
            (long long)(head_first + n_heads), (long long)m->st_heads);
        return RAD_E_INVAL;
    }
    std::unique_ptr<RidgeFillResident> r(new RidgeFillResident);
    r->n_embd = n;
    r->wide = wide;
    r->split = S;
    r->n_layer = L;
    r->heads = n_heads;
    r->sd0 = m->st_sd0;
    r->sd1 = m->st_sd1;
    r->n_vocab = m->n_vocab;
    r->int8 = int8 != 0;
    r->w_at.assign((size_t)L, -1);
    r->scale_at.assign((size_t)L, -1);
    r->bias_at.assign((size_t)L, -1);
    r->st_at.assign((size_t)L, -1);

    std::vector<Piece> plan;
    int64_t end = 0;
    const RadParam params[] = { RAD_INT("M", 1), RAD_INT("N", n), RAD_INT("K", wide), RAD_INT("group", 128),
                                RAD_STR("dtype", "i8a8") };
    const int n_p = (int)(sizeof params / sizeof params[0]);
    const RadEncoding enc = rad_enc_affine(RAD_I8, RAD_BF16, 1, 128);
    for (int64_t li = S; li < L; ++li) {
        const std::string p = "proj." + std::to_string(li);
        if (int8) {
            RadTensor codes{}, scale{};
            ridgefill_folder_tensor(f, (p + ".codes").c_str(), &codes);
            ridgefill_folder_tensor(f, (p + ".scale").c_str(), &scale);
            RadLayout lc{}, ls{};
            const int sc = 0, ss = 1;
            rc = ridgefill_gemm_q_layout(params, n_p, GQ_B, &enc, &sc, &codes, 1, &lc);
            if (rc == RAD_OK) rc = ridgefill_gemm_q_layout(params, n_p, GQ_B_SCALE, &enc, &ss, &scale, 1, &ls);
            if (rc != RAD_OK) {
                say(why, nw, "the int8 GEMM row cannot store %s at [%lld, %lld] (N a multiple of 16, K of 128)",
                    p.c_str(), (long long)n, (long long)wide);
                return RAD_E_UNSUPPORTED;
            }
            r->w_at[(size_t)li] = place(plan, &end, nullptr, lc.bytes);
            plan.back().owned.resize((size_t)lc.bytes);
            rc = ridgefill_gemm_q_relayout(params, n_p, GQ_B, &enc, &sc, &codes, 1, plan.back().owned.data(), lc.bytes);
            plan.back().src = plan.back().owned.data();
            r->scale_at[(size_t)li] = place(plan, &end, nullptr, ls.bytes);
            plan.back().owned.resize((size_t)ls.bytes);
            if (rc == RAD_OK)
                rc = ridgefill_gemm_q_relayout(params, n_p, GQ_B_SCALE, &enc, &ss, &scale, 1, plan.back().owned.data(),
                                               ls.bytes);
            plan.back().src = plan.back().owned.data();
            if (rc != RAD_OK) {
                say(why, nw, "the int8 GEMM row's relayout refused %s", p.c_str());
                return RAD_E_UNSUPPORTED;
            }
        } else {
            const HostTensor* w = f->find(p + ".weight");
            r->w_at[(size_t)li] = place(plan, &end, w->data, w->bytes);
        }
        const HostTensor* b = f->find(p + ".bias");
        r->bias_at[(size_t)li] = place(plan, &end, b->data, b->bytes);
        const HostTensor* st = full_layer(f, m, li) ? nullptr : f->find("st." + std::to_string(li));
        if (st && n_heads > 0) {
            const int64_t head = m->st_sd0 * m->st_sd1 * 4;
            r->st_at[(size_t)li] = place(plan, &end, st->data + head_first * head, n_heads * head);
        }
    }
    for (const char* name : kTables)
        if (const HostTensor* t = f->find(name)) r->table_at[name] = place(plan, &end, t->data, t->bytes);
    if (member(&f->manifest, "final")) {
        const HostTensor* w = f->find("final.weight");
        const HostTensor* b = f->find("final.bias");
        r->final_w_at = place(plan, &end, w->data, w->bytes);
        r->final_b_at = place(plan, &end, b->data, b->bytes);
    }
    r->bytes = (end + 255) / 256 * 256;
    if (r->bytes == 0) {
        *out = r.release();
        return RAD_OK;
    }
    if (cudaGetDevice(&r->device) != cudaSuccess || cudaMalloc(&r->block, (size_t)r->bytes) != cudaSuccess) {
        cudaGetLastError();
        r->block = nullptr;
        say(why, nw, "could not allocate %.1f MiB of device memory for the folder", (double)r->bytes / (1 << 20));
        return RAD_E_NOMEM;
    }
    const cudaStream_t stream = (cudaStream_t)s;
    bool ok = true;
    for (const Piece& p : plan)
        ok = ok && cudaMemcpyAsync(r->at(p.at), p.src, (size_t)p.bytes, cudaMemcpyHostToDevice, stream) == cudaSuccess;
    ok = cudaStreamSynchronize(stream) == cudaSuccess && ok;
    if (!ok) {
        say(why, nw, "the folder's upload failed: %s", cudaGetErrorString(cudaGetLastError()));
        return RAD_E_DEVICE;
    }
    *out = r.release();
    return RAD_OK;
}

extern "C" void ridgefill_resident_free(RidgeFillResident* r) { delete r; }

extern "C" int64_t ridgefill_resident_bytes(const RidgeFillResident* r) { return r ? r->bytes : 0; }

extern "C" int ridgefill_resident_map(const RidgeFillResident* r, int64_t li, RadTensor* w, RadTensor* scale,
                                      RadTensor* bias) {
    if (!r || li < 0 || li >= r->n_layer || r->w_at[(size_t)li] < 0) return RAD_E_INVAL;
    const int64_t n = r->n_embd, wide = r->wide;
    if (w) *w = device_view(r->at(r->w_at[(size_t)li]), r->int8 ? RAD_I8 : RAD_BF16, { n, wide });
    if (scale)
        *scale = r->int8 ? device_view(r->at(r->scale_at[(size_t)li]), RAD_F32, { wide / 128, n }) : RadTensor{};
    if (bias) *bias = device_view(r->at(r->bias_at[(size_t)li]), RAD_BF16, { n });
    return RAD_OK;
}

extern "C" int ridgefill_resident_correction(const RidgeFillResident* r, int64_t li, RadTensor* out) {
    if (!r || !out || li < 0 || li >= r->n_layer || r->st_at[(size_t)li] < 0) return RAD_E_INVAL;
    *out = device_view(r->at(r->st_at[(size_t)li]), RAD_F32, { r->heads, r->sd0, r->sd1 });
    return RAD_OK;
}

extern "C" int ridgefill_resident_table(const RidgeFillResident* r, const char* name, RadTensor* out) {
    if (!r || !name || !out) return RAD_E_INVAL;
    const auto it = r->table_at.find(name);
    if (it == r->table_at.end()) return RAD_E_INVAL;
    *out = device_view(r->at(it->second), RAD_F32, { r->n_vocab });
    return RAD_OK;
}

extern "C" int ridgefill_resident_final(const RidgeFillResident* r, RadTensor* w, RadTensor* bias) {
    if (!r || r->final_w_at < 0) return RAD_E_INVAL;
    if (w) *w = device_view(r->at(r->final_w_at), RAD_BF16, { r->wide, r->wide });
    if (bias) *bias = device_view(r->at(r->final_b_at), RAD_BF16, { r->wide });
    return RAD_OK;
}
