// Fixture-format reader / writer (host C++): version 1/2 manifests of JSON array descriptors
// plus a little-endian binary payload, the format of the reference's test fixtures
// (tests/oracles/fixture.py:13-49).  read_fixture's checks are kept with its messages:
// version 1 or 2 and little endian ("Unsupported fixture format"), payload length and SHA-256
// ("Fixture payload length/hash mismatch"), 4-byte aligned offsets, nbytes = prod(shape) *
// itemsize and in range ("Invalid array descriptor: <name>").  write_fixture's layout is kept:
// arrays in order, each starting on a 4-byte boundary (zero padding), the payload padded to
// 4 bytes, the manifest = metadata + version, endianness, binary, byte_length, sha256, arrays.
//
// SHA-256 is FIPS 180-4; its round constants and initial hash are computed here from their
// definition (the first 32 fractional bits of the cube / square roots of the first primes).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include <sys/stat.h>

#include "bgtq_internal.h"

namespace bgtq {
namespace fx {

// ---- SHA-256 ----
struct Sha256Consts {
    uint32_t k[64], h0[8];
    Sha256Consts() {
        int primes[64], n = 0;
        for (int c = 2; n < 64; ++c) {
            bool p = true;
            for (int q = 2; q * q <= c; ++q)
                if (c % q == 0) { p = false; break; }
            if (p) primes[n++] = c;
        }
        auto frac32 = [](long double x) {
            const long double f = x - floorl(x);
            return (uint32_t)(uint64_t)floorl(f * 4294967296.0L);
        };
        for (int i = 0; i < 64; ++i) k[i] = frac32(cbrtl((long double)primes[i]));
        for (int i = 0; i < 8; ++i) h0[i] = frac32(sqrtl((long double)primes[i]));
    }
};

std::string sha256_hex(const unsigned char *data, size_t len) {
    static const Sha256Consts C;
    uint32_t h[8];
    std::memcpy(h, C.h0, sizeof(h));
    auto rotr = [](uint32_t x, int r) { return (x >> r) | (x << (32 - r)); };
    auto block = [&](const unsigned char *b) {
        uint32_t w[64];
        for (int i = 0; i < 16; ++i)
            w[i] = (uint32_t)b[4 * i] << 24 | (uint32_t)b[4 * i + 1] << 16 | (uint32_t)b[4 * i + 2] << 8 | b[4 * i + 3];
        for (int i = 16; i < 64; ++i) {
            const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        uint32_t a = h[0], bb = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
        for (int i = 0; i < 64; ++i) {
            const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25), ch = (e & f) ^ (~e & g);
            const uint32_t t1 = hh + S1 + ch + C.k[i] + w[i];
            const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22), mj = (a & bb) ^ (a & c) ^ (bb & c);
            const uint32_t t2 = S0 + mj;
            hh = g; g = f; f = e; e = d + t1; d = c; c = bb; bb = a; a = t1 + t2;
        }
        h[0] += a; h[1] += bb; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
    };
    size_t i = 0;
    for (; i + 64 <= len; i += 64) block(data + i);
    unsigned char tail[128] = {0};
    const size_t rem = len - i;
    std::memcpy(tail, data + i, rem);
    tail[rem] = 0x80;
    const size_t tl = rem + 9 <= 64 ? 64 : 128;
    const uint64_t bits = (uint64_t)len * 8;
    for (int b = 0; b < 8; ++b) tail[tl - 1 - b] = (unsigned char)(bits >> (8 * b));
    block(tail);
    if (tl == 128) block(tail + 64);
    char out[65];
    for (int k = 0; k < 8; ++k) std::snprintf(out + 8 * k, 9, "%08x", h[k]);
    return std::string(out, 64);
}

// ---- minimal JSON ----
struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;  // insertion order
    const Json *get(const std::string &k) const {
        for (auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct Parser {
    const std::string &s;
    size_t i = 0;
    bool ok = true;
    explicit Parser(const std::string &t) : s(t) {}
    void ws() { while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i; }
    bool lit(const char *w) {
        const size_t n = std::strlen(w);
        if (s.compare(i, n, w) == 0) { i += n; return true; }
        return false;
    }
    std::string string() {
        std::string out;
        if (s[i] != '"') { ok = false; return out; }
        ++i;
        while (i < s.size() && s[i] != '"') {
            char c = s[i++];
            if (c == '\\') {
                if (i >= s.size()) { ok = false; return out; }
                const char e = s[i++];
                switch (e) {
                    case '"': out += '"'; break;
                    case '\\': out += '\\'; break;
                    case '/': out += '/'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'n': out += '\n'; break;
                    case 'r': out += '\r'; break;
                    case 't': out += '\t'; break;
                    case 'u': {
                        if (i + 4 > s.size()) { ok = false; return out; }
                        unsigned cp = 0;
                        for (int k = 0; k < 4; ++k) {
                            const char hch = s[i + k];
                            const int dv = hch >= '0' && hch <= '9' ? hch - '0'
                                           : hch >= 'a' && hch <= 'f' ? hch - 'a' + 10
                                           : hch >= 'A' && hch <= 'F' ? hch - 'A' + 10 : -1;
                            if (dv < 0) { ok = false; return out; }
                            cp = cp * 16 + (unsigned)dv;
                        }
                        i += 4;
                        if (cp < 0x80) out += (char)cp;
                        else if (cp < 0x800) { out += (char)(0xc0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3f)); }
                        else { out += (char)(0xe0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3f)); out += (char)(0x80 | (cp & 0x3f)); }
                        break;
                    }
                    default: ok = false; return out;
                }
            } else {
                out += c;
            }
        }
        if (i >= s.size()) { ok = false; return out; }
        ++i;
        return out;
    }
    Json value() {
        Json v;
        ws();
        if (i >= s.size()) { ok = false; return v; }
        const char c = s[i];
        if (c == '{') {
            v.kind = Json::Obj;
            ++i;
            ws();
            if (i < s.size() && s[i] == '}') { ++i; return v; }
            while (ok) {
                ws();
                std::string k = string();
                ws();
                if (i >= s.size() || s[i] != ':') { ok = false; break; }
                ++i;
                v.obj.emplace_back(k, value());
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                if (i < s.size() && s[i] == '}') { ++i; break; }
                ok = false;
            }
        } else if (c == '[') {
            v.kind = Json::Arr;
            ++i;
            ws();
            if (i < s.size() && s[i] == ']') { ++i; return v; }
            while (ok) {
                v.arr.push_back(value());
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                if (i < s.size() && s[i] == ']') { ++i; break; }
                ok = false;
            }
        } else if (c == '"') {
            v.kind = Json::Str;
            v.str = string();
        } else if (lit("true")) {
            v.kind = Json::Bool; v.b = true;
        } else if (lit("false")) {
            v.kind = Json::Bool;
        } else if (lit("null")) {
            v.kind = Json::Null;
        } else {
            size_t end = i;
            while (end < s.size() && std::strchr("+-0123456789.eE", s[end])) ++end;
            if (end == i) { ok = false; return v; }
            v.kind = Json::Num;
            v.num = std::strtod(s.substr(i, end - i).c_str(), nullptr);
            i = end;
        }
        return v;
    }
};

void dump(const Json &v, std::ostringstream &o, int indent, int depth) {
    auto pad = [&](int d) { o << '\n' << std::string((size_t)(indent * d), ' '); };
    switch (v.kind) {
        case Json::Null: o << "null"; break;
        case Json::Bool: o << (v.b ? "true" : "false"); break;
        case Json::Num: {
            if (std::isfinite(v.num) && v.num == std::floor(v.num) && std::fabs(v.num) < 9007199254740992.0) {
                o << (long long)v.num;
            } else {
                char buf[40];
                std::snprintf(buf, sizeof(buf), "%.17g", v.num);
                o << buf;
            }
            break;
        }
        case Json::Str: {
            o << '"';
            for (unsigned char c : v.str) {
                if (c == '"') o << "\\\"";
                else if (c == '\\') o << "\\\\";
                else if (c == '\n') o << "\\n";
                else if (c < 0x20) { char b[8]; std::snprintf(b, sizeof(b), "\\u%04x", c); o << b; }
                else o << c;
            }
            o << '"';
            break;
        }
        case Json::Arr: {
            if (v.arr.empty()) { o << "[]"; break; }
            o << '[';
            for (size_t k = 0; k < v.arr.size(); ++k) {
                if (k) o << ',';
                pad(depth + 1);
                dump(v.arr[k], o, indent, depth + 1);
            }
            pad(depth);
            o << ']';
            break;
        }
        case Json::Obj: {
            if (v.obj.empty()) { o << "{}"; break; }
            o << '{';
            for (size_t k = 0; k < v.obj.size(); ++k) {
                if (k) o << ',';
                pad(depth + 1);
                Json key;
                key.kind = Json::Str;
                key.str = v.obj[k].first;
                dump(key, o, indent, depth + 1);
                o << ": ";
                dump(v.obj[k].second, o, indent, depth + 1);
            }
            pad(depth);
            o << '}';
            break;
        }
    }
}

size_t itemsize(const std::string &dt) {
    if (dt == "f32" || dt == "u32") return 4;
    if (dt == "f16" || dt == "u16") return 2;
    if (dt == "u8") return 1;
    return 0;
}

bool read_file(const std::string &path, std::string &out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::ostringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

// mkdir -p of the directory holding `path` (write_fixture creates its parent directories)
void make_parents(const std::string &path) {
    for (size_t i = 1; i < path.size(); ++i)
        if (path[i] == '/') mkdir(path.substr(0, i).c_str(), 0755);
}

std::string sibling(const std::string &json_path, const std::string &name) {
    const size_t slash = json_path.find_last_of('/');
    return slash == std::string::npos ? name : json_path.substr(0, slash + 1) + name;
}

}  // namespace fx
}  // namespace bgtq

struct bgtq_fixture {
    std::string manifest;  // the manifest text as read
    std::string payload;
    struct Array {
        std::string name, dtype;
        std::vector<uint64_t> shape;
        uint64_t offset, nbytes;
    };
    std::vector<Array> arrays;
};

using namespace bgtq;

extern "C" {

bgtq_status bgtq_fixture_read(const char *json_path, bgtq_fixture **out) {
    if (!json_path || !out) {
        set_last_error("bgtq_fixture_read: invalid arguments");
        return BGTQ_EINVAL;
    }
    *out = nullptr;
    std::unique_ptr<bgtq_fixture> f(new bgtq_fixture());
    if (!fx::read_file(json_path, f->manifest)) {
        set_last_error(std::string("cannot read ") + json_path);
        return BGTQ_EINVAL;
    }
    fx::Parser p(f->manifest);
    const fx::Json meta = p.value();
    if (!p.ok || meta.kind != fx::Json::Obj) {
        set_last_error("Unsupported fixture format");
        return BGTQ_ELAYOUT;
    }
    const fx::Json *ver = meta.get("version"), *end = meta.get("endianness"), *bin = meta.get("binary");
    if (!ver || ver->kind != fx::Json::Num || (ver->num != 1 && ver->num != 2) || !end || end->kind != fx::Json::Str ||
        end->str != "little" || !bin || bin->kind != fx::Json::Str) {
        set_last_error("Unsupported fixture format");
        return BGTQ_ELAYOUT;
    }
    const fx::Json *bl = meta.get("byte_length"), *sha = meta.get("sha256"), *arrs = meta.get("arrays");
    if (!fx::read_file(fx::sibling(json_path, bin->str), f->payload) || !bl || bl->kind != fx::Json::Num ||
        (double)f->payload.size() != bl->num || !sha || sha->kind != fx::Json::Str ||
        fx::sha256_hex(reinterpret_cast<const unsigned char *>(f->payload.data()), f->payload.size()) != sha->str) {
        set_last_error("Fixture payload length/hash mismatch");
        return BGTQ_ELAYOUT;
    }
    if (!arrs || arrs->kind != fx::Json::Obj) {
        set_last_error("Unsupported fixture format");
        return BGTQ_ELAYOUT;
    }
    for (auto &kv : arrs->obj) {
        const fx::Json &d = kv.second;
        const fx::Json *dt = d.get("dtype"), *sh = d.get("shape"), *of = d.get("offset"), *nb = d.get("nbytes");
        bool good = dt && dt->kind == fx::Json::Str && fx::itemsize(dt->str) && sh && sh->kind == fx::Json::Arr && of &&
                    of->kind == fx::Json::Num && nb && nb->kind == fx::Json::Num;
        bgtq_fixture::Array a;
        a.name = kv.first;
        uint64_t count = 1;
        if (good) {
            a.dtype = dt->str;
            for (auto &e : sh->arr) {
                if (e.kind != fx::Json::Num || e.num < 0) { good = false; break; }
                a.shape.push_back((uint64_t)e.num);
                count *= (uint64_t)e.num;
            }
            a.offset = (uint64_t)of->num;
            a.nbytes = (uint64_t)nb->num;
        }
        if (!good || a.offset % 4 || a.nbytes != count * fx::itemsize(a.dtype) ||
            a.offset + a.nbytes > f->payload.size()) {
            set_last_error("Invalid array descriptor: " + kv.first);
            return BGTQ_ELAYOUT;
        }
        f->arrays.push_back(a);
    }
    *out = f.release();
    return BGTQ_OK;
}

bgtq_status bgtq_fixture_array_count(const bgtq_fixture *f, uint32_t *n) {
    if (!f || !n) return BGTQ_EINVAL;
    *n = (uint32_t)f->arrays.size();
    return BGTQ_OK;
}

bgtq_status bgtq_fixture_array(const bgtq_fixture *f, uint32_t index, const char **name, const char **dtype,
                               uint32_t *ndim, const uint64_t **shape, const void **data, uint64_t *nbytes) {
    if (!f || index >= f->arrays.size()) {
        set_last_error("bgtq_fixture_array: index out of range");
        return BGTQ_EINVAL;
    }
    const auto &a = f->arrays[index];
    if (name) *name = a.name.c_str();
    if (dtype) *dtype = a.dtype.c_str();
    if (ndim) *ndim = (uint32_t)a.shape.size();
    if (shape) *shape = a.shape.data();
    if (data) *data = f->payload.data() + a.offset;
    if (nbytes) *nbytes = a.nbytes;
    return BGTQ_OK;
}

bgtq_status bgtq_fixture_manifest(const bgtq_fixture *f, const char **json) {
    if (!f || !json) return BGTQ_EINVAL;
    *json = f->manifest.c_str();
    return BGTQ_OK;
}

void bgtq_fixture_destroy(bgtq_fixture *f) { delete f; }

bgtq_status bgtq_fixture_write(const char *json_path, const char *metadata_json, uint32_t n_arrays,
                               const char *const *names, const char *const *dtypes, const uint32_t *ndims,
                               const uint64_t *const *shapes, const void *const *data) {
    if (!json_path || (n_arrays && (!names || !dtypes || !ndims || !shapes || !data))) {
        set_last_error("bgtq_fixture_write: invalid arguments");
        return BGTQ_EINVAL;
    }
    fx::Json meta;
    meta.kind = fx::Json::Obj;
    if (metadata_json && *metadata_json) {
        std::string text(metadata_json);
        fx::Parser p(text);
        meta = p.value();
        if (!p.ok || meta.kind != fx::Json::Obj) {
            set_last_error("bgtq_fixture_write: metadata must be a JSON object");
            return BGTQ_EINVAL;
        }
    }
    std::string payload;
    fx::Json descs;
    descs.kind = fx::Json::Obj;
    for (uint32_t k = 0; k < n_arrays; ++k) {
        const size_t is = fx::itemsize(dtypes[k] ? dtypes[k] : "");
        if (!is || !names[k]) {
            set_last_error("bgtq_fixture_write: unknown dtype");
            return BGTQ_EINVAL;
        }
        uint64_t count = 1;
        fx::Json shape;
        shape.kind = fx::Json::Arr;
        for (uint32_t d = 0; d < ndims[k]; ++d) {
            count *= shapes[k][d];
            fx::Json e;
            e.kind = fx::Json::Num;
            e.num = (double)shapes[k][d];
            shape.arr.push_back(e);
        }
        payload.append((4 - payload.size() % 4) % 4, '\0');
        fx::Json d;
        d.kind = fx::Json::Obj;
        fx::Json v;
        v.kind = fx::Json::Str; v.str = dtypes[k]; d.obj.emplace_back("dtype", v);
        d.obj.emplace_back("shape", shape);
        v = fx::Json(); v.kind = fx::Json::Num; v.num = (double)payload.size(); d.obj.emplace_back("offset", v);
        v.num = (double)(count * is); d.obj.emplace_back("nbytes", v);
        descs.obj.emplace_back(names[k], d);
        payload.append(static_cast<const char *>(data[k]), count * is);
    }
    payload.append((4 - payload.size() % 4) % 4, '\0');
    std::string path(json_path), stem = path;
    const size_t dot = stem.find_last_of('.'), slash = stem.find_last_of('/');
    if (dot != std::string::npos && (slash == std::string::npos || dot > slash)) stem = stem.substr(0, dot);
    const std::string bin_path = stem + ".bin";
    const std::string bin_name = bin_path.substr(bin_path.find_last_of('/') == std::string::npos ? 0 : bin_path.find_last_of('/') + 1);
    auto set = [&](const std::string &k, const fx::Json &v) {
        for (auto &kv : meta.obj)
            if (kv.first == k) { kv.second = v; return; }
        meta.obj.emplace_back(k, v);
    };
    fx::Json v;
    if (!meta.get("version")) { v.kind = fx::Json::Num; v.num = 1; set("version", v); }
    v = fx::Json(); v.kind = fx::Json::Str; v.str = "little"; set("endianness", v);
    v.str = bin_name; set("binary", v);
    v = fx::Json(); v.kind = fx::Json::Num; v.num = (double)payload.size(); set("byte_length", v);
    v = fx::Json(); v.kind = fx::Json::Str;
    v.str = fx::sha256_hex(reinterpret_cast<const unsigned char *>(payload.data()), payload.size());
    set("sha256", v);
    set("arrays", descs);
    fx::make_parents(path);
    std::ofstream fb(bin_path, std::ios::binary);
    fb.write(payload.data(), (std::streamsize)payload.size());
    if (!fb) {
        set_last_error("cannot write " + bin_path);
        return BGTQ_EINVAL;
    }
    std::ostringstream o;
    fx::dump(meta, o, 2, 0);
    std::ofstream fj(path, std::ios::binary);
    fj << o.str() << '\n';
    if (!fj) {
        set_last_error("cannot write " + path);
        return BGTQ_EINVAL;
    }
    return BGTQ_OK;
}

}  // extern "C"
