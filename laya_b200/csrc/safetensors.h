// safetensors.h — the safetensors container (host C++): an 8-byte little-endian header length, a JSON header of
// {name: {dtype, shape, data_offsets}} (plus "__metadata__": {string: string}) padded with spaces to 8 bytes, then
// the raw little-endian tensor bytes.  The layout SafetensorsWriter (Base/Io/SafetensorsWriter.cs:10-64) writes and
// the checkpoint loaders read; F32, F16 and BF16 payloads.
#pragma once
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace laya {
namespace st {

struct Entry {
    std::string dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;
};

struct Header {
    std::map<std::string, Entry> tensors;
    std::map<std::string, std::string> metadata;
    uint64_t data_start = 0;   // file offset of the payload
};

inline int elem_size(const std::string& dtype) {
    if (dtype == "F32") return 4;
    if (dtype == "F16" || dtype == "BF16") return 2;
    return 0;
}

// fp32 → bf16 bits, round to nearest even, NaN kept quiet (SafetensorsWriter.ToBFloat16, :77-83).
inline uint16_t to_bf16(float value) {
    uint32_t bits;
    std::memcpy(&bits, &value, 4);
    if ((bits & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((bits >> 16) | 0x40);
    const uint32_t rounding = 0x7FFFu + ((bits >> 16) & 1u);
    return static_cast<uint16_t>((bits + rounding) >> 16);
}
inline float from_bf16(uint16_t b) {
    const uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

inline std::string escape(const std::string& s) {
    std::string o;
    for (char c : s) {
        if (c == '"' || c == '\\') { o += '\\'; o += c; }
        else if (static_cast<unsigned char>(c) < 0x20) { char b[8]; std::snprintf(b, sizeof b, "\\u%04x", c); o += b; }
        else o += c;
    }
    return o;
}

// ---- a minimal JSON reader for the header: objects, arrays, strings, integers
struct Reader {
    const char* p;
    const char* e;
    bool ok = true;
    void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
    bool eat(char c) { ws(); if (p < e && *p == c) { ++p; return true; } return false; }
    std::string str() {
        std::string o;
        ws();
        if (p >= e || *p != '"') { ok = false; return o; }
        ++p;
        while (p < e && *p != '"') {
            if (*p == '\\' && p + 1 < e) {
                ++p;
                switch (*p) {
                    case 'n': o += '\n'; break;
                    case 't': o += '\t'; break;
                    case 'r': o += '\r'; break;
                    case 'b': o += '\b'; break;
                    case 'f': o += '\f'; break;
                    case 'u': {
                        if (e - p < 5) { ok = false; return o; }
                        unsigned v = static_cast<unsigned>(std::strtoul(std::string(p + 1, 4).c_str(), nullptr, 16));
                        if (v < 0x80) o += static_cast<char>(v);
                        else if (v < 0x800) { o += static_cast<char>(0xC0 | (v >> 6)); o += static_cast<char>(0x80 | (v & 0x3F)); }
                        else { o += static_cast<char>(0xE0 | (v >> 12)); o += static_cast<char>(0x80 | ((v >> 6) & 0x3F)); o += static_cast<char>(0x80 | (v & 0x3F)); }
                        p += 4;
                        break;
                    }
                    default: o += *p;
                }
                ++p;
            } else {
                o += *p++;
            }
        }
        if (p >= e) { ok = false; return o; }
        ++p;
        return o;
    }
    int64_t integer() {
        ws();
        char* q = nullptr;
        const long long v = std::strtoll(p, &q, 10);
        if (q == p) ok = false;
        p = q;
        return v;
    }
    void skip() {   // any value
        ws();
        if (p >= e) { ok = false; return; }
        if (*p == '"') { str(); return; }
        if (*p == '{') { ++p; if (eat('}')) return; do { str(); if (!eat(':')) { ok = false; return; } skip(); } while (ok && eat(',')); if (!eat('}')) ok = false; return; }
        if (*p == '[') { ++p; if (eat(']')) return; do { skip(); } while (ok && eat(',')); if (!eat(']')) ok = false; return; }
        while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
    }
};

// Parses the header of a safetensors file; false with a message on a malformed file.
inline bool read_header(std::FILE* f, Header* h, std::string* err) {
    uint64_t n = 0;
    unsigned char len[8];
    if (std::fread(len, 1, 8, f) != 8) { *err = "file shorter than the header length"; return false; }
    for (int i = 7; i >= 0; --i) n = (n << 8) | len[i];
    if (n == 0 || n > (1ull << 30)) { *err = "implausible header length"; return false; }
    std::string js(n, '\0');
    if (std::fread(&js[0], 1, n, f) != n) { *err = "file shorter than its header"; return false; }
    h->data_start = 8 + n;
    Reader r{js.data(), js.data() + js.size()};
    if (!r.eat('{')) { *err = "header is not a JSON object"; return false; }
    if (!r.eat('}')) {
        do {
            const std::string name = r.str();
            if (!r.ok || !r.eat(':')) break;
            if (name == "__metadata__") {
                if (!r.eat('{')) { r.ok = false; break; }
                if (!r.eat('}')) {
                    do {
                        const std::string k = r.str();
                        if (!r.eat(':')) { r.ok = false; break; }
                        h->metadata[k] = r.str();
                    } while (r.ok && r.eat(','));
                    if (!r.eat('}')) r.ok = false;
                }
                continue;
            }
            Entry en;
            if (!r.eat('{')) { r.ok = false; break; }
            do {
                const std::string k = r.str();
                if (!r.eat(':')) { r.ok = false; break; }
                if (k == "dtype") en.dtype = r.str();
                else if (k == "shape") {
                    if (!r.eat('[')) { r.ok = false; break; }
                    if (!r.eat(']')) { do { en.shape.push_back(r.integer()); } while (r.ok && r.eat(',')); if (!r.eat(']')) r.ok = false; }
                } else if (k == "data_offsets") {
                    if (!r.eat('[')) { r.ok = false; break; }
                    en.begin = static_cast<uint64_t>(r.integer());
                    if (!r.eat(',')) { r.ok = false; break; }
                    en.end = static_cast<uint64_t>(r.integer());
                    if (!r.eat(']')) r.ok = false;
                } else r.skip();
            } while (r.ok && r.eat(','));
            if (!r.eat('}')) r.ok = false;
            h->tensors[name] = en;
        } while (r.ok && r.eat(','));
        if (r.ok && !r.eat('}')) r.ok = false;
    }
    if (!r.ok) { *err = "malformed JSON header"; return false; }
    return true;
}

}  // namespace st
}  // namespace laya
