// gguf_reader.cpp -- see gguf_reader.h.
#include "gguf_reader.h"

#include <cstdio>
#include <cstring>

namespace gsvcu {

namespace {

struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <class T>
    T get() {
        T v{};
        if ((size_t)(end - p) < sizeof(T)) { ok = false; return v; }
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || (uint64_t)(end - p) < n) { ok = false; return {}; }
        std::string s((const char*)p, (size_t)n);
        p += n;
        return s;
    }
    void skip(uint64_t n) {
        if ((uint64_t)(end - p) < n) { ok = false; return; }
        p += n;
    }
};

// GGUF value types
enum { U8 = 0, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 };

size_t scalar_size(uint32_t t) {
    switch (t) {
        case U8: case I8: case BOOL: return 1;
        case U16: case I16: return 2;
        case U32: case I32: case F32: return 4;
        case U64: case I64: case F64: return 8;
        default: return 0;
    }
}

bool skip_value(Cursor& c, uint32_t t, int depth = 0) {
    if (t == STR) { c.str(); return c.ok; }
    if (t == ARR) {
        if (depth > 4) return false;
        const uint32_t et = c.get<uint32_t>();
        const uint64_t n = c.get<uint64_t>();
        if (!c.ok) return false;
        const size_t es = scalar_size(et);
        if (es) { c.skip(n * es); return c.ok; }
        for (uint64_t i = 0; i < n && c.ok; i++)
            if (!skip_value(c, et, depth + 1)) return false;
        return c.ok;
    }
    const size_t s = scalar_size(t);
    if (!s) return false;
    c.skip(s);
    return c.ok;
}

}  // namespace

bool GgufFile::open(const std::string& path, std::string& err) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) { err = "cannot open " + path; return false; }
    std::fseek(f, 0, SEEK_END);
    const long sz = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    if (sz <= 0) { std::fclose(f); err = "empty file " + path; return false; }
    buf_.resize((size_t)sz);
    const size_t rd = std::fread(buf_.data(), 1, (size_t)sz, f);
    std::fclose(f);
    if (rd != (size_t)sz) { err = "short read " + path; return false; }

    Cursor c{buf_.data(), buf_.data() + buf_.size()};
    const uint32_t magic = c.get<uint32_t>();
    if (!c.ok || magic != 0x46554747u) { err = "not a GGUF file: " + path; return false; }
    const uint32_t version = c.get<uint32_t>();
    if (version < 2 || version > 3) { err = "unsupported GGUF version " + std::to_string(version); return false; }
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    if (!c.ok || n_tensors > (1u << 20) || n_kv > (1u << 20)) { err = "corrupt GGUF header"; return false; }
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv; i++) {
        const std::string key = c.str();
        const uint32_t t = c.get<uint32_t>();
        if (!c.ok) { err = "corrupt GGUF KV section"; return false; }
        if (t == U8 || t == U16 || t == U32 || t == U64 || t == I8 || t == I16 || t == I32 || t == I64) {
            uint64_t v = 0;
            switch (t) {
                case U8: v = c.get<uint8_t>(); break;
                case I8: v = (uint64_t)(int64_t)c.get<int8_t>(); break;
                case U16: v = c.get<uint16_t>(); break;
                case I16: v = (uint64_t)(int64_t)c.get<int16_t>(); break;
                case U32: v = c.get<uint32_t>(); break;
                case I32: v = (uint64_t)(int64_t)c.get<int32_t>(); break;
                case U64: v = c.get<uint64_t>(); break;
                default: v = (uint64_t)c.get<int64_t>(); break;
            }
            if (!c.ok) { err = "corrupt GGUF KV section"; return false; }
            u64_[key] = v;
            if (key == "general.alignment") alignment = v;
        } else if (t == F32) {
            const float v = c.get<float>();
            if (!c.ok) { err = "corrupt GGUF KV section"; return false; }
            f32_[key] = v;
        } else if (!skip_value(c, t)) {
            err = "corrupt GGUF value for key " + key;
            return false;
        }
    }
    if (alignment == 0 || (alignment & (alignment - 1))) { err = "bad GGUF alignment"; return false; }
    tensors_.resize((size_t)n_tensors);
    for (uint64_t i = 0; i < n_tensors; i++) {
        GgufTensor& T = tensors_[(size_t)i];
        T.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (!c.ok || nd == 0 || nd > 4) { err = "corrupt GGUF tensor info"; return false; }
        T.dims.resize(nd);
        int64_t ne = 1;
        for (uint32_t d = 0; d < nd; d++) {
            T.dims[d] = (int64_t)c.get<uint64_t>();
            if (T.dims[d] <= 0 || T.dims[d] > (1ll << 32)) { err = "bad tensor dims for " + T.name; return false; }
            ne *= T.dims[d];
        }
        T.type = c.get<uint32_t>();
        T.offset = c.get<uint64_t>();
        if (!c.ok) { err = "corrupt GGUF tensor info"; return false; }
        switch (T.type) {
            case 0: T.nbytes = (uint64_t)ne * 4; break;
            case 1:    // F16
            case 30:   // BF16
                T.nbytes = (uint64_t)ne * 2;
                break;
            case 2:    // Q4_0: fp16 d + 16 bytes of nibbles per 32 values
            case 20:   // IQ4_NL: fp16 d + 16 bytes of nibbles (table indices)
            case 6:    // Q5_0: fp16 d + 4 bytes of high bits + 16 bytes of nibbles
            case 8:    // Q8_0: fp16 d + 32 int8
            case 3:    // Q4_1: fp16 d, m + 16 bytes of nibbles
            case 7:    // Q5_1: fp16 d, m + 4 bytes of high bits + 16 bytes of nibbles
                if (T.dims[0] % 32) { err = "block-quantized row not a multiple of 32: " + T.name; return false; }
                T.nbytes = (uint64_t)ne / 32 *
                           (T.type == 8 ? 34 : T.type == 7 ? 24 : T.type == 6 ? 22 : T.type == 3 ? 20 : 18);
                break;
            case 12:   // Q4_K: 144 bytes per 256 values
            case 13:   // Q5_K: 176 bytes
            case 14:   // Q6_K: 210 bytes
                if (T.dims[0] % 256) { err = "K-quant row not a multiple of 256: " + T.name; return false; }
                T.nbytes = (uint64_t)ne / 256 * (T.type == 12 ? 144 : T.type == 13 ? 176 : 210);
                break;
            default: T.nbytes = 0; break;   // unsupported types are rejected by the consumer
        }
        index_[T.name] = (size_t)i;
    }
    const uint64_t hdr = (uint64_t)(c.p - buf_.data());
    const uint64_t data_off = (hdr + alignment - 1) / alignment * alignment;
    for (GgufTensor& T : tensors_) {
        if (T.nbytes == 0) continue;
        if (data_off + T.offset + T.nbytes > buf_.size()) { err = "tensor data out of file bounds: " + T.name; return false; }
        T.data = buf_.data() + data_off + T.offset;
    }
    return true;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

bool GgufFile::get_f32(const std::string& key, float& out) const {
    auto it = f32_.find(key);
    if (it == f32_.end()) return false;
    out = it->second;
    return true;
}

bool GgufFile::get_u32(const std::string& key, uint32_t& out) const {
    auto it = u64_.find(key);
    if (it == u64_.end()) return false;
    out = (uint32_t)it->second;
    return true;
}

}  // namespace gsvcu
