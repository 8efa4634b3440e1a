#include "gguf_reader.h"

#include <cstdio>
#include <cstring>
#include <memory>

namespace vxb {

namespace {

// GGUF value types
enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32v = 6, kBool = 7,
    kStr = 8, kArr = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

struct Reader {
    FILE* f = nullptr;
    bool ok = true;
    template <class T>
    T get() {
        T v{};
        if (ok && std::fread(&v, sizeof(T), 1, f) != 1) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 20)) {
            ok = false;
            return {};
        }
        std::string s(n, '\0');
        if (n && std::fread(&s[0], 1, n, f) != n) ok = false;
        return s;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32v: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

int64_t read_int(Reader& r, uint32_t t) {
    switch (t) {
        case kU8: return r.get<uint8_t>();
        case kI8: return r.get<int8_t>();
        case kU16: return r.get<uint16_t>();
        case kI16: return r.get<int16_t>();
        case kU32: return r.get<uint32_t>();
        case kI32: return r.get<int32_t>();
        case kU64: return static_cast<int64_t>(r.get<uint64_t>());
        case kI64: return r.get<int64_t>();
        case kBool: return r.get<uint8_t>();
        case kF32v: return static_cast<int64_t>(r.get<float>());
        case kF64: return static_cast<int64_t>(r.get<double>());
        default: r.ok = false; return 0;
    }
}

}  // namespace

size_t ggml_type_nbytes(int type, int64_t n) {
    switch (type) {
        case kF32: return static_cast<size_t>(n) * 4;
        case kF16: return static_cast<size_t>(n) * 2;
        case kQ4_0: return n % 32 ? 0 : static_cast<size_t>(n / 32) * 18;
        case kQ8_0: return n % 32 ? 0 : static_cast<size_t>(n / 32) * 34;
        default: return 0;
    }
}

bool GgufFile::open(const std::string& p, std::string* err) {
    path = p;
    std::unique_ptr<FILE, int (*)(FILE*)> fh(std::fopen(p.c_str(), "rb"), &std::fclose);
    if (!fh) {
        *err = "cannot open " + p;
        return false;
    }
    Reader r{fh.get()};
    char magic[4];
    if (std::fread(magic, 1, 4, r.f) != 4 || std::memcmp(magic, "GGUF", 4) != 0) {
        *err = "not a GGUF file: " + p;
        return false;
    }
    const uint32_t version = r.get<uint32_t>();
    if (version < 2 || version > 3) {
        *err = "unsupported GGUF version";
        return false;
    }
    const uint64_t n_t = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (!r.ok || n_t > (1u << 20) || n_kv > (1u << 20)) {
        *err = "corrupt GGUF header";
        return false;
    }
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string key = r.str();
        GgufValue v;
        v.type = static_cast<int>(r.get<uint32_t>());
        if (v.type == kStr) {
            v.s = r.str();
        } else if (v.type == kArr) {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t n = r.get<uint64_t>();
            if (n > (1u << 24)) {
                r.ok = false;
                break;
            }
            for (uint64_t j = 0; j < n && r.ok; ++j) {
                if (et == kStr) {
                    r.str();
                } else if (scalar_size(et)) {
                    v.arr_i.push_back(read_int(r, et));
                } else {
                    r.ok = false;
                }
            }
        } else if (scalar_size(v.type)) {
            v.i = read_int(r, v.type);
            v.u = static_cast<uint64_t>(v.i);
            v.b = v.i != 0;
        } else {
            r.ok = false;
        }
        if (key == "general.alignment" && v.u) alignment = v.u;
        kvs[key] = v;
    }
    for (uint64_t i = 0; i < n_t && r.ok; ++i) {
        GgufTensorInfo t;
        t.name = r.str();
        t.n_dims = static_cast<int>(r.get<uint32_t>());
        if (t.n_dims < 1 || t.n_dims > 4) {
            r.ok = false;
            break;
        }
        int64_t n = 1;
        for (int d = 0; d < t.n_dims; ++d) {
            t.ne[d] = static_cast<int64_t>(r.get<uint64_t>());
            n *= t.ne[d];
        }
        t.type = static_cast<int>(r.get<uint32_t>());
        t.offset = r.get<uint64_t>();
        t.nbytes = ggml_type_nbytes(t.type, n);
        tensors.push_back(t);
    }
    if (!r.ok) {
        *err = "truncated or corrupt GGUF metadata";
        return false;
    }
    const long pos = std::ftell(r.f);
    data_offset = (static_cast<uint64_t>(pos) + alignment - 1) / alignment * alignment;
    return true;
}

const GgufTensorInfo* GgufFile::find(const std::string& name) const {
    for (const auto& t : tensors)
        if (t.name == name) return &t;
    return nullptr;
}

const GgufValue* GgufFile::kv(const std::string& key) const {
    auto it = kvs.find(key);
    return it == kvs.end() ? nullptr : &it->second;
}

bool GgufFile::read_tensor(const GgufTensorInfo& t, void* dst, std::string* err) const {
    std::unique_ptr<FILE, int (*)(FILE*)> fh(std::fopen(path.c_str(), "rb"), &std::fclose);
    if (!fh) {
        *err = "cannot reopen " + path;
        return false;
    }
    if (std::fseek(fh.get(), static_cast<long>(data_offset + t.offset), SEEK_SET) != 0 ||
        std::fread(dst, 1, t.nbytes, fh.get()) != t.nbytes) {
        *err = "short read of tensor " + t.name;
        return false;
    }
    return true;
}

}  // namespace vxb
