// Minimal GGUF (v2/v3) reader for the decoder checkpoint: KV metadata and
// tensor infos, with tensor bytes read straight from the file.  Replaces the
// ggml gguf.cpp parsing that VoxCPMWeightStore::load_from_file relies on in
// the reference (src/weight-store.cpp:78-225) for the types this path needs
// (F32, F16, Q4_0, Q8_0).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace vxb {

enum GgmlType : int { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ8_0 = 8 };

struct GgufTensorInfo {
    std::string name;
    int type = 0;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;  // relative to the data section
    size_t nbytes = 0;
};

struct GgufValue {
    int type = -1;  // GGUF value type
    uint64_t u = 0;
    int64_t i = 0;
    bool b = false;
    std::string s;
    std::vector<int64_t> arr_i;  // integer arrays
};

class GgufFile {
public:
    // Returns false and fills err on a malformed or unreadable file.
    bool open(const std::string& path, std::string* err);
    const GgufTensorInfo* find(const std::string& name) const;
    const GgufValue* kv(const std::string& key) const;
    // Reads the bytes of one tensor into dst (nbytes of it).
    bool read_tensor(const GgufTensorInfo& t, void* dst, std::string* err) const;

    std::vector<GgufTensorInfo> tensors;
    std::map<std::string, GgufValue> kvs;
    std::string path;
    uint64_t data_offset = 0;
};

// Bytes of a tensor of `type` with `nelem` elements; 0 for unsupported types.
size_t ggml_type_nbytes(int type, int64_t nelem);

}  // namespace vxb
