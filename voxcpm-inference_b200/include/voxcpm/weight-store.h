/**
 * @file weight-store.h
 * @brief GGUF weight store (reference include/voxcpm/weight-store.h:20-69).
 *
 * load_from_file parses the GGUF on the host and uploads every tensor's
 * bytes unchanged to the backend's GPU.  get_tensor returns the tensor's
 * metadata (its data lives in device memory and is not host-addressable).
 */
#ifndef VOXCPM_WEIGHT_STORE_H
#define VOXCPM_WEIGHT_STORE_H

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "voxcpm/common.h"

namespace voxcpm {

class VoxCPMBackend;

using WeightGroupFn = bool (*)(const ggml_tensor* t);

class VOXCPM_API VoxCPMWeightStore {
public:
    VoxCPMWeightStore() = default;
    ~VoxCPMWeightStore();
    VoxCPMWeightStore(const VoxCPMWeightStore&) = delete;
    VoxCPMWeightStore& operator=(const VoxCPMWeightStore&) = delete;

    // group_fn (the reference's HTP bucketing) is accepted and ignored.
    bool load_from_file(const std::string& gguf_path, VoxCPMBackend& backend, WeightGroupFn group_fn = nullptr);
    ggml_tensor* get_tensor(const char* name) const;
    bool get_u32(const char* key, uint32_t& value) const;
    bool get_bool(const char* key, bool& value) const;
    bool get_string(const char* key, std::string& value) const;
    bool get_i32_array(const char* key, std::vector<int>& values) const;

    const std::string& path() const { return path_; }
    int tensor_count() const { return static_cast<int>(tensors_.size()); }
    bool owns_storage() const { return backend_ != nullptr && !tensors_.empty(); }
    VoxCPMBackend* backend() const { return backend_; }

private:
    struct Impl;
    std::shared_ptr<Impl> kv_;
    std::map<std::string, std::unique_ptr<ggml_tensor>> tensors_;
    VoxCPMBackend* backend_ = nullptr;
    std::string path_;
};

using SharedWeightStore = std::shared_ptr<VoxCPMWeightStore>;

}  // namespace voxcpm

#endif  // VOXCPM_WEIGHT_STORE_H
