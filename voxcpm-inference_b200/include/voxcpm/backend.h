/**
 * @file backend.h
 * @brief Compute backend (reference include/voxcpm/backend.h:24-183).
 *
 * BackendType::CUDA runs the decode graph on a B200 through libvxb; this
 * build provides no CPU or HTP execution, and asking for them throws
 * voxcpm::Error(ErrorCode::NotImplemented) instead of falling back.
 */
#ifndef VOXCPM_BACKEND_H
#define VOXCPM_BACKEND_H

#include <memory>
#include <string>
#include <vector>

#include "voxcpm/common.h"

struct vxb_ctx;

namespace voxcpm {

enum class BackendType {
    CPU,
    HTP,
    CUDA,
};

class VOXCPM_API VoxCPMBackend {
public:
    explicit VoxCPMBackend(BackendType type = BackendType::CUDA, int n_threads = 4, int device = 0);
    ~VoxCPMBackend();
    VoxCPMBackend(const VoxCPMBackend&) = delete;
    VoxCPMBackend& operator=(const VoxCPMBackend&) = delete;
    VoxCPMBackend(VoxCPMBackend&& other) noexcept;
    VoxCPMBackend& operator=(VoxCPMBackend&& other) noexcept;

    void init_allocator() {}
    // Builds the launch plan (and its CUDA graph) for the decode node's shape.
    void reserve_compute_memory(ggml_cgraph* graph, const char* stage = nullptr);
    // Binds host staging to the graph's input and output tensors.
    void alloc_graph(ggml_cgraph* graph, const char* stage = nullptr);
    // Host->device copy of the latent, the decode, device->host copy of the audio.
    ggml_status compute(ggml_cgraph* graph);
    void tensor_set(ggml_tensor* tensor, const void* data, size_t offset, size_t size);
    void tensor_set(ggml_tensor* tensor, const void* data) { tensor_set(tensor, data, 0, ggml_nbytes(tensor)); }
    void tensor_get(const ggml_tensor* tensor, void* data, size_t offset, size_t size);
    void tensor_get(const ggml_tensor* tensor, void* data) { tensor_get(tensor, data, 0, ggml_nbytes(tensor)); }

    int n_threads() const { return n_threads_; }
    BackendType type() const { return type_; }
    const char* backend_name() const { return "CUDA"; }
    const char* backend_description() const { return description_.c_str(); }
    bool is_htp_active() const { return false; }
    size_t compute_buffer_size() const { return staging_bytes_; }

    // The libvxb context of this backend.
    vxb_ctx* vxb() const { return ctx_; }

private:
    BackendType type_;
    int n_threads_;
    vxb_ctx* ctx_ = nullptr;
    std::string description_;
    std::vector<std::unique_ptr<std::vector<uint8_t>>> staging_;  // host buffers of graph tensors
    size_t staging_bytes_ = 0;
    int plan_b_ = 0, plan_t_ = 0;
    int enc_plan_t_ = 0;  // frames of the encode plan (batch 1)
};

}  // namespace voxcpm

#endif  // VOXCPM_BACKEND_H
