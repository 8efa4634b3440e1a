/**
 * @file context.h
 * @brief Graph metadata arena (reference include/voxcpm/context.h:51-108).
 */
#ifndef VOXCPM_CONTEXT_H
#define VOXCPM_CONTEXT_H

#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

#include "voxcpm/common.h"

namespace voxcpm {

enum class ContextType {
    Weights,
    Graph,
};

class VOXCPM_API VoxCPMContext {
public:
    VoxCPMContext(ContextType type, int n_tensors, int max_nodes = 0, size_t extra_mem_size = 0);
    ~VoxCPMContext();
    VoxCPMContext(const VoxCPMContext&) = delete;
    VoxCPMContext& operator=(const VoxCPMContext&) = delete;
    VoxCPMContext(VoxCPMContext&& other) noexcept;
    VoxCPMContext& operator=(VoxCPMContext&& other) noexcept;

    ggml_tensor* new_tensor_2d(ggml_type type, int64_t ne0, int64_t ne1);
    ggml_tensor* new_tensor_3d(ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2);
    ggml_cgraph* new_graph();
    ggml_cgraph* new_graph(size_t size);
    void build_forward(ggml_cgraph* graph, ggml_tensor* output);

    ggml_context* raw_context() const { return ctx_; }
    ContextType type() const { return type_; }
    size_t mem_size() const { return mem_size_; }
    size_t max_nodes() const { return max_nodes_; }
    bool is_valid() const { return ctx_ != nullptr; }

    // Internal: a new node (tensor) owned by this context.
    ggml_tensor* new_node(ggml_type type, int n_dims, const int64_t* ne);

private:
    ContextType type_;
    ggml_context* ctx_;
    size_t mem_size_;
    size_t max_nodes_;
};

}  // namespace voxcpm

#endif  // VOXCPM_CONTEXT_H
