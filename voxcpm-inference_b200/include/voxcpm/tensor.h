/**
 * @file tensor.h
 * @brief Tensor / graph handles of the voxcpm C++ API on the B200 backend.
 *
 * The reference API (nowang6/voxcpm-inference, include/voxcpm/*.h) passes
 * ggml handles: ggml_tensor*, ggml_cgraph*, ggml_context*, ggml_type and
 * ggml_status.  This header declares the same names with the fields and
 * functions a caller of the decode path touches (ne/nb/type/data/name,
 * ggml_set_input, ggml_set_output, ggml_nelements, ggml_nbytes, ggml_n_dims,
 * ggml_build_forward_expand), so caller code such as the reference's
 * decode_waveform (vae_decode_mock.cpp:1116-1203) compiles unchanged.  The
 * graph is metadata only: AudioVAE::decode adds one node that
 * VoxCPMBackend::compute runs through libvxb.
 */
#ifndef VOXCPM_TENSOR_H
#define VOXCPM_TENSOR_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VOXCPM_API __attribute__((visibility("default")))
#else
#define VOXCPM_API
#endif

#define GGML_MAX_DIMS 4
#define GGML_MAX_NAME 64
#define GGML_DEFAULT_GRAPH_SIZE 2048

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_0 = 2,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_I32 = 26,
};

enum ggml_status {
    GGML_STATUS_ALLOC_FAILED = -2,
    GGML_STATUS_FAILED = -1,
    GGML_STATUS_SUCCESS = 0,
    GGML_STATUS_ABORTED = 1,
};

enum ggml_tensor_flag {
    GGML_TENSOR_FLAG_INPUT = 1,
    GGML_TENSOR_FLAG_OUTPUT = 2,
};

// What produces a tensor of the decode graph.
enum voxcpm_op {
    VOXCPM_OP_NONE = 0,          // leaf (input or weight)
    VOXCPM_OP_AUDIO_VAE_DECODE,  // src[0] = latent ne=[T, latent_dim(, B)]
    VOXCPM_OP_AUDIO_VAE_ENCODE,  // src[0] = waveform ne=[hop*T, 1, 1] -> latent ne=[T, latent_dim, 1]
};

struct ggml_context;

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[GGML_MAX_DIMS];  // elements per dimension, ne[0] fastest
    size_t nb[GGML_MAX_DIMS];   // strides in bytes
    int32_t flags;
    enum voxcpm_op op;
    struct ggml_tensor* src[2];
    void* data;    // host staging owned by the backend after alloc_graph
    void* buffer;  // non-null once allocated
    void* extra;   // the AudioVAE that produced a decode node
    char name[GGML_MAX_NAME];
};

struct ggml_cgraph {
    int size;
    int n_nodes;
    struct ggml_tensor** nodes;
};

#ifdef __cplusplus
extern "C" {
#endif

VOXCPM_API int64_t ggml_nelements(const struct ggml_tensor* t);
VOXCPM_API size_t ggml_nbytes(const struct ggml_tensor* t);
VOXCPM_API int ggml_n_dims(const struct ggml_tensor* t);
VOXCPM_API void ggml_set_input(struct ggml_tensor* t);
VOXCPM_API void ggml_set_output(struct ggml_tensor* t);
VOXCPM_API void ggml_set_name_str(struct ggml_tensor* t, const char* name);
VOXCPM_API void ggml_build_forward_expand(struct ggml_cgraph* g, struct ggml_tensor* t);

#ifdef __cplusplus
}
#endif

#endif  // VOXCPM_TENSOR_H
