// Test infrastructure only: a thin extern "C" harness around the reference's
// own decoder and encoder code (nowang6/voxcpm-inference, compiled unmodified from its
// sources by oracle/Makefile.ref into oracle/_ref/liboracle_ref.so).
//
// It is the checker and the CPU baseline, never part of the product path.
// Two reference decode paths are exposed:
//   * "L2" = AudioVAE::decode() as HEAD ships it (src/audio-vae.cpp:666-700,
//     graph from decode_tensor_l2 :1584-1633). HEAD only accepts Q4_0 convT
//     weights (split_convt_weight_rows asserts it, :739), and re-quantises the
//     transposed-conv halves to Q8_0 (:766-819).
//   * "L1" = the reference's original graph functions, still compiled but no
//     longer called by decode(): causal_conv1d_dw (:495-510), causal_conv1d
//     (:476-493), decoder_block_forward (:572-591), snake_activation
//     (:278-289) and ggml_tanh, in the order decode used before L2. This is
//     the only reference path that runs F16 weights, and it keeps the exact
//     Q4_0 dequantisation for the transposed convs (:142-152).
// The L1 member functions are private in audio-vae.h, hence the access
// override around that one include.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#define private public
#include "voxcpm/audio-vae.h"
#undef private
#include "voxcpm/backend.h"
#include "voxcpm/context.h"
#include "voxcpm/weight-store.h"

#include "ggml.h"
#include "ggml-cpu.h"

using namespace voxcpm;

namespace {

struct RefModel {
    std::unique_ptr<VoxCPMBackend> backend;
    std::shared_ptr<VoxCPMWeightStore> store;
    std::unique_ptr<AudioVAE> vae;
    bool derived = false;
};

// Builds and runs one decode graph; mirrors the caller in
// vae_decode_mock.cpp:1116-1203 (graph ctx sizes, reserve/alloc/compute).
int run_decode(RefModel* m, const float* z, int T, float* out, bool l1, int stage = -1) {
    VoxCPMContext gc(ContextType::Graph, 32768, 262144);
    ggml_context* c = gc.raw_context();
    ggml_tensor* lat = gc.new_tensor_2d(GGML_TYPE_F32, T, m->vae->config().latent_dim);
    ggml_set_input(lat);
    ggml_tensor* y = nullptr;
    if (l1) {
        AudioVAE& vae = *m->vae;
        const AudioVAEWeights& W = vae.weights_;
        // Optional early exit after `stage` (0 = model.0, 1 = model.1, then per
        // block b: 2+4b transposed conv, 3+4b..5+4b residual units), returned
        // transposed to [t][c] (channels fastest).
        int cur = 0;
        auto at_stage = [&](ggml_tensor* t) -> bool {
            if (stage == cur++) {
                y = ggml_cont(c, ggml_transpose(c, ggml_reshape_2d(c, t, t->ne[0], t->ne[1])));
                return true;
            }
            return false;
        };
        ggml_tensor* x = ggml_reshape_3d(c, lat, T, vae.config_.latent_dim, 1);
        x = vae.causal_conv1d_dw(c, x, W.decoder_model_0_weight, W.decoder_model_0_bias, 1, 1, 3);
        if (!at_stage(x)) {
            x = vae.causal_conv1d(c, x, W.decoder_model_1_weight, W.decoder_model_1_bias, 1, 1, 1, 0);
        }
        if (y == nullptr && !at_stage(x)) {
            // decoder_block_forward (audio-vae.cpp:572-591) unrolled so that
            // every stage can be observed; same calls in the same order.
            for (size_t i = 0; i < W.decoder_blocks.size() && y == nullptr; ++i) {
                const DecoderBlockWeights& bw = W.decoder_blocks[i];
                const int s = vae.config_.decoder_rates[i];
                x = snake_activation(c, x, bw.snake_alpha);
                x = vae.causal_transpose_conv1d(c, x, bw.conv_weight, bw.conv_bias, s * 2, s,
                                                static_cast<int>(std::ceil(s / 2.0f)), s % 2);
                if (at_stage(x)) break;
                x = vae.residual_unit_forward(c, x, bw.res0, 1);
                if (at_stage(x)) break;
                x = vae.residual_unit_forward(c, x, bw.res1, 3);
                if (at_stage(x)) break;
                x = vae.residual_unit_forward(c, x, bw.res2, 9);
                if (at_stage(x)) break;
            }
            if (y == nullptr) {
                x = snake_activation(c, x, W.decoder_final_snake_alpha);
                x = vae.causal_conv1d(c, x, W.decoder_final_conv_weight, W.decoder_final_conv_bias,
                                      7, 1, 1, 3);
                y = ggml_tanh(c, x);
            }
        }
        ggml_set_output(y);
    } else {
        if (!m->derived) {
            if (!m->vae->ensure_derived_weights(*m->backend)) return -3;
            m->derived = true;
        }
        y = m->vae->decode(gc, lat);
    }
    ggml_cgraph* g = gc.new_graph();
    gc.build_forward(g, y);
    m->backend->reserve_compute_memory(g);
    m->backend->alloc_graph(g);
    const size_t zin = (size_t)T * m->vae->config().latent_dim;
    m->backend->tensor_set(lat, z, 0, zin * sizeof(float));
    m->vae->prepare_decode_inputs(*m->backend);
    if (m->backend->compute(g) != GGML_STATUS_SUCCESS) return -4;
    m->backend->tensor_get(y, out, 0, (size_t)ggml_nelements(y) * sizeof(float));
    return (int)ggml_nelements(y);
}

}  // namespace

extern "C" {

void* ref_open(const char* gguf_path, int n_threads) {
    auto* m = new RefModel();
    try {
        m->backend = std::make_unique<VoxCPMBackend>(BackendType::CPU, n_threads);
        m->store = std::make_shared<VoxCPMWeightStore>();
        if (!m->store->load_from_file(gguf_path, *m->backend)) { delete m; return nullptr; }
        m->vae = std::make_unique<AudioVAE>();
        if (!m->vae->load_from_store(m->store)) { delete m; return nullptr; }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ref_open: %s\n", e.what());
        delete m;
        return nullptr;
    }
    return m;
}

void ref_close(void* h) { delete static_cast<RefModel*>(h); }

// out must hold 640*T floats (product of decoder rates times T).
int ref_decode_l1(void* h, const float* z, int T, float* out) {
    return run_decode(static_cast<RefModel*>(h), z, T, out, true);
}

// Activation after one L1 stage, [t][c]; returns its element count.
int ref_decode_l1_stage(void* h, const float* z, int T, int stage, float* out) {
    return run_decode(static_cast<RefModel*>(h), z, T, out, true, stage);
}

int ref_decode_l2(void* h, const float* z, int T, float* out) {
    return run_decode(static_cast<RefModel*>(h), z, T, out, false);
}

// The reference's own encoder, AudioVAE::encode (src/audio-vae.cpp:652-664,
// graph from encode_tensor :640-650), on one waveform of n samples (padded
// to a hop multiple by its preprocess, :465-474); the latent [64][T] (t
// fastest) into out.  Returns its element count, or < 0 on failure.
long long ref_encode(void* h, const float* audio, long long n, float* out, long long cap) {
    RefModel* m = static_cast<RefModel*>(h);
    VoxCPMContext gc(ContextType::Graph, 32768, 262144);
    std::vector<float> a(audio, audio + n);
    ggml_tensor* y = m->vae->encode(gc, a, -1);
    ggml_cgraph* g = gc.new_graph();
    gc.build_forward(g, y);
    m->backend->reserve_compute_memory(g);
    m->backend->alloc_graph(g);
    const std::vector<float>& pa = m->vae->last_preprocessed_audio();
    m->backend->tensor_set(m->vae->last_input_tensor(), pa.data(), 0, pa.size() * sizeof(float));
    if (m->backend->compute(g) != GGML_STATUS_SUCCESS) return -4;
    const long long ne = ggml_nelements(y);
    if (ne > cap) return -5;
    m->backend->tensor_get(y, out, 0, (size_t)ne * sizeof(float));
    return ne;
}

// The same encoder built from the reference's own layer functions with an
// early exit: stage 0 = head conv, then per block b: 1+4b..3+4b the residual
// units, 4+4b the Snake + strided conv (encode_tensor :640-650,
// encoder_block_forward :553-570).  The activation is returned as [t][c].
long long ref_encode_stage(void* h, const float* audio, long long n, int stage, float* out, long long cap) {
    RefModel* m = static_cast<RefModel*>(h);
    AudioVAE& vae = *m->vae;
    const AudioVAEWeights& W = vae.weights_;
    VoxCPMContext gc(ContextType::Graph, 32768, 262144);
    ggml_context* c = gc.raw_context();
    std::vector<float> a = vae.preprocess(std::vector<float>(audio, audio + n), -1);
    ggml_tensor* in = gc.new_tensor_3d(GGML_TYPE_F32, (int64_t)a.size(), 1, 1);
    ggml_set_input(in);
    int cur = 0;
    ggml_tensor* y = nullptr;
    auto at_stage = [&](ggml_tensor* t) {
        if (stage == cur++) y = ggml_cont(c, ggml_transpose(c, ggml_reshape_2d(c, t, t->ne[0], t->ne[1])));
        return y != nullptr;
    };
    ggml_tensor* x = vae.causal_conv1d(c, in, W.encoder_block_0_weight, W.encoder_block_0_bias, 7, 1, 1, 3);
    if (!at_stage(x)) {
        for (int i = 0; i < vae.config_.num_encoder_blocks(); ++i) {
            const EncoderBlockWeights& bw = W.encoder_blocks[(size_t)i];
            const int s = vae.config_.encoder_rates[(size_t)i];
            x = vae.residual_unit_forward(c, x, bw.res0, 1);
            if (at_stage(x)) break;
            x = vae.residual_unit_forward(c, x, bw.res1, 3);
            if (at_stage(x)) break;
            x = vae.residual_unit_forward(c, x, bw.res2, 9);
            if (at_stage(x)) break;
            x = snake_activation(c, x, bw.snake_alpha);
            x = vae.causal_conv1d(c, x, bw.conv_weight, bw.conv_bias, s * 2, s, 1, (int)std::ceil(s / 2.0f));
            if (at_stage(x)) break;
        }
    }
    if (!y) return -6;
    ggml_set_output(y);
    ggml_cgraph* g = gc.new_graph();
    gc.build_forward(g, y);
    m->backend->reserve_compute_memory(g);
    m->backend->alloc_graph(g);
    m->backend->tensor_set(in, a.data(), 0, a.size() * sizeof(float));
    if (m->backend->compute(g) != GGML_STATUS_SUCCESS) return -4;
    const long long ne = ggml_nelements(y);
    if (ne > cap) return -5;
    m->backend->tensor_get(y, out, 0, (size_t)ne * sizeof(float));
    return ne;
}

// ggml's own Q4_0 row conversion (ggml-quants.c:459-477 dequantize_row_q4_0,
// :113-145 quantize_row_q4_0_ref), reached through the public type traits.
void ref_dequant_q4_0(const void* blocks, long long n, float* out) {
    ggml_get_type_traits(GGML_TYPE_Q4_0)->to_float(blocks, out, n);
}

void ref_quantize_q4_0(const float* x, long long n, void* blocks) {
    ggml_get_type_traits(GGML_TYPE_Q4_0)->from_float_ref(x, blocks, n);
}

void ref_quantize_q8_0(const float* x, long long n, void* blocks) {
    ggml_get_type_traits(GGML_TYPE_Q8_0)->from_float_ref(x, blocks, n);
}

void ref_dequant_q8_0(const void* blocks, long long n, float* out) {
    ggml_get_type_traits(GGML_TYPE_Q8_0)->to_float(blocks, out, n);
}

unsigned short ref_fp32_to_fp16(float x) { return ggml_fp32_to_fp16(x); }
float ref_fp16_to_fp32(unsigned short h) { return ggml_fp16_to_fp32(h); }

// HEAD's fused snake callback (audio-vae.cpp:1443-1479, polynomial sin
// :1216-1247) applied to x laid out [T][C] (channels fastest).
void ref_snake_fused(const float* x, const float* alpha, const float* inv, int C, int T, float* y) {
    ggml_init_params p = {ggml_tensor_overhead() * 4 + 1024, nullptr, true};
    ggml_context* c = ggml_init(p);
    ggml_tensor* tx = ggml_new_tensor_3d(c, GGML_TYPE_F32, C, T, 1);
    ggml_tensor* ty = ggml_new_tensor_3d(c, GGML_TYPE_F32, C, T, 1);
    tx->data = const_cast<float*>(x);
    ty->data = y;
    AudioVAESnakeOpData op;
    op.alpha = alpha;
    op.inv = inv;
    snake_fused_l2_custom(ty, tx, 0, 1, &op);
    ggml_free(c);
}

// ggml mul_mat as the pointwise convs use it (pointwise_l2, audio-vae.cpp:1421-1435):
// y[n][m] = sum_k W[m][k] * x[n][k]; W is a [K, M] tensor of type wtype
// (0 = F32, 1 = F16, 2 = Q4_0, 8 = Q8_0) whose rows are raw bytes.
int ref_mul_mat(const void* w, int wtype, int K, int M, const float* x, int N, float* y, int n_threads) {
    ggml_init_params p = {64 * 1024 * 1024, nullptr, false};
    ggml_context* c = ggml_init(p);
    ggml_tensor* tw = ggml_new_tensor_2d(c, (ggml_type)wtype, K, M);
    std::memcpy(tw->data, w, ggml_nbytes(tw));
    ggml_tensor* tx = ggml_new_tensor_2d(c, GGML_TYPE_F32, K, N);
    std::memcpy(tx->data, x, ggml_nbytes(tx));
    ggml_tensor* ty = ggml_mul_mat(c, tw, tx);
    ggml_cgraph* g = ggml_new_graph(c);
    ggml_build_forward_expand(g, ty);
    const int st = ggml_graph_compute_with_ctx(c, g, n_threads);
    std::memcpy(y, ty->data, ggml_nbytes(ty));
    ggml_free(c);
    return st;
}

}  // extern "C"
