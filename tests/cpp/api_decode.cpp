// A caller of the voxcpm C++ decode API written exactly like the
// reference's own caller (vae_decode_mock.cpp decode_waveform: backend,
// store, load_from_store, ensure_derived_weights, then per step a graph
// context, decode, reserve/alloc, tensor_set, compute, tensor_get).
//
//   api_decode MODEL.gguf Z.f32 T STEPS OUT.f32
// Z.f32: STEPS x [64][T] float32; OUT.f32: STEPS x [hop*T] float32.
// Exit codes: 0 ok, 2 store load, 3 load_from_store, 4 derived weights,
// 5 compute, 6 I/O, 7 voxcpm::Error (message on stderr).
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <vector>

#include "voxcpm/audio-vae.h"
#include "voxcpm/backend.h"
#include "voxcpm/context.h"
#include "voxcpm/weight-store.h"

using namespace voxcpm;

int main(int argc, char** argv) {
    if (argc < 6) {
        std::fprintf(stderr, "usage: %s MODEL.gguf Z.f32 T STEPS OUT.f32\n", argv[0]);
        return 1;
    }
    const int T = std::atoi(argv[3]), steps = std::atoi(argv[4]);
    try {
        VoxCPMBackend backend(BackendType::CUDA, 4);
        auto store = std::make_shared<VoxCPMWeightStore>();
        if (!store->load_from_file(argv[1], backend)) return 2;
        AudioVAE vae;
        if (!vae.load_from_store(store)) return 3;
        if (!vae.ensure_derived_weights(backend)) return 4;
        const int L = vae.config().latent_dim;
        std::vector<float> z(static_cast<size_t>(steps) * L * T);
        FILE* f = std::fopen(argv[2], "rb");
        if (!f || std::fread(z.data(), sizeof(float), z.size(), f) != z.size()) return 6;
        std::fclose(f);
        FILE* o = std::fopen(argv[5], "wb");
        if (!o) return 6;
        for (int s = 0; s < steps; ++s) {
            VoxCPMContext graph_ctx(ContextType::Graph, 32768, 262144);
            ggml_tensor* latent = graph_ctx.new_tensor_2d(GGML_TYPE_F32, T, L);
            ggml_set_input(latent);
            ggml_tensor* audio = vae.decode(graph_ctx, latent);
            ggml_cgraph* graph = graph_ctx.new_graph();
            graph_ctx.build_forward(graph, audio);
            backend.reserve_compute_memory(graph, "api_decode");
            backend.alloc_graph(graph, "api_decode");
            backend.tensor_set(latent, z.data() + static_cast<size_t>(s) * L * T, 0,
                               static_cast<size_t>(L) * T * sizeof(float));
            vae.prepare_decode_inputs(backend);
            if (backend.compute(graph) != GGML_STATUS_SUCCESS) return 5;
            std::vector<float> wave(static_cast<size_t>(ggml_nelements(audio)));
            backend.tensor_get(audio, wave.data(), 0, wave.size() * sizeof(float));
            std::fwrite(wave.data(), sizeof(float), wave.size(), o);
        }
        std::fclose(o);
    } catch (const Error& e) {
        std::fprintf(stderr, "voxcpm::Error(%d): %s\n", static_cast<int>(e.code()), e.what());
        return 7;
    }
    return 0;
}
