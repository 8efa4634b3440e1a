// A caller of the voxcpm C++ encode API, in the reference's pattern
// (AudioVAE::encode adds the graph; the caller reserves/allocates, fills
// last_input_tensor() with last_preprocessed_audio(), computes and reads the
// latent back; reference src/audio-vae.cpp:652-664, include/voxcpm/audio-vae.h:103-146).
//
//   api_encode MODEL.gguf AUDIO.f32 N STEPS OUT.f32
// AUDIO.f32: STEPS x [N] float32 waveforms at 16 kHz; OUT.f32: STEPS x [64][T]
// float32 latents, T = ceil(N / hop).
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
        std::fprintf(stderr, "usage: %s MODEL.gguf AUDIO.f32 N STEPS OUT.f32\n", argv[0]);
        return 1;
    }
    const long N = std::atol(argv[3]);
    const int steps = std::atoi(argv[4]);
    try {
        VoxCPMBackend backend(BackendType::CUDA, 4);
        auto store = std::make_shared<VoxCPMWeightStore>();
        if (!store->load_from_file(argv[1], backend)) return 2;
        AudioVAE vae;
        if (!vae.load_from_store(store)) return 3;
        if (!vae.ensure_derived_weights(backend)) return 4;
        std::vector<float> all(static_cast<size_t>(steps) * N);
        FILE* f = std::fopen(argv[2], "rb");
        if (!f || std::fread(all.data(), sizeof(float), all.size(), f) != all.size()) return 6;
        std::fclose(f);
        FILE* o = std::fopen(argv[5], "wb");
        if (!o) return 6;
        for (int s = 0; s < steps; ++s) {
            VoxCPMContext graph_ctx(ContextType::Graph, 32768, 262144);
            std::vector<float> audio(all.begin() + static_cast<long>(s) * N, all.begin() + static_cast<long>(s + 1) * N);
            ggml_tensor* latent = vae.encode(graph_ctx, audio, -1);
            ggml_cgraph* graph = graph_ctx.new_graph();
            graph_ctx.build_forward(graph, latent);
            backend.reserve_compute_memory(graph, "api_encode");
            backend.alloc_graph(graph, "api_encode");
            const std::vector<float>& pre = vae.last_preprocessed_audio();
            backend.tensor_set(vae.last_input_tensor(), pre.data(), 0, pre.size() * sizeof(float));
            if (backend.compute(graph) != GGML_STATUS_SUCCESS) return 5;
            std::vector<float> z(static_cast<size_t>(ggml_nelements(latent)));
            backend.tensor_get(latent, z.data(), 0, z.size() * sizeof(float));
            std::fwrite(z.data(), sizeof(float), z.size(), o);
        }
        std::fclose(o);
    } catch (const Error& e) {
        std::fprintf(stderr, "voxcpm::Error(%d): %s\n", static_cast<int>(e.code()), e.what());
        return 7;
    }
    return 0;
}
