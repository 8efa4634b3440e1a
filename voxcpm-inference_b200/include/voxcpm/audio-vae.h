/**
 * @file audio-vae.h
 * @brief AudioVAE (reference include/voxcpm/audio-vae.h:91-146).
 *
 * Same API as the reference for decoding (load_from_store,
 * ensure_derived_weights, decode, prepare_decode_inputs) and encoding
 * (encode, preprocess, last_input_tensor, last_preprocessed_audio).
 * decode() and encode() each add one node to the caller's graph;
 * VoxCPMBackend::compute executes it on the GPU.
 */
#ifndef VOXCPM_AUDIO_VAE_H
#define VOXCPM_AUDIO_VAE_H

#include <memory>
#include <string>
#include <vector>

#include "voxcpm/common.h"
#include "voxcpm/config.h"
#include "voxcpm/context.h"

namespace voxcpm {

class VoxCPMBackend;
class VoxCPMWeightStore;

class VOXCPM_API AudioVAE {
public:
    explicit AudioVAE(const AudioVAEConfig& config = AudioVAEConfig());
    ~AudioVAE();
    AudioVAE(const AudioVAE&) = delete;
    AudioVAE& operator=(const AudioVAE&) = delete;

    // false if the store owns no storage, a required KV key or tensor is
    // missing (reference src/audio-vae.cpp:421-463).
    bool load_from_store(const std::shared_ptr<VoxCPMWeightStore>& store);
    // Derived weights on the device; idempotent; must precede decode.
    bool ensure_derived_weights(VoxCPMBackend& backend);
    // z: ne=[T, latent_dim] (or [T, latent_dim, B]) F32 -> audio ne=[decode_hop*T(, B)].
    ggml_tensor* decode(VoxCPMContext& ctx, ggml_tensor* z);
    void prepare_decode_inputs(VoxCPMBackend& backend) const { VOXCPM_UNUSED(backend); }
    // Waveform at config().sample_rate (sample_rate < 0: that rate) ->
    // latent ne=[T, latent_dim], T = ceil(n / hop); the input tensor is
    // last_input_tensor(), to be filled with last_preprocessed_audio()
    // (the waveform zero-padded to a hop multiple) before compute
    // (reference src/audio-vae.cpp:652-664).
    ggml_tensor* encode(VoxCPMContext& ctx, std::vector<float>& audio_data, int sample_rate = -1);
    std::vector<float> preprocess(std::vector<float> audio_data, int sample_rate) const;
    ggml_tensor* last_input_tensor() const { return last_input_tensor_; }
    const std::vector<float>& last_preprocessed_audio() const { return last_preprocessed_audio_; }

    const AudioVAEConfig& config() const { return config_; }
    bool uses_shared_weights() const { return store_ != nullptr; }
    bool derived_ready() const { return derived_ready_; }

private:
    AudioVAEConfig config_;
    std::shared_ptr<VoxCPMWeightStore> store_;
    bool derived_ready_ = false;
    ggml_tensor* last_input_tensor_ = nullptr;
    std::vector<float> last_preprocessed_audio_;
};

}  // namespace voxcpm

#endif  // VOXCPM_AUDIO_VAE_H
