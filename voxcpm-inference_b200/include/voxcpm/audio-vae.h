/**
 * @file audio-vae.h
 * @brief AudioVAE decoder (reference include/voxcpm/audio-vae.h:91-140).
 *
 * Same decode-path API: load_from_store, ensure_derived_weights, decode,
 * prepare_decode_inputs.  decode() adds one node to the caller's graph;
 * VoxCPMBackend::compute executes it on the GPU.  The encoder is not part of
 * this build (its tensors are still required by load_from_store, as in the
 * reference, which checks their presence).
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

    const AudioVAEConfig& config() const { return config_; }
    bool uses_shared_weights() const { return store_ != nullptr; }
    bool derived_ready() const { return derived_ready_; }

private:
    AudioVAEConfig config_;
    std::shared_ptr<VoxCPMWeightStore> store_;
    bool derived_ready_ = false;
};

}  // namespace voxcpm

#endif  // VOXCPM_AUDIO_VAE_H
