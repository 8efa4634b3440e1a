/**
 * @file config.h
 * @brief AudioVAE configuration, as read from the GGUF KV
 *        voxcpm_audio_vae_config_* (reference include/voxcpm/config.h:34-133).
 */
#ifndef VOXCPM_CONFIG_H
#define VOXCPM_CONFIG_H

#include <string>
#include <vector>

namespace voxcpm {

struct AudioVAEConfig {
    int encoder_dim = 128;
    int latent_dim = 64;
    int decoder_dim = 1536;
    int sample_rate = 16000;
    int out_sample_rate = 0;
    std::vector<int> sr_bin_boundaries = {20000, 30000, 40000};
    std::vector<int> encoder_rates = {2, 5, 8, 8};
    std::vector<int> decoder_rates = {8, 8, 5, 2};
    bool depthwise = true;
    bool use_noise_block = false;
    std::string cond_type = "scale_bias";
    int cond_dim = 128;
    bool cond_out_layer = false;

    int hop_length() const {
        int h = 1;
        for (int r : encoder_rates) h *= r;
        return h;
    }
    int decode_hop_length() const {
        int h = 1;
        for (int r : decoder_rates) h *= r;
        return h;
    }
    int num_encoder_blocks() const { return static_cast<int>(encoder_rates.size()); }
    int num_decoder_blocks() const { return static_cast<int>(decoder_rates.size()); }
    int output_sample_rate() const { return out_sample_rate > 0 ? out_sample_rate : sample_rate; }
    std::vector<int> decoder_channels() const {
        std::vector<int> ch{decoder_dim};
        int c = decoder_dim;
        for (size_t i = 0; i < decoder_rates.size(); ++i) ch.push_back(c /= 2);
        return ch;
    }
};

}  // namespace voxcpm

#endif  // VOXCPM_CONFIG_H
