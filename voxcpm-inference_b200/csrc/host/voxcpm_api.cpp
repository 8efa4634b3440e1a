// The voxcpm C++ API (VoxCPMBackend, VoxCPMWeightStore, AudioVAE,
// VoxCPMContext) over the libvxb C ABI.  Same class and method names,
// argument meaning and error behaviour as the reference
// (include/voxcpm/{backend,weight-store,audio-vae,context}.h), so that a
// caller written against the reference's decode path runs on the B200.
#include <cstring>
#include <map>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "gguf_reader.h"
#include "voxcpm/audio-vae.h"
#include "voxcpm/backend.h"
#include "voxcpm/context.h"
#include "voxcpm/weight-store.h"
#include "vxb.h"

// ------------------------------------------------------ tensor handles ----

struct ggml_context {
    std::vector<std::unique_ptr<ggml_tensor>> tensors;
    std::vector<std::unique_ptr<ggml_cgraph>> graphs;
    std::vector<std::unique_ptr<std::vector<ggml_tensor*>>> node_arrays;
};

namespace {

size_t type_size(ggml_type t) {
    switch (t) {
        case GGML_TYPE_F32: return 4;
        case GGML_TYPE_F16: return 2;
        case GGML_TYPE_I32: return 4;
        default: return 0;
    }
}

void set_contiguous_strides(ggml_tensor* t) {
    const size_t es = type_size(t->type);
    if (t->type == GGML_TYPE_Q4_0 || t->type == GGML_TYPE_Q8_0) {
        const size_t blk = t->type == GGML_TYPE_Q4_0 ? 18 : 34;
        t->nb[0] = blk;  // per 32-element block
        t->nb[1] = static_cast<size_t>(t->ne[0] / 32) * blk;
    } else {
        t->nb[0] = es;
        t->nb[1] = es * static_cast<size_t>(t->ne[0]);
    }
    for (int d = 2; d < GGML_MAX_DIMS; ++d) t->nb[d] = t->nb[d - 1] * static_cast<size_t>(t->ne[d - 1]);
}

}  // namespace

extern "C" {

int64_t ggml_nelements(const ggml_tensor* t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

size_t ggml_nbytes(const ggml_tensor* t) {
    if (t->type == GGML_TYPE_Q4_0) return static_cast<size_t>(ggml_nelements(t) / 32) * 18;
    if (t->type == GGML_TYPE_Q8_0) return static_cast<size_t>(ggml_nelements(t) / 32) * 34;
    return static_cast<size_t>(ggml_nelements(t)) * type_size(t->type);
}

int ggml_n_dims(const ggml_tensor* t) {
    for (int d = GGML_MAX_DIMS - 1; d >= 1; --d)
        if (t->ne[d] > 1) return d + 1;
    return 1;
}

void ggml_set_input(ggml_tensor* t) { t->flags |= GGML_TENSOR_FLAG_INPUT; }
void ggml_set_output(ggml_tensor* t) { t->flags |= GGML_TENSOR_FLAG_OUTPUT; }

void ggml_set_name_str(ggml_tensor* t, const char* name) {
    std::snprintf(t->name, sizeof(t->name), "%s", name ? name : "");
}

void ggml_build_forward_expand(ggml_cgraph* g, ggml_tensor* t) {
    if (!g || !t) return;
    for (int i = 0; i < 2; ++i)
        if (t->src[i]) ggml_build_forward_expand(g, t->src[i]);
    for (int i = 0; i < g->n_nodes; ++i)
        if (g->nodes[i] == t) return;
    VOXCPM_ASSERT(g->n_nodes < g->size);
    g->nodes[g->n_nodes++] = t;
}

}  // extern "C"

namespace voxcpm {

// ---------------------------------------------------------- VoxCPMContext --

VoxCPMContext::VoxCPMContext(ContextType type, int n_tensors, int max_nodes, size_t extra_mem_size)
    : type_(type), ctx_(new ggml_context()), mem_size_(0), max_nodes_(max_nodes) {
    mem_size_ = static_cast<size_t>(n_tensors) * sizeof(ggml_tensor) + extra_mem_size;
}

VoxCPMContext::~VoxCPMContext() { delete ctx_; }

VoxCPMContext::VoxCPMContext(VoxCPMContext&& o) noexcept
    : type_(o.type_), ctx_(o.ctx_), mem_size_(o.mem_size_), max_nodes_(o.max_nodes_) {
    o.ctx_ = nullptr;
}

VoxCPMContext& VoxCPMContext::operator=(VoxCPMContext&& o) noexcept {
    if (this != &o) {
        delete ctx_;
        type_ = o.type_;
        ctx_ = o.ctx_;
        mem_size_ = o.mem_size_;
        max_nodes_ = o.max_nodes_;
        o.ctx_ = nullptr;
    }
    return *this;
}

ggml_tensor* VoxCPMContext::new_node(ggml_type type, int n_dims, const int64_t* ne) {
    auto t = std::make_unique<ggml_tensor>();
    std::memset(t.get(), 0, sizeof(ggml_tensor));
    t->type = type;
    for (int d = 0; d < GGML_MAX_DIMS; ++d) t->ne[d] = d < n_dims ? ne[d] : 1;
    set_contiguous_strides(t.get());
    ctx_->tensors.push_back(std::move(t));
    return ctx_->tensors.back().get();
}

ggml_tensor* VoxCPMContext::new_tensor_2d(ggml_type type, int64_t ne0, int64_t ne1) {
    const int64_t ne[2] = {ne0, ne1};
    return new_node(type, 2, ne);
}

ggml_tensor* VoxCPMContext::new_tensor_3d(ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2) {
    const int64_t ne[3] = {ne0, ne1, ne2};
    return new_node(type, 3, ne);
}

ggml_cgraph* VoxCPMContext::new_graph() { return new_graph(max_nodes_ > 0 ? max_nodes_ : GGML_DEFAULT_GRAPH_SIZE); }

ggml_cgraph* VoxCPMContext::new_graph(size_t size) {
    auto arr = std::make_unique<std::vector<ggml_tensor*>>(size, nullptr);
    auto g = std::make_unique<ggml_cgraph>();
    g->size = static_cast<int>(size);
    g->n_nodes = 0;
    g->nodes = arr->data();
    ctx_->node_arrays.push_back(std::move(arr));
    ctx_->graphs.push_back(std::move(g));
    return ctx_->graphs.back().get();
}

void VoxCPMContext::build_forward(ggml_cgraph* graph, ggml_tensor* output) { ggml_build_forward_expand(graph, output); }

// ---------------------------------------------------------- VoxCPMBackend --

VoxCPMBackend::VoxCPMBackend(BackendType type, int n_threads, int device) : type_(type), n_threads_(n_threads) {
    if (type != BackendType::CUDA)
        throw Error(ErrorCode::NotImplemented, "this build runs the decoder on BackendType::CUDA only");
    if (vxb_open(device, &ctx_) != VXB_OK)
        throw Error(ErrorCode::BackendError, std::string("Failed to initialize CUDA backend: ") + vxb_last_error());
    description_ = "B200 (sm_100a) device " + std::to_string(device);
}

VoxCPMBackend::~VoxCPMBackend() {
    if (ctx_) vxb_close(ctx_);
}

VoxCPMBackend::VoxCPMBackend(VoxCPMBackend&& o) noexcept
    : type_(o.type_), n_threads_(o.n_threads_), ctx_(o.ctx_), description_(std::move(o.description_)),
      staging_(std::move(o.staging_)), staging_bytes_(o.staging_bytes_), plan_b_(o.plan_b_), plan_t_(o.plan_t_),
      enc_plan_t_(o.enc_plan_t_) {
    o.ctx_ = nullptr;
}

VoxCPMBackend& VoxCPMBackend::operator=(VoxCPMBackend&& o) noexcept {
    if (this != &o) {
        if (ctx_) vxb_close(ctx_);
        type_ = o.type_;
        n_threads_ = o.n_threads_;
        ctx_ = o.ctx_;
        description_ = std::move(o.description_);
        staging_ = std::move(o.staging_);
        staging_bytes_ = o.staging_bytes_;
        plan_b_ = o.plan_b_;
        plan_t_ = o.plan_t_;
        enc_plan_t_ = o.enc_plan_t_;
        o.ctx_ = nullptr;
    }
    return *this;
}

void VoxCPMBackend::reserve_compute_memory(ggml_cgraph* graph, const char* stage) {
    VOXCPM_UNUSED(stage);
    for (int i = 0; i < graph->n_nodes; ++i) {
        ggml_tensor* t = graph->nodes[i];
        if (t->op == VOXCPM_OP_AUDIO_VAE_ENCODE) {
            const int T = static_cast<int>(t->ne[0]);
            if (T == enc_plan_t_) continue;
            if (vxb_build_encode_plan(ctx_, 1, T) != VXB_OK)
                throw Error(ErrorCode::BackendError, std::string("reserve_compute_memory: ") + vxb_last_error());
            enc_plan_t_ = T;
            continue;
        }
        if (t->op != VOXCPM_OP_AUDIO_VAE_DECODE) continue;
        const ggml_tensor* z = t->src[0];
        const int T = static_cast<int>(z->ne[0]);
        const int B = static_cast<int>(z->ne[2]);
        if (B == plan_b_ && T == plan_t_) continue;
        if (vxb_build_plan(ctx_, B, T, 1) != VXB_OK)
            throw Error(ErrorCode::BackendError, std::string("reserve_compute_memory: ") + vxb_last_error());
        plan_b_ = B;
        plan_t_ = T;
    }
}

void VoxCPMBackend::alloc_graph(ggml_cgraph* graph, const char* stage) {
    VOXCPM_UNUSED(stage);
    for (int i = 0; i < graph->n_nodes; ++i) {
        ggml_tensor* t = graph->nodes[i];
        const bool io = t->op == VOXCPM_OP_AUDIO_VAE_DECODE || t->op == VOXCPM_OP_AUDIO_VAE_ENCODE ||
                        (t->flags & GGML_TENSOR_FLAG_INPUT);
        if (!io || t->buffer) continue;
        auto buf = std::make_unique<std::vector<uint8_t>>(ggml_nbytes(t));
        t->data = buf->data();
        t->buffer = buf.get();
        staging_bytes_ += buf->size();
        staging_.push_back(std::move(buf));
    }
}

ggml_status VoxCPMBackend::compute(ggml_cgraph* graph) {
    for (int i = 0; i < graph->n_nodes; ++i) {
        ggml_tensor* t = graph->nodes[i];
        if (t->op == VOXCPM_OP_AUDIO_VAE_ENCODE) {
            const ggml_tensor* a = t->src[0];
            if (!t->data || !a->data) return GGML_STATUS_ALLOC_FAILED;
            if (static_cast<int>(t->ne[0]) != enc_plan_t_) reserve_compute_memory(graph);
            if (vxb_encode(ctx_, static_cast<const float*>(a->data), static_cast<float*>(t->data)) != VXB_OK) {
                std::fprintf(stderr, "[voxcpm] encode failed: %s\n", vxb_last_error());
                return GGML_STATUS_FAILED;
            }
            continue;
        }
        if (t->op != VOXCPM_OP_AUDIO_VAE_DECODE) continue;
        const ggml_tensor* z = t->src[0];
        if (!t->data || !z->data) return GGML_STATUS_ALLOC_FAILED;
        if (static_cast<int>(z->ne[2]) != plan_b_ || static_cast<int>(z->ne[0]) != plan_t_)
            reserve_compute_memory(graph);
        if (vxb_decode(ctx_, static_cast<const float*>(z->data), static_cast<float*>(t->data)) != VXB_OK) {
            std::fprintf(stderr, "[voxcpm] decode failed: %s\n", vxb_last_error());
            return GGML_STATUS_FAILED;
        }
    }
    return GGML_STATUS_SUCCESS;
}

void VoxCPMBackend::tensor_set(ggml_tensor* tensor, const void* data, size_t offset, size_t size) {
    if (!tensor) throw Error(ErrorCode::BackendError, "tensor_set received a null tensor");
    if (!data && size > 0) throw Error(ErrorCode::BackendError, "tensor_set received a null data pointer");
    const size_t bytes = ggml_nbytes(tensor);
    if (offset > bytes || size > bytes - offset) {
        std::ostringstream oss;
        oss << "tensor_set overflow for tensor '" << tensor->name << "': tensor_bytes=" << bytes
            << ", offset=" << offset << ", size=" << size;
        throw Error(ErrorCode::BackendError, oss.str());
    }
    if (!tensor->buffer || !tensor->data) {
        std::ostringstream oss;
        oss << "tensor_set target is not allocated for tensor '" << tensor->name << "'";
        throw Error(ErrorCode::BackendError, oss.str());
    }
    std::memcpy(static_cast<uint8_t*>(tensor->data) + offset, data, size);
}

void VoxCPMBackend::tensor_get(const ggml_tensor* tensor, void* data, size_t offset, size_t size) {
    if (!tensor || !tensor->data) throw Error(ErrorCode::BackendError, "tensor_get on an unallocated tensor");
    const size_t bytes = ggml_nbytes(tensor);
    if (offset > bytes || size > bytes - offset) throw Error(ErrorCode::BackendError, "tensor_get overflow");
    std::memcpy(data, static_cast<const uint8_t*>(tensor->data) + offset, size);
}

// ------------------------------------------------------ VoxCPMWeightStore --

struct VoxCPMWeightStore::Impl {
    vxb::GgufFile file;
};

VoxCPMWeightStore::~VoxCPMWeightStore() = default;

bool VoxCPMWeightStore::load_from_file(const std::string& gguf_path, VoxCPMBackend& backend, WeightGroupFn group_fn) {
    VOXCPM_UNUSED(group_fn);
    auto impl = std::make_shared<Impl>();
    std::string err;
    if (!impl->file.open(gguf_path, &err)) {
        std::fprintf(stderr, "[weight-store] %s\n", err.c_str());
        return false;
    }
    if (vxb_load_gguf(backend.vxb(), gguf_path.c_str()) != VXB_OK) {
        std::fprintf(stderr, "[weight-store] upload failed: %s\n", vxb_last_error());
        return false;
    }
    tensors_.clear();
    for (const auto& ti : impl->file.tensors) {
        auto t = std::make_unique<ggml_tensor>();
        std::memset(t.get(), 0, sizeof(ggml_tensor));
        t->type = static_cast<ggml_type>(ti.type);
        for (int d = 0; d < GGML_MAX_DIMS; ++d) t->ne[d] = ti.ne[d];
        set_contiguous_strides(t.get());
        std::snprintf(t->name, sizeof(t->name), "%s", ti.name.c_str());
        t->buffer = backend.vxb();  // resident on the backend's device
        tensors_[ti.name] = std::move(t);
    }
    kv_ = impl;
    backend_ = &backend;
    path_ = gguf_path;
    return true;
}

ggml_tensor* VoxCPMWeightStore::get_tensor(const char* name) const {
    auto it = tensors_.find(name ? name : "");
    return it == tensors_.end() ? nullptr : it->second.get();
}

bool VoxCPMWeightStore::get_u32(const char* key, uint32_t& value) const {
    const vxb::GgufValue* v = kv_ ? kv_->file.kv(key) : nullptr;
    if (!v || (v->type != 4 && v->type != 5)) return false;
    value = static_cast<uint32_t>(v->i);
    return true;
}

bool VoxCPMWeightStore::get_bool(const char* key, bool& value) const {
    const vxb::GgufValue* v = kv_ ? kv_->file.kv(key) : nullptr;
    if (!v || v->type != 7) return false;
    value = v->b;
    return true;
}

bool VoxCPMWeightStore::get_string(const char* key, std::string& value) const {
    const vxb::GgufValue* v = kv_ ? kv_->file.kv(key) : nullptr;
    if (!v || v->type != 8) return false;
    value = v->s;
    return true;
}

bool VoxCPMWeightStore::get_i32_array(const char* key, std::vector<int>& values) const {
    const vxb::GgufValue* v = kv_ ? kv_->file.kv(key) : nullptr;
    if (!v || v->type != 9) return false;
    values.assign(v->arr_i.begin(), v->arr_i.end());
    return true;
}

// --------------------------------------------------------------- AudioVAE --

AudioVAE::AudioVAE(const AudioVAEConfig& config) : config_(config) {}
AudioVAE::~AudioVAE() = default;

bool AudioVAE::load_from_store(const std::shared_ptr<VoxCPMWeightStore>& store) {
    if (!store || !store->owns_storage()) return false;
    store_ = store;
    uint32_t u = 0;
    const bool has_enc = store->get_u32("voxcpm_audio_vae_config_encoder_dim", u);
    if (has_enc) config_.encoder_dim = static_cast<int>(u);
    const bool has_dec = store->get_u32("voxcpm_audio_vae_config_decoder_dim", u);
    if (has_dec) config_.decoder_dim = static_cast<int>(u);
    const bool has_lat = store->get_u32("voxcpm_audio_vae_config_latent_dim", u);
    if (has_lat) config_.latent_dim = static_cast<int>(u);
    const bool has_sr = store->get_u32("voxcpm_audio_vae_config_sample_rate", u);
    if (has_sr) config_.sample_rate = static_cast<int>(u);
    if (store->get_u32("voxcpm_audio_vae_config_out_sample_rate", u)) config_.out_sample_rate = static_cast<int>(u);
    store->get_bool("voxcpm_audio_vae_config_depthwise", config_.depthwise);
    store->get_bool("voxcpm_audio_vae_config_use_noise_block", config_.use_noise_block);
    const bool has_er = store->get_i32_array("voxcpm_audio_vae_config_encoder_rates", config_.encoder_rates);
    const bool has_dr = store->get_i32_array("voxcpm_audio_vae_config_decoder_rates", config_.decoder_rates);
    if (!has_enc || !has_dec || !has_lat || !has_sr || !has_er || !has_dr) return false;
    if (config_.encoder_rates.empty() || config_.decoder_rates.empty()) return false;

    // Required tensors, by the names load_decoder_weights / load_encoder_weights bind.
    std::vector<std::string> names = {"audio_vae.encoder.block.0.weight", "audio_vae.encoder.block.0.bias",
                                      "audio_vae.encoder.fc_mu.weight", "audio_vae.encoder.fc_mu.bias"};
    for (int b = 1; b <= config_.num_encoder_blocks(); ++b) {
        const std::string bp = "audio_vae.encoder.block." + std::to_string(b) + ".block.";
        for (int r = 0; r < 3; ++r)
            for (const char* n : {"0.alpha", "1.weight", "1.bias", "2.alpha", "3.weight", "3.bias"})
                names.push_back(bp + std::to_string(r) + ".block." + n);
        for (const char* n : {"3.alpha", "4.weight", "4.bias"}) names.push_back(bp + n);
    }
    const std::string p = "audio_vae.decoder.model.";
    for (const char* n : {"0.weight", "0.bias", "1.weight", "1.bias"}) names.push_back(p + n);
    const int nb = config_.num_decoder_blocks();
    names.push_back(p + std::to_string(nb + 2) + ".alpha");
    names.push_back(p + std::to_string(nb + 3) + ".weight");
    names.push_back(p + std::to_string(nb + 3) + ".bias");
    for (int i = 0; i < nb; ++i) {
        const std::string bp = p + std::to_string(i + 2) + ".block.";
        for (const char* n : {"0.alpha", "1.weight", "1.bias"}) names.push_back(bp + n);
        for (int r = 0; r < 3; ++r)
            for (const char* n : {"0.alpha", "1.weight", "1.bias", "2.alpha", "3.weight", "3.bias"})
                names.push_back(bp + std::to_string(r + 2) + ".block." + n);
    }
    for (const auto& n : names)
        if (!store->get_tensor(n.c_str())) return false;
    return true;
}

bool AudioVAE::ensure_derived_weights(VoxCPMBackend& backend) {
    if (derived_ready_) return true;
    if (vxb_prepare(backend.vxb()) != VXB_OK) {
        std::fprintf(stderr, "[audio-vae] derived weights: %s\n", vxb_last_error());
        return false;
    }
    derived_ready_ = true;
    return true;
}

ggml_tensor* AudioVAE::decode(VoxCPMContext& ctx, ggml_tensor* z) {
    VOXCPM_ASSERT(z != nullptr);
    VOXCPM_ASSERT(derived_ready_ && "call ensure_derived_weights() before decode()");
    VOXCPM_ASSERT(z->type == GGML_TYPE_F32);
    VOXCPM_ASSERT(z->ne[1] == config_.latent_dim);
    VOXCPM_ASSERT(z->ne[0] >= 1 && z->ne[3] == 1);
    const int64_t ne[3] = {1, config_.decode_hop_length() * z->ne[0], z->ne[2]};
    ggml_tensor* y = ctx.new_node(GGML_TYPE_F32, 3, ne);
    y->op = VOXCPM_OP_AUDIO_VAE_DECODE;
    y->src[0] = z;
    y->extra = this;
    std::snprintf(y->name, sizeof(y->name), "audio_vae.decode");
    ggml_set_output(y);
    return y;
}

std::vector<float> AudioVAE::preprocess(std::vector<float> audio_data, int sample_rate) const {
    const int sr = sample_rate < 0 ? config_.sample_rate : sample_rate;
    VOXCPM_ASSERT(sr == config_.sample_rate);
    const size_t hop = static_cast<size_t>(config_.hop_length());
    audio_data.resize((audio_data.size() + hop - 1) / hop * hop, 0.0f);
    return audio_data;
}

ggml_tensor* AudioVAE::encode(VoxCPMContext& ctx, std::vector<float>& audio_data, int sample_rate) {
    VOXCPM_ASSERT(derived_ready_ && "call ensure_derived_weights() before encode()");
    last_preprocessed_audio_ = preprocess(audio_data, sample_rate);
    const int64_t n = static_cast<int64_t>(last_preprocessed_audio_.size());
    VOXCPM_ASSERT(n > 0);
    last_input_tensor_ = ctx.new_tensor_3d(GGML_TYPE_F32, n, 1, 1);
    ggml_set_input(last_input_tensor_);
    const int64_t ne[3] = {n / config_.hop_length(), config_.latent_dim, 1};
    ggml_tensor* y = ctx.new_node(GGML_TYPE_F32, 3, ne);
    y->op = VOXCPM_OP_AUDIO_VAE_ENCODE;
    y->src[0] = last_input_tensor_;
    y->extra = this;
    std::snprintf(y->name, sizeof(y->name), "audio_vae.encode");
    ggml_set_output(y);
    return y;
}

}  // namespace voxcpm
