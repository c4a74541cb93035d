// device_decoder.cpp -- nedo::DeviceDecoder (cpp/compat/nedo/device_decoder.hpp)
// over the decoder entry points of include/nedo_gpu.h.
#include "nedo/device_decoder.hpp"

#include <stdexcept>
#include <string>

#include "nedo_gpu.h"

namespace nedo {

namespace {
[[noreturn]] void raise_gpu() { throw std::runtime_error(nedo_gpu_last_error()); }

nedo_gpu_tensor_view view_of(const DeviceTensor& t) {
    nedo_gpu_tensor_view v{};
    if (t.first == nullptr) return v;
    const TensorInfo& ti = *t.first;
    if (ti.shape.size() > 2) throw std::runtime_error("decoder tensor of rank above 2: " + ti.name);
    v.type = static_cast<uint32_t>(ti.type);
    v.ndims = static_cast<uint32_t>(ti.shape.size());
    for (size_t i = 0; i < ti.shape.size(); ++i) v.shape[i] = ti.shape[i];
    if (t.second.size() < ti.n_bytes) throw std::runtime_error("decoder tensor bytes shorter than its shape: " + ti.name);
    v.data = t.second.data();
    v.nbytes = ti.n_bytes;
    return v;
}
}  // namespace

DeviceDecoder::DeviceDecoder(const DeviceDecoderConfig& cfg, const std::vector<DeviceTensor>& tensors) : cfg_(cfg) {
    nedo_gpu_decoder_config c{};
    c.vocab = cfg.vocab;
    c.dim = cfg.dim;
    c.layers = cfg.layers;
    c.heads = cfg.heads;
    c.kv_heads = cfg.kv_heads;
    c.head_dim = cfg.head_dim;
    c.ffn = cfg.ffn;
    c.context = cfg.context;
    c.sliding = cfg.sliding;
    c.morph_layers = cfg.morph_layers;
    c.morph_shared = cfg.morph_shared;
    c.morph_root = cfg.morph_root;
    c.morph_suffix = cfg.morph_suffix;
    c.rms_eps = cfg.rms_eps;
    c.rope_theta = cfg.rope_theta;
    std::vector<nedo_gpu_tensor_view> views;
    views.reserve(tensors.size());
    for (const auto& t : tensors) views.push_back(view_of(t));
    if (nedo_gpu_decoder_create(&c, views.data(), views.size(), &d_) != NEDO_GPU_OK) raise_gpu();
}

DeviceDecoder::~DeviceDecoder() { nedo_gpu_decoder_destroy(d_); }

uint32_t DeviceDecoder::forward(uint32_t token, uint64_t pos, float* logits) {
    uint32_t pick = 0;
    if (nedo_gpu_decoder_forward(d_, token, pos, logits, &pick) != NEDO_GPU_OK) raise_gpu();
    return pick;
}

std::vector<uint32_t> DeviceDecoder::generate(uint32_t token, uint64_t pos, uint32_t n) {
    std::vector<uint32_t> ids(n);
    if (nedo_gpu_decoder_generate(d_, token, pos, n, ids.data()) != NEDO_GPU_OK) raise_gpu();
    return ids;
}

void DeviceDecoder::reset() {
    if (nedo_gpu_decoder_reset(d_) != NEDO_GPU_OK) raise_gpu();
}

}  // namespace nedo
