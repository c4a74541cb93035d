// device_decoder.hpp -- the device-resident decode forward pass for
// NedoModel::generate_ids (src/model.cpp:151-281), declared for the reference's
// include/ tree (a maintainer adds this header there) and implemented in
// libnedo_kernels_cuda.so over the C ABI of include/nedo_gpu.h.
//
// One DeviceDecoder holds a model's weights and its fp32 KV cache on the GPU.
// forward(token, pos, logits) replaces the `forward` lambda of generate_ids
// (src/model.cpp:212-260): the same sequence of steps for one token at one
// position, with the LM-head logits copied into `logits` (vocab floats) when
// it is non-null; it returns the greedy pick (the first index of the largest
// logit, as std::max_element).  generate(token, pos, n) runs n greedy passes
// with the loop on the device (each pass fed the previous pick) and returns
// the n picks.  Errors throw std::runtime_error with the reference's messages
// where it has them ("invalid GQA dimensions", "context_length is zero",
// "prompt token id out of range", "bad RMSNorm tensor: <name>", ...).
#pragma once

#include <cstdint>
#include <span>
#include <utility>
#include <vector>

#include "nedo/gguf.hpp"

struct nedo_gpu_decoder;

namespace nedo {

// The fields of ModelConfig (include/nedo/model.hpp:12-16) the pass uses.
struct DeviceDecoderConfig {
    uint32_t vocab = 0, dim = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, ffn = 0, context = 0, sliding = 0;
    uint32_t morph_layers = 0, morph_shared = 0, morph_root = 0, morph_suffix = 0;
    float rms_eps = 1e-5f, rope_theta = 10000.f;
};

// A tensor and its bytes (GgufFile::bytes, src/gguf.cpp:139); a null info = absent.
using DeviceTensor = std::pair<const TensorInfo*, std::span<const std::byte>>;

class DeviceDecoder {
public:
    // tensors: token_embd, output_norm, output (null info: tied to token_embd),
    // the MorphFFN routing table (null info: none), then per layer attn_norm,
    // attn_q, attn_k, attn_v, attn_output, ffn_norm, ffn_gate, ffn_up, ffn_down --
    // the TensorInfo pointers NedoModel::load_schema resolves (src/model.cpp:94-118).
    DeviceDecoder(const DeviceDecoderConfig& cfg, const std::vector<DeviceTensor>& tensors);
    ~DeviceDecoder();
    DeviceDecoder(const DeviceDecoder&) = delete;
    DeviceDecoder& operator=(const DeviceDecoder&) = delete;

    uint32_t forward(uint32_t token, uint64_t pos, float* logits = nullptr);
    std::vector<uint32_t> generate(uint32_t token, uint64_t pos, uint32_t n);
    void reset();
    const DeviceDecoderConfig& config() const noexcept { return cfg_; }

private:
    DeviceDecoderConfig cfg_;
    nedo_gpu_decoder* d_ = nullptr;
};

}  // namespace nedo
