// Test infrastructure (oracle side): runs the REFERENCE's own decode loop,
// NedoModel::generate_ids (src/model.cpp:151-281), compiled from the reference
// sources, on a GGUF file, and records the LM-head logits of every forward
// pass (src/model.cpp:258-259).  The logits are captured by wrapping the
// reference's nedo::kernels::matvec at link time (-Wl,--wrap): the wrapper
// calls the reference implementation unchanged and copies its output when the
// tensor is the head.  Nothing under the product links or runs this file.
//
// usage: ref_decode <model.gguf> <out.bin> <max_new_tokens> <temperature> <top_k> <top_p> <seed> <prompt id>...
// out.bin: u32 steps, u32 vocab, f32 logits[steps][vocab], u32 generated, u32 ids[generated]
#include <cstdio>
#include <cstdlib>
#include <exception>
#include <span>
#include <string>
#include <vector>

#include "nedo/kernels.hpp"
#include "nedo/model.hpp"

static std::string g_head;
static std::vector<float> g_logits;
static uint64_t g_vocab = 0;

#define MATVEC_SYM _ZN4nedo7kernels6matvecERKNS_10TensorInfoESt4spanIKSt4byteLm18446744073709551615EEPKfPf
#define CAT2(a, b) a##b
#define CAT(a, b) CAT2(a, b)

extern "C" void CAT(__real_, MATVEC_SYM)(const nedo::TensorInfo& t, std::span<const std::byte> b, const float* x,
                                         float* y);
extern "C" void CAT(__wrap_, MATVEC_SYM)(const nedo::TensorInfo& t, std::span<const std::byte> b, const float* x,
                                         float* y) {
    CAT(__real_, MATVEC_SYM)(t, b, x, y);
    if (t.name == g_head) {
        g_vocab = t.shape[1];
        g_logits.insert(g_logits.end(), y, y + t.shape[1]);
    }
}

int main(int argc, char** argv) {
    if (argc < 9) {
        std::fprintf(stderr, "usage: %s model.gguf out.bin max_new temperature top_k top_p seed prompt_id...\n", argv[0]);
        return 2;
    }
    try {
        nedo::NedoModel m(argv[1]);
        g_head = m.gguf().tensor("output.weight") ? "output.weight" : "token_embd.weight";
        nedo::GenerationConfig gc;
        gc.max_new_tokens = static_cast<uint32_t>(std::atoi(argv[3]));
        gc.temperature = static_cast<float>(std::atof(argv[4]));
        gc.top_k = static_cast<uint32_t>(std::atoi(argv[5]));
        gc.top_p = static_cast<float>(std::atof(argv[6]));
        gc.seed = std::strtoull(argv[7], nullptr, 10);
        gc.add_bos = false;
        std::vector<uint32_t> prompt;
        for (int i = 8; i < argc; ++i) prompt.push_back(static_cast<uint32_t>(std::atoi(argv[i])));
        const auto ids = m.generate_ids(prompt, gc);
        FILE* f = std::fopen(argv[2], "wb");
        if (!f) return 3;
        const uint32_t vocab = static_cast<uint32_t>(g_vocab);
        const uint32_t steps = vocab ? static_cast<uint32_t>(g_logits.size() / vocab) : 0u;
        const uint32_t n = static_cast<uint32_t>(ids.size());
        std::fwrite(&steps, 4, 1, f);
        std::fwrite(&vocab, 4, 1, f);
        std::fwrite(g_logits.data(), 4, g_logits.size(), f);
        std::fwrite(&n, 4, 1, f);
        std::fwrite(ids.data(), 4, ids.size(), f);
        std::fclose(f);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    return 0;
}
