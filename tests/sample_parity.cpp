// Sampling parity through the C++ drop-in: nedo::kernels::sample_lm_head (LM
// head matvec on the GPU, top-k on the device, the reference's draw on the
// host) against the reference's sampler (restated in oracle/sample_ref.hpp,
// src/model.cpp:33-63) fed the logits of the same GPU matvec, with two
// generators started from the same seed.  Every draw must pick the same token
// and leave the generators in the same state.  Prints "ok <draws>".
#include <cstdint>
#include <cstring>
#include <iostream>
#include <random>
#include <vector>

#include "nedo/kernels.hpp"
#include "sample_ref.hpp"

int main() {
    const uint32_t vocab = 32000, dim = 2048;
    nedo::TensorInfo head{"output.weight", {dim, vocab}, nedo::TensorType::F16};
    std::vector<std::byte> w(size_t(vocab) * dim * 2);
    std::mt19937_64 gen(12345);
    std::normal_distribution<float> nd(0.f, 0.02f);
    for (size_t i = 0; i < size_t(vocab) * dim; ++i) {
        const uint16_t h = nedo::kernels::fp32_to_fp16(nd(gen));
        std::memcpy(w.data() + 2 * i, &h, 2);
    }
    struct Cfg {
        float t;
        uint32_t k;
        float p;
    };
    const Cfg cfgs[] = {{0.8f, 40, 0.95f}, {1.0f, 1, 0.9f}, {0.5f, 256, 0.5f}, {1.3f, 300, 0.99f},
                        {0.8f, 0, 0.95f},  {0.7f, 40, 1.0f}, {0.f, 40, 0.95f},  {2.0f, 100, 0.0f}};
    std::vector<float> x(dim), logits(vocab);
    uint32_t draws = 0;
    for (uint32_t xi = 0; xi < 3; ++xi) {
        std::normal_distribution<float> xd(0.f, 1.f + float(xi));
        for (float& v : x) v = xd(gen);
        nedo::kernels::matvec(head, w, x.data(), logits.data());
        for (const Cfg& c : cfgs) {
            for (uint64_t seed = 1; seed <= 4; ++seed) {
                std::mt19937_64 ra(seed * 7919 + xi), rb(seed * 7919 + xi);
                for (int d = 0; d < 6; ++d) {
                    const uint32_t a = oracle_ref::sample_token(logits, c.t, c.k, c.p, ra);
                    const uint32_t b = nedo::kernels::sample_lm_head(head, w, x.data(), c.t, c.k, c.p, rb);
                    ++draws;
                    if (a != b) {
                        std::cout << "mismatch t=" << c.t << " k=" << c.k << " p=" << c.p << " seed=" << seed
                                  << " draw=" << d << ": reference " << a << " drop-in " << b << "\n";
                        return 1;
                    }
                }
                if (!(ra == rb)) {
                    std::cout << "generator states differ t=" << c.t << " k=" << c.k << "\n";
                    return 2;
                }
            }
        }
    }
    std::cout << "ok " << draws << "\n";
    return 0;
}
