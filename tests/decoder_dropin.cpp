// Test program: the C++ drop-in nedo::DeviceDecoder driven the way
// NedoModel::generate_ids would drive it (src/model.cpp:151-281), on a GGUF
// file read by a minimal test-side reader (header, metadata, tensor infos;
// src/gguf.cpp:78-104 describes the format).
//
// usage: decoder_dropin <model.gguf> <out.bin> <n_generate> <prompt_len> <token>...
// Runs forward() teacher-forced over the given tokens (position = index),
// writing every pass's logits, then a fresh sequence: the first prompt_len - 1
// tokens through forward() and generate(n) from token prompt_len - 1.  out.bin: u32 passes, u32 vocab, f32 logits[passes][vocab],
// u32 n, u32 picks_of_forward[passes], u32 generated[n].
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "nedo/device_decoder.hpp"

namespace {

struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    template <class T>
    T get() {
        if (static_cast<size_t>(end - p) < sizeof(T)) throw std::runtime_error("truncated GGUF");
        T v;
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
};

// metadata values as double (numbers) or skipped (strings, arrays)
double value(Reader& r, uint32_t t, bool* numeric) {
    *numeric = true;
    switch (t) {
        case 0: return r.get<uint8_t>();
        case 1: return r.get<int8_t>();
        case 2: return r.get<uint16_t>();
        case 3: return r.get<int16_t>();
        case 4: return r.get<uint32_t>();
        case 5: return r.get<int32_t>();
        case 6: return r.get<float>();
        case 7: return r.get<uint8_t>();
        case 10: return static_cast<double>(r.get<uint64_t>());
        case 11: return static_cast<double>(r.get<int64_t>());
        case 12: return r.get<double>();
        case 8: r.str(); *numeric = false; return 0;
        case 9: {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t n = r.get<uint64_t>();
            bool num = false;
            for (uint64_t i = 0; i < n; ++i) value(r, et, &num);
            *numeric = false;
            return static_cast<double>(n);
        }
        default: throw std::runtime_error("bad GGUF value type");
    }
}

uint64_t nbytes(uint32_t type, uint64_t n) {
    switch (type) {
        case 0: return 4 * n;
        case 1: return 2 * n;
        case 2: return n / 32 * 18;
        case 8: return n / 32 * 34;
        default: throw std::runtime_error("tensor type not used by the test models");
    }
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 6) {
        std::fprintf(stderr, "usage: %s model.gguf out.bin n_generate prompt_len token...\n", argv[0]);
        return 2;
    }
    try {
        const int fd = ::open(argv[1], O_RDONLY);
        if (fd < 0) throw std::runtime_error("cannot open GGUF");
        struct stat st {};
        fstat(fd, &st);
        const auto* base = static_cast<const uint8_t*>(mmap(nullptr, st.st_size, PROT_READ, MAP_PRIVATE, fd, 0));
        Reader r{base, base + st.st_size};
        if (r.get<uint32_t>() != 0x46554747u) throw std::runtime_error("not a GGUF file (bad magic)");
        r.get<uint32_t>();
        const uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
        std::map<std::string, double> md;
        uint64_t ntokens = 0;
        for (uint64_t i = 0; i < nkv; ++i) {
            const std::string k = r.str();
            const uint32_t t = r.get<uint32_t>();
            bool num = false;
            const double v = value(r, t, &num);
            if (num) md[k] = v;
            if (k == "tokenizer.ggml.tokens") ntokens = static_cast<uint64_t>(v);
        }
        const uint64_t align = md.count("general.alignment") ? static_cast<uint64_t>(md["general.alignment"]) : 32;
        std::map<std::string, nedo::TensorInfo> infos;
        std::vector<std::string> order;
        for (uint64_t i = 0; i < nt; ++i) {
            nedo::TensorInfo ti;
            ti.name = r.str();
            const uint32_t nd = r.get<uint32_t>();
            ti.n_elements = 1;
            for (uint32_t d = 0; d < nd; ++d) {
                ti.shape.push_back(r.get<uint64_t>());
                ti.n_elements *= ti.shape.back();
            }
            ti.type = static_cast<nedo::TensorType>(r.get<uint32_t>());
            ti.relative_offset = r.get<uint64_t>();
            ti.n_bytes = nbytes(static_cast<uint32_t>(ti.type), ti.n_elements);
            order.push_back(ti.name);
            infos[ti.name] = ti;
        }
        const uint64_t data = (static_cast<uint64_t>(r.p - base) + align - 1) / align * align;
        for (auto& kv : infos) kv.second.absolute_offset = data + kv.second.relative_offset;
        auto u = [&](const char* k, double def) { return static_cast<uint32_t>(md.count(k) ? md[k] : def); };
        nedo::DeviceDecoderConfig c;
        c.vocab = u("nedolm.vocab_size", static_cast<double>(ntokens));
        c.dim = u("nedolm.embedding_length", 1536);
        c.layers = u("nedolm.block_count", 24);
        c.heads = u("nedolm.attention.head_count", 12);
        c.kv_heads = u("nedolm.attention.head_count_kv", 4);
        c.head_dim = u("nedolm.rope.dimension_count", c.heads ? c.dim / c.heads : 0);
        c.ffn = u("nedolm.feed_forward_length", 5632);
        c.context = u("nedolm.context_length", 4096);
        c.sliding = u("nedolm.attention.sliding_window", 2048);
        c.morph_layers = u("nedolm.morph.layer_count", 0);
        c.morph_shared = u("nedolm.morph.shared_width", 0);
        c.morph_root = u("nedolm.morph.root_width", 0);
        c.morph_suffix = u("nedolm.morph.suffix_width", 0);
        c.rms_eps = static_cast<float>(md.count("nedolm.attention.layer_norm_rms_epsilon")
                                           ? md["nedolm.attention.layer_norm_rms_epsilon"] : 1e-5);
        c.rope_theta = static_cast<float>(md.count("nedolm.rope.freq_base") ? md["nedolm.rope.freq_base"] : 10000.0);
        auto tensor = [&](const std::string& name) -> nedo::DeviceTensor {
            auto it = infos.find(name);
            if (it == infos.end()) return {nullptr, {}};
            const nedo::TensorInfo& ti = it->second;
            return {&ti, std::span<const std::byte>(reinterpret_cast<const std::byte*>(base + ti.absolute_offset),
                                                    ti.n_bytes)};
        };
        std::vector<nedo::DeviceTensor> ts = {tensor("token_embd.weight"), tensor("output_norm.weight"),
                                              tensor("output.weight"), tensor("blk.0.ffn_gate_tid2eid.weight")};
        static const char* kLayer[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                        "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
        for (uint32_t li = 0; li < c.layers; ++li)
            for (const char* k : kLayer) ts.push_back(tensor("blk." + std::to_string(li) + "." + k + ".weight"));
        nedo::DeviceDecoder dec(c, ts);
        const uint32_t ngen = static_cast<uint32_t>(std::atoi(argv[3]));
        const size_t plen = static_cast<size_t>(std::atoi(argv[4]));
        std::vector<uint32_t> seq;
        for (int i = 5; i < argc; ++i) seq.push_back(static_cast<uint32_t>(std::atoi(argv[i])));
        if (plen == 0 || plen > seq.size()) throw std::runtime_error("prompt_len out of range");
        const uint32_t vocab = static_cast<uint32_t>((infos.count("output.weight") ? infos["output.weight"]
                                                                                  : infos["token_embd.weight"]).shape[1]);
        std::vector<float> logits(static_cast<size_t>(seq.size()) * vocab);
        std::vector<uint32_t> picks(seq.size());
        for (size_t pos = 0; pos < seq.size(); ++pos)
            picks[pos] = dec.forward(seq[pos], pos, logits.data() + pos * vocab);
        // a fresh sequence: the prompt but its last token through forward, then the device loop
        dec.reset();
        for (size_t pos = 0; pos + 1 < plen; ++pos) dec.forward(seq[pos], pos);
        const std::vector<uint32_t> gen = dec.generate(seq[plen - 1], plen - 1, ngen);
        FILE* f = std::fopen(argv[2], "wb");
        const uint32_t passes = static_cast<uint32_t>(seq.size());
        std::fwrite(&passes, 4, 1, f);
        std::fwrite(&vocab, 4, 1, f);
        std::fwrite(logits.data(), 4, logits.size(), f);
        std::fwrite(&ngen, 4, 1, f);
        std::fwrite(picks.data(), 4, picks.size(), f);
        std::fwrite(gen.data(), 4, gen.size(), f);
        std::fclose(f);
        // an argument error surfaces as the reference's message
        try {
            dec.forward(c.vocab, 0);
            std::fprintf(stderr, "no error for an out-of-range token\n");
            return 4;
        } catch (const std::runtime_error& e) {
            if (std::string(e.what()).find("prompt token id out of range") == std::string::npos) return 5;
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    std::printf("ok\n");
    return 0;
}
