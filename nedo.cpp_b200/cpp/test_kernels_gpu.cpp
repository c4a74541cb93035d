// test_kernels_gpu.cpp -- nedo.cpp's kernel known-answer tests (tests/test_kernels.cpp:33-65),
// run through the drop-in nedo::kernels::matvec / embedding_row, i.e. on the GPU.
// Same harness shape as the reference: plain int return codes, "ok" on success.
// Added cases: an F16 row, a multi-row Q8_0 matrix large enough for the
// streaming kernel, the drop-in's batched matvec (512 token vectors), and the
// reference's error messages.
#include <cmath>
#include <cstring>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "nedo/kernels.hpp"

namespace {
bool near(float a, float b, float eps = 1e-4f) { return std::abs(a - b) <= eps; }

int test_q8_matvec() {  // tests/test_kernels.cpp:33-44
    nedo::TensorInfo t{"q8", {32, 1}, nedo::TensorType::Q8_0};
    std::vector<std::byte> w(34);
    const uint16_t one = nedo::kernels::fp32_to_fp16(1.f);
    std::memcpy(w.data(), &one, 2);
    for (int i = 0; i < 32; ++i) w[2 + i] = std::byte(static_cast<unsigned char>(static_cast<int8_t>(i - 16)));
    float x[32];
    for (float& v : x) v = 1.f;
    float y = 0.f;
    nedo::kernels::matvec(t, w, x, &y);
    return near(y, -16.f) ? 0 : 3;
}

int test_q4_matvec_and_embedding() {  // tests/test_kernels.cpp:46-65
    nedo::TensorInfo t{"q4", {32, 1}, nedo::TensorType::Q4_0};
    std::vector<std::byte> w(18);
    const uint16_t one = nedo::kernels::fp32_to_fp16(1.f);
    std::memcpy(w.data(), &one, 2);
    for (int i = 0; i < 16; ++i) w[2 + i] = std::byte(static_cast<unsigned char>(((15 - i) << 4) | i));
    float x[32];
    for (float& v : x) v = 1.f;
    float y = 0.f;
    nedo::kernels::matvec(t, w, x, &y);
    if (!near(y, -16.f)) return 4;
    float row[32]{};
    nedo::kernels::embedding_row(t, w, 0, row);
    for (int i = 0; i < 16; ++i)
        if (!near(row[i], float(i - 8)) || !near(row[i + 16], float(7 - i))) return 5;
    return 0;
}

int test_f16_matvec() {
    nedo::TensorInfo t{"f16", {40, 2}, nedo::TensorType::F16};
    std::vector<std::byte> w(2 * 40 * 2);
    for (int r = 0; r < 2; ++r)
        for (int i = 0; i < 40; ++i) {
            const uint16_t h = nedo::kernels::fp32_to_fp16(r == 0 ? 0.5f : float(i % 5) - 2.f);
            std::memcpy(w.data() + 2 * (r * 40 + i), &h, 2);
        }
    float x[40];
    for (int i = 0; i < 40; ++i) x[i] = float(i);
    float y[2]{};
    nedo::kernels::matvec(t, w, x, y);
    float e1 = 0.f;
    for (int i = 0; i < 40; ++i) e1 += (float(i % 5) - 2.f) * float(i);
    return (near(y[0], 0.5f * 780.f, 1e-3f) && near(y[1], e1, 1e-3f)) ? 0 : 7;
}

int test_q8_many_rows() {
    // 300 rows x 512 columns: goes through the streaming kernel.
    const int rows = 300, cols = 512, nb = cols / 32;
    nedo::TensorInfo t{"q8big", {uint64_t(cols), uint64_t(rows)}, nedo::TensorType::Q8_0};
    std::vector<std::byte> w(size_t(rows) * nb * 34);
    std::vector<float> x(cols), y(rows), expect(rows, 0.f);
    for (int i = 0; i < cols; ++i) x[i] = float((i * 7) % 11) - 5.f;
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < nb; ++b) {
            std::byte* blk = w.data() + (size_t(r) * nb + b) * 34;
            const float d = float(1 + (r + b) % 4) * 0.25f;
            const uint16_t h = nedo::kernels::fp32_to_fp16(d);
            std::memcpy(blk, &h, 2);
            float s = 0.f;
            for (int i = 0; i < 32; ++i) {
                const int8_t q = int8_t(((r * 31 + b * 17 + i * 5) % 255) - 127);
                blk[2 + i] = std::byte(static_cast<unsigned char>(q));
                s += float(q) * x[b * 32 + i];
            }
            expect[r] += d * s;
        }
    nedo::kernels::matvec(t, w, x.data(), y.data());
    for (int r = 0; r < rows; ++r)
        if (!near(y[r], expect[r], 1e-3f * (1.f + std::abs(expect[r])))) return 8;
    return 0;
}

int test_q8_batch() {
    // The drop-in's added matvec_batch: 512 token vectors through one Q8_0
    // 300 x 1024 weight (the batched tensor-core path), each checked against
    // its serial dot product computed here in double.  Weights and x are small
    // integers times powers of two, exact in every arithmetic the GPU may use.
    const int rows = 300, cols = 1024, nb = cols / 32, batch = 512;
    nedo::TensorInfo t{"q8batch", {uint64_t(cols), uint64_t(rows)}, nedo::TensorType::Q8_0};
    std::vector<std::byte> w(size_t(rows) * nb * 34);
    std::vector<float> deq(size_t(rows) * cols);
    for (int r = 0; r < rows; ++r)
        for (int b = 0; b < nb; ++b) {
            std::byte* blk = w.data() + (size_t(r) * nb + b) * 34;
            const float d = float(1 + (r + 3 * b) % 4) * 0.25f;
            const uint16_t h = nedo::kernels::fp32_to_fp16(d);
            std::memcpy(blk, &h, 2);
            for (int i = 0; i < 32; ++i) {
                const int8_t q = int8_t(((r * 29 + b * 13 + i * 7) % 255) - 127);
                blk[2 + i] = std::byte(static_cast<unsigned char>(q));
                deq[size_t(r) * cols + b * 32 + i] = d * float(q);
            }
        }
    std::vector<float> x(size_t(batch) * cols), y(size_t(batch) * rows);
    for (int k = 0; k < batch; ++k)
        for (int i = 0; i < cols; ++i) x[size_t(k) * cols + i] = float((i * 7 + k * 3) % 11) - 5.f;
    nedo::kernels::matvec_batch(t, w, x.data(), y.data(), batch);
    for (int k = 0; k < batch; ++k)
        for (int r = 0; r < rows; ++r) {
            double e = 0.0, a = 0.0;
            for (int i = 0; i < cols; ++i) {
                const double p = double(deq[size_t(r) * cols + i]) * double(x[size_t(k) * cols + i]);
                e += p;
                a += std::abs(p);
            }
            if (std::abs(double(y[size_t(k) * rows + r]) - e) > 1e-4 * a) return 14;
        }
    return 0;
}

template <typename F>
bool throws_with(F&& f, const std::string& msg) {
    try {
        f();
    } catch (const std::runtime_error& e) {
        return std::string(e.what()).find(msg) != std::string::npos;
    }
    return false;
}

int test_errors() {
    float x[64]{}, y[4]{};
    std::vector<std::byte> w(4 * 64 * 4);
    nedo::TensorInfo rank1{"r1", {64}, nedo::TensorType::Q8_0};
    if (!throws_with([&] { nedo::kernels::matvec(rank1, w, x, y); }, "matvec requires rank-2 tensor: r1")) return 9;
    nedo::TensorInfo odd{"odd", {48, 2}, nedo::TensorType::Q4_0};
    if (!throws_with([&] { nedo::kernels::matvec(odd, w, x, y); }, "Q4_0 elements not block aligned")) return 10;
    nedo::TensorInfo f32{"f32", {64, 2}, nedo::TensorType::F32};
    if (!throws_with([&] { nedo::kernels::matvec(f32, w, x, y); }, "matvec tensor type not supported")) return 11;
    nedo::TensorInfo q4k{"q4k", {256, 2}, nedo::TensorType::Q4_K};
    if (!throws_with([&] { nedo::kernels::matvec(q4k, w, x, y); }, "tensor type not implemented: 12")) return 12;
    nedo::TensorInfo q8{"q8", {64, 2}, nedo::TensorType::Q8_0};
    if (!throws_with([&] { nedo::kernels::embedding_row(q8, w, 2, y); }, "bad embedding row")) return 13;
    if (!throws_with([&] { nedo::kernels::matvec_batch(rank1, w, x, y, 2); }, "matvec requires rank-2 tensor: r1"))
        return 15;
    if (!throws_with([&] { nedo::kernels::matvec_batch(f32, w, x, y, 2); }, "matvec tensor type not supported"))
        return 16;
    return 0;
}
}  // namespace

int main() {
    if (int rc = test_q8_matvec()) return rc;
    if (int rc = test_q4_matvec_and_embedding()) return rc;
    if (int rc = test_f16_matvec()) return rc;
    if (int rc = test_q8_many_rows()) return rc;
    if (int rc = test_q8_batch()) return rc;
    if (int rc = test_errors()) return rc;
    std::cout << "ok\n";
    return 0;
}
