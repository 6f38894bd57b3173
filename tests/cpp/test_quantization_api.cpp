// C++ tests of the zyron::quantization drop-in (zyron_b200/cpp), in the shape
// of the reference's tests/test_phase5.cpp:94-155 (test_quantization,
// test_quantized_linear): same seeds, shapes and tolerance checks, plus
// bit-exact comparison of every output against the oracle (oracle/zq_oracle.c,
// linked as liboracle.so; test infrastructure only).
#include "zyron/quantization/quantization.hpp"
#include "zyron/quantization/quantized_linear.hpp"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <iostream>
#include <sstream>
#include <stdexcept>
#include <vector>

extern "C" {
void zo_quantize_weights(const float* w, size_t K, size_t N, int type, void* payload, float* scales);
void zo_matmul(const float* x, size_t M, size_t K, int type, const void* payload, const float* col_scale,
               size_t N, const float* bias, int8_t* q_scratch, float* s_scratch, int32_t* acc, float* y);
void zo_dequantize(int type, const void* payload, const float* col_scale, size_t K, size_t N, float* out);
size_t zo_payload_bytes(int type, size_t K, size_t N);
}

namespace {

void check(bool ok, const char* msg) {
    if (!ok) throw std::runtime_error(msg);
}

void same_bits(const float* a, const float* b, size_t n, const char* msg) {
    if (std::memcmp(a, b, n * sizeof(float)) != 0) throw std::runtime_error(msg);
}

template <class F>
void expect_throw_msg(F&& f, const char* want, const char* what) {
    try {
        f();
    } catch (const std::exception& e) {
        if (std::string(e.what()) == want) return;
        throw std::runtime_error(std::string(what) + ": wrong message: " + e.what());
    }
    throw std::runtime_error(std::string(what) + ": no exception");
}

// Matrix product of fp32 inputs with a dequantized weight (the reference
// test's math::matmul comparison).
std::vector<float> ref_fp32(const zyron::Tensor& x, const zyron::Tensor& w, size_t M, size_t K, size_t N) {
    std::vector<float> y(M * N, 0.0f);
    for (size_t m = 0; m < M; ++m)
        for (size_t k = 0; k < K; ++k)
            for (size_t n = 0; n < N; ++n) y[m * N + n] += x[m * K + k] * w[k * N + n];
    return y;
}

void test_quantization() {
    namespace zq = zyron::quantization;
    auto weights = zyron::Tensor::random(zyron::Shape{32, 24}, -1.0f, 1.0f, 21);
    auto input = zyron::Tensor::random(zyron::Shape{7, 32}, -1.0f, 1.0f, 22);
    for (const auto type : {zq::Type::Int8, zq::Type::Int4}) {
        const int t = static_cast<int>(type);
        const auto q = zq::quantize(weights, type);
        check(q.rows() == 32 && q.cols() == 24, "quantized shape");
        check(q.scales().size() == 24, "quantized scales");
        check(q.bytes() < q.float_bytes(), "quantized storage reduction");

        // bit-exact codes and scales vs the oracle
        std::vector<uint8_t> pay(zo_payload_bytes(t, 32, 24));
        std::vector<float> sc(24);
        zo_quantize_weights(weights.data(), 32, 24, t, pay.data(), sc.data());
        same_bits(q.scales().data(), sc.data(), 24, "scales differ from the oracle");
        for (size_t c = 0; c < 24; ++c)
            for (size_t r = 0; r < 32; ++r) {
                const size_t lin = c * 32 + r;
                int want = t == 1 ? (int)(int8_t)pay[lin] : (int)((lin & 1) ? (pay[lin >> 1] >> 4) : (pay[lin >> 1] & 15));
                if (t == 2 && want >= 8) want -= 16;
                check(q.value(c, r) == want, "code differs from the oracle");
            }

        const auto deq = q.dequantize();
        std::vector<float> deq_o(32 * 24);
        zo_dequantize(t, pay.data(), sc.data(), 32, 24, deq_o.data());
        same_bits(deq.data(), deq_o.data(), deq_o.size(), "dequantize differs from the oracle");
        float max_error = 0.0f;
        for (size_t i = 0; i < weights.size(); ++i) max_error = std::max(max_error, std::fabs(weights[i] - deq[i]));
        check(max_error < (type == zq::Type::Int8 ? 0.02f : 0.2f), "quantization error");

        const auto qout = zq::matmul(input, q);
        std::vector<int8_t> qs(7 * 32);
        std::vector<float> ss(7), yo(7 * 24);
        zo_matmul(input.data(), 7, 32, t, pay.data(), sc.data(), 24, nullptr, qs.data(), ss.data(), nullptr, yo.data());
        same_bits(qout.data(), yo.data(), yo.size(), "matmul differs from the oracle");
        const auto fp = ref_fp32(input, deq, 7, 32, 24);
        const float tol = type == zq::Type::Int8 ? 0.15f : 0.5f;
        for (size_t i = 0; i < fp.size(); ++i) check(std::fabs(fp[i] - qout[i]) <= tol, "quantized matmul mismatch");

        const auto path = std::filesystem::temp_directory_path() /
                          (type == zq::Type::Int8 ? "zyron_b200_q8.zyq" : "zyron_b200_q4.zyq");
        q.save(path.string());
        const auto loaded = zq::QuantizedMatrix::load(path.string());
        const auto a = q.dequantize();
        const auto b = loaded.dequantize();
        same_bits(a.data(), b.data(), a.size(), "quantized serialization mismatch");
        std::filesystem::remove(path);

        // copies share one device upload and give identical results
        const zq::QuantizedMatrix copy = loaded;
        check(copy.device_weight() == loaded.device_weight(), "copies should share the device weight");
        const auto y2 = zq::matmul(input, copy);
        same_bits(y2.data(), qout.data(), qout.size(), "copy matmul differs");
    }
}

void test_quantized_linear() {
    namespace zq = zyron::quantization;
    auto weight = zyron::Tensor::random(zyron::Shape{16, 8}, -0.5f, 0.5f, 31);
    auto bias = zyron::Tensor::random(zyron::Shape{8}, -0.2f, 0.2f, 32);
    auto input = zyron::Tensor::random(zyron::Shape{4, 5, 16}, -1.0f, 1.0f, 33);
    for (const auto type : {zq::Type::Int8, zq::Type::Int4}) {
        const int t = static_cast<int>(type);
        zq::QuantizedLinear lin(weight, &bias, type);
        auto out = lin.forward(input);
        check(out.shape() == zyron::Shape({4, 5, 8}), "linear output shape");
        std::vector<uint8_t> pay(zo_payload_bytes(t, 16, 8));
        std::vector<float> sc(8), yo(20 * 8), ss(20);
        std::vector<int8_t> qs(20 * 16);
        zo_quantize_weights(weight.data(), 16, 8, t, pay.data(), sc.data());
        zo_matmul(input.data(), 20, 16, t, pay.data(), sc.data(), 8, bias.data(), qs.data(), ss.data(), nullptr,
                  yo.data());
        same_bits(out.data(), yo.data(), yo.size(), "QuantizedLinear differs from the oracle");
        auto fp = ref_fp32(input, weight, 20, 16, 8);
        for (size_t r = 0; r < 20; ++r)
            for (size_t c = 0; c < 8; ++c) fp[r * 8 + c] += bias[c];
        const float tol = type == zq::Type::Int8 ? 0.2f : 0.6f;
        for (size_t i = 0; i < fp.size(); ++i) check(std::fabs(fp[i] - out[i]) <= tol, "quantized linear mismatch");
    }
}

void test_errors() {
    namespace zq = zyron::quantization;
    zq::QuantizedMatrix empty;
    auto x = zyron::Tensor::random(zyron::Shape{2, 4}, -1, 1, 1);
    expect_throw_msg([&] { (void)zq::matmul(x, empty); }, "ZYRON quantization: weights are empty", "empty weights");
    auto v = zyron::Tensor::random(zyron::Shape{4}, -1, 1, 1);
    expect_throw_msg([&] { (void)zq::matmul(v, empty); }, "ZYRON quantization: input rank must be >= 2", "rank");
    auto w = zq::quantize(zyron::Tensor::random(zyron::Shape{5, 3}, -1, 1, 2), zq::Type::Int8);
    expect_throw_msg([&] { (void)zq::matmul(x, w); }, "ZYRON quantization: input/weight dimension mismatch", "dims");
    expect_throw_msg([&] { (void)w.value(3, 0); }, "ZYRON quantization: matrix index out of range", "value");
    expect_throw_msg([&] { (void)zq::quantize(x.reshape(zyron::Shape{2, 2, 2}), zq::Type::Int8); },
                     "ZYRON quantization: weights must be rank-2", "quantize rank");
    std::stringstream bad("QYZ");
    expect_throw_msg([&] { (void)zq::QuantizedMatrix::load(bad); }, "ZYRON quantization: corrupted file", "load");
    std::stringstream ss;
    w.save(ss);
    std::string s = ss.str();
    s[8] = 7;
    std::stringstream bad2(s);
    expect_throw_msg([&] { (void)zq::QuantizedMatrix::load(bad2); }, "ZYRON quantization: invalid type", "type");
    expect_throw_msg([&] { zq::QuantizedLinear l(empty); }, "ZYRON QuantizedLinear: weight cannot be empty", "linear");
    auto b = zyron::Tensor::random(zyron::Shape{4}, -1, 1, 3);
    expect_throw_msg([&] { zq::QuantizedLinear l(w, b); }, "ZYRON QuantizedLinear: bias shape mismatch", "bias");
}

}  // namespace

int main() {
    try {
        test_quantization();
        test_quantized_linear();
        test_errors();
        std::cout << "zyron_b200 C++ quantization API tests: PASS\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "zyron_b200 C++ quantization API tests: FAIL: " << e.what() << '\n';
        return 1;
    }
}
