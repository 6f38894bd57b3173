// B200 drop-in of src/quantization/quantization.cpp (ZYRON).  Validation,
// messages, storage and the .zyq format follow the reference; quantize(),
// dequantize() and matmul() run on the GPU through include/zq.h.
#include "zyron/quantization/quantization.hpp"

#include "zq.h"

#include <cmath>
#include <cstring>
#include <fstream>
#include <istream>
#include <limits>
#include <mutex>
#include <ostream>
#include <stdexcept>

namespace zyron::quantization {

namespace detail {

struct DeviceWeight {
    std::once_flag once;
    zq_weight* w = nullptr;
    ~DeviceWeight() { zq_weight_destroy(w); }
};

void throw_status(int status) {
    const std::string msg = zq_last_error();
    switch (status) {
        case ZQ_ERR_INVALID_ARGUMENT: throw std::invalid_argument(msg);
        case ZQ_ERR_OUT_OF_RANGE: throw std::out_of_range(msg);
        case ZQ_ERR_OVERFLOW: throw std::overflow_error(msg);
        default: throw std::runtime_error(msg);
    }
}

void check(int status) {
    if (status != ZQ_OK) throw_status(status);
}

}  // namespace detail

namespace {

constexpr std::uint32_t kMagic = 0x315A5951u;  // "QYZ1", quantization.cpp:20
constexpr std::uint32_t kVersion = 1;

void put(std::ostream& out, const void* p, std::size_t n) {
    out.write(static_cast<const char*>(p), static_cast<std::streamsize>(n));
    if (!out) throw std::runtime_error("ZYRON quantization: write failure");
}

void get(std::istream& in, void* p, std::size_t n) {
    in.read(static_cast<char*>(p), static_cast<std::streamsize>(n));
    if (!in) throw std::runtime_error("ZYRON quantization: corrupted file");
}

template <class T>
T get_le(std::istream& in) {
    T v{};
    get(in, &v, sizeof v);
    return v;
}

std::size_t checked_product(std::size_t a, std::size_t b, const char* msg) {
    if (a != 0 && b > std::numeric_limits<std::size_t>::max() / a) throw std::overflow_error(msg);
    return a * b;
}

}  // namespace

QuantizedMatrix::QuantizedMatrix() : device_(std::make_shared<detail::DeviceWeight>()) {}

std::size_t QuantizedMatrix::elements() const noexcept { return empty() ? 0 : rows_ * cols_; }

std::size_t QuantizedMatrix::bytes() const noexcept {
    const std::size_t payload = type_ == Type::Int8 ? int8_data_.size() : int4_data_.size();
    return payload + scales_.size() * sizeof(float);
}

std::size_t QuantizedMatrix::float_bytes() const noexcept { return elements() * sizeof(float); }

double QuantizedMatrix::compression_ratio() const noexcept {
    const auto q = bytes();
    return q == 0 ? 0.0 : static_cast<double>(float_bytes()) / static_cast<double>(q);
}

std::int8_t QuantizedMatrix::value(std::size_t column, std::size_t row) const {
    if (column >= cols_ || row >= rows_) throw std::out_of_range("ZYRON quantization: matrix index out of range");
    const std::size_t linear = checked_product(column, rows_, "ZYRON quantization: index overflow") + row;
    if (type_ == Type::Int8) return int8_data_[linear];
    const std::uint8_t b = int4_data_[linear >> 1];
    const unsigned nib = (linear & 1u) ? (b >> 4) : (b & 0x0Fu);
    return static_cast<std::int8_t>(nib < 8u ? static_cast<int>(nib) : static_cast<int>(nib) - 16);
}

const zq_weight* QuantizedMatrix::device_weight() const {
    if (empty()) throw std::invalid_argument("ZYRON quantization: weights are empty");
    std::call_once(device_->once, [this] {
        const void* payload = type_ == Type::Int8 ? static_cast<const void*>(int8_data_.data())
                                                  : static_cast<const void*>(int4_data_.data());
        const std::size_t n = type_ == Type::Int8 ? int8_data_.size() : int4_data_.size();
        zq_weight* w = nullptr;
        detail::check(zq_weight_create(static_cast<int>(type_), rows_, cols_, scales_.data(), payload, n, nullptr, &w));
        device_->w = w;
    });
    return device_->w;
}

QuantizedMatrix quantize(const Tensor& weights, Type type) {
    if (weights.rank() != 2) throw std::invalid_argument("ZYRON quantization: weights must be rank-2");
    if (!weights.is_contiguous()) throw std::invalid_argument("ZYRON quantization: weights must be contiguous");
    if (type != Type::Int8 && type != Type::Int4) throw std::invalid_argument("ZYRON quantization: unsupported type");

    QuantizedMatrix result;
    result.type_ = type;
    result.rows_ = weights.shape()[0];
    result.cols_ = weights.shape()[1];
    const std::size_t elements =
        checked_product(result.rows_, result.cols_, "ZYRON quantization: matrix size overflow");
    zq_weight* w = nullptr;
    detail::check(zq_weight_quantize_host(weights.data(), result.rows_, result.cols_, static_cast<int>(type), nullptr,
                                          &w));
    std::call_once(result.device_->once, [&] { result.device_->w = w; });
    result.scales_.resize(result.cols_);
    void* payload = nullptr;
    if (type == Type::Int8) {
        result.int8_data_.resize(elements);
        payload = result.int8_data_.data();
    } else {
        result.int4_data_.assign((elements + 1) / 2, 0u);
        payload = result.int4_data_.data();
    }
    detail::check(zq_weight_download(w, result.scales_.data(), payload, nullptr));
    return result;
}

Tensor QuantizedMatrix::dequantize() const {
    Tensor result(Shape{rows_, cols_});  // throws for an empty matrix, as the reference does
    detail::check(zq_dequantize_host(device_weight(), result.data(), nullptr));
    return result;
}

Tensor matmul(const Tensor& input, const QuantizedMatrix& weights) {
    if (input.rank() < 2) throw std::invalid_argument("ZYRON quantization: input rank must be >= 2");
    if (weights.empty()) throw std::invalid_argument("ZYRON quantization: weights are empty");
    if (input.shape()[input.rank() - 1] != weights.rows_)
        throw std::invalid_argument("ZYRON quantization: input/weight dimension mismatch");
    const Tensor x = input.is_contiguous() ? input : input.contiguous();
    const std::size_t m = x.size() / weights.rows_;
    auto dims = x.shape().dims();
    dims.back() = weights.cols_;
    Tensor output{Shape(std::move(dims))};
    detail::check(zq_matmul_host(weights.device_weight(), x.data(), m, nullptr, output.data(), nullptr));
    return output;
}

void QuantizedMatrix::save(const std::string& path) const {
    if (empty()) throw std::runtime_error("ZYRON quantization: cannot save empty matrix");
    std::ofstream out(path, std::ios::binary);
    if (!out) throw std::runtime_error("ZYRON quantization: failed to open: " + path);
    save(out);
}

void QuantizedMatrix::save(std::ostream& out) const {
    if (empty()) throw std::runtime_error("ZYRON quantization: cannot save empty matrix");
    const std::uint32_t h32[3] = {kMagic, kVersion, static_cast<std::uint32_t>(type_)};
    const std::uint64_t h64[3] = {rows_, cols_, scales_.size()};
    put(out, h32, sizeof h32);
    put(out, h64, sizeof h64);
    put(out, scales_.data(), scales_.size() * sizeof(float));
    const std::uint64_t payload = type_ == Type::Int8 ? int8_data_.size() : int4_data_.size();
    put(out, &payload, sizeof payload);
    if (type_ == Type::Int8)
        put(out, int8_data_.data(), int8_data_.size());
    else
        put(out, int4_data_.data(), int4_data_.size());
}

QuantizedMatrix QuantizedMatrix::load(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("ZYRON quantization: failed to open: " + path);
    return load(in);
}

// Same checks in the same order as the reference (quantization.cpp:269-311).
QuantizedMatrix QuantizedMatrix::load(std::istream& in) {
    if (get_le<std::uint32_t>(in) != kMagic || get_le<std::uint32_t>(in) != kVersion)
        throw std::runtime_error("ZYRON quantization: unsupported format");
    QuantizedMatrix r;
    const auto type = get_le<std::uint32_t>(in);
    if (type != static_cast<std::uint32_t>(Type::Int8) && type != static_cast<std::uint32_t>(Type::Int4))
        throw std::runtime_error("ZYRON quantization: invalid type");
    r.type_ = static_cast<Type>(type);
    const auto rows = get_le<std::uint64_t>(in);
    const auto cols = get_le<std::uint64_t>(in);
    if (rows == 0 || cols == 0) throw std::runtime_error("ZYRON quantization: invalid matrix dimensions");
    r.rows_ = static_cast<std::size_t>(rows);
    r.cols_ = static_cast<std::size_t>(cols);
    const std::size_t elements = checked_product(r.rows_, r.cols_, "ZYRON quantization: matrix size overflow");
    if (get_le<std::uint64_t>(in) != r.cols_) throw std::runtime_error("ZYRON quantization: invalid scale count");
    r.scales_.resize(r.cols_);
    get(in, r.scales_.data(), r.scales_.size() * sizeof(float));
    for (float s : r.scales_)
        if (!(s > 0.0f) || !std::isfinite(s)) throw std::runtime_error("ZYRON quantization: invalid scale");
    const auto payload = get_le<std::uint64_t>(in);
    const std::size_t expected = r.type_ == Type::Int8 ? elements : (elements + 1) / 2;
    if (payload != expected) throw std::runtime_error("ZYRON quantization: invalid payload size");
    if (r.type_ == Type::Int8) {
        r.int8_data_.resize(expected);
        get(in, r.int8_data_.data(), expected);
    } else {
        r.int4_data_.resize(expected);
        get(in, r.int4_data_.data(), expected);
    }
    return r;
}

}  // namespace zyron::quantization
