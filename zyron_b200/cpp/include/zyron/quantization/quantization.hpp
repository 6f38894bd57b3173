// zyron/quantization/quantization.hpp -- B200 drop-in of ZYRON's
// zyron::quantization API (reference: include/zyron/quantization/
// quantization.hpp:11-60).  Same types, signatures, accessors, exceptions
// and messages; the arithmetic runs in sm_100a CUDA kernels behind the C ABI
// of include/zq.h.  The host copy of the codes is kept (value(), scales(),
// save() and bytes() behave exactly as in the reference); the device copy is
// uploaded once, on first use, and shared by all copies of the matrix.
#pragma once

#include "zyron/core/tensor.hpp"

#include <cstddef>
#include <cstdint>
#include <iosfwd>
#include <memory>
#include <string>
#include <vector>

struct zq_weight;

namespace zyron::quantization {

enum class Type : std::uint8_t {
    Int8 = 1,
    Int4 = 2,
};

namespace detail {
struct DeviceWeight;  // owns the zq_weight handle (quantization.cpp)
}

class QuantizedMatrix {
public:
    QuantizedMatrix();

    [[nodiscard]] Type type() const noexcept { return type_; }
    [[nodiscard]] std::size_t rows() const noexcept { return rows_; }
    [[nodiscard]] std::size_t cols() const noexcept { return cols_; }
    [[nodiscard]] std::size_t elements() const noexcept;
    [[nodiscard]] std::size_t bytes() const noexcept;
    [[nodiscard]] std::size_t float_bytes() const noexcept;
    [[nodiscard]] double compression_ratio() const noexcept;
    [[nodiscard]] const std::vector<float>& scales() const noexcept { return scales_; }
    [[nodiscard]] std::int8_t value(std::size_t column, std::size_t row) const;
    [[nodiscard]] bool empty() const noexcept { return rows_ == 0 || cols_ == 0; }

    [[nodiscard]] Tensor dequantize() const;

    void save(const std::string& path) const;
    static QuantizedMatrix load(const std::string& path);
    void save(std::ostream& out) const;
    static QuantizedMatrix load(std::istream& in);

    // The device-resident copy on the current device, uploaded on first call
    // (thread-safe).  Throws std::invalid_argument for an empty matrix.
    [[nodiscard]] const zq_weight* device_weight() const;

private:
    Type type_{Type::Int8};
    std::size_t rows_{0};
    std::size_t cols_{0};
    // Column-major storage as in the reference: (row, col) at col*rows + row.
    std::vector<std::int8_t> int8_data_;
    std::vector<std::uint8_t> int4_data_;
    std::vector<float> scales_;
    std::shared_ptr<detail::DeviceWeight> device_;

    friend QuantizedMatrix quantize(const Tensor&, Type);
    friend Tensor matmul(const Tensor&, const QuantizedMatrix&);
};

[[nodiscard]] QuantizedMatrix quantize(const Tensor& weights, Type type);

// Inference-only matmul. The activation is dynamically quantized per row and
// the weight uses symmetric per-output-column INT8 or packed INT4 scales.
[[nodiscard]] Tensor matmul(const Tensor& input, const QuantizedMatrix& weights);

namespace detail {
// Throws the exception type the reference uses for a zq_status.
[[noreturn]] void throw_status(int status);
void check(int status);
}  // namespace detail

}  // namespace zyron::quantization
