// zyron/core/tensor.hpp -- host fp32 tensor for the standalone drop-in build.
//
// The quantized matmul path uses only this part of the reference's
// zyron::Tensor interface (include/zyron/core/tensor.hpp:16-67 of ZYRON):
// construction from a Shape, shape()/rank()/size(), data(), operator[],
// is_contiguous()/contiguous(), reshape() and the seeded random()/zeros()
// factories.  Inside a ZYRON checkout the reference's own tensor.hpp is used
// instead; the drop-in sources compile against either.  Storage here is
// always contiguous and shared between copies (like the reference's Memory).
#pragma once

#include <cstddef>
#include <cstdint>
#include <initializer_list>
#include <memory>
#include <stdexcept>
#include <vector>

namespace zyron {

class Shape {
public:
    Shape() = default;
    Shape(std::initializer_list<std::size_t> dims) : dims_(dims) { validate(); }
    explicit Shape(std::vector<std::size_t> dims) : dims_(std::move(dims)) { validate(); }

    [[nodiscard]] std::size_t rank() const noexcept { return dims_.size(); }
    [[nodiscard]] std::size_t size() const;
    [[nodiscard]] const std::vector<std::size_t>& dims() const noexcept { return dims_; }
    [[nodiscard]] std::size_t operator[](std::size_t i) const { return dims_.at(i); }
    [[nodiscard]] bool empty() const noexcept { return dims_.empty(); }
    friend bool operator==(const Shape& a, const Shape& b) noexcept { return a.dims_ == b.dims_; }
    friend bool operator!=(const Shape& a, const Shape& b) noexcept { return !(a == b); }

private:
    void validate() const;
    std::vector<std::size_t> dims_;
};

class Tensor {
public:
    Tensor() = default;
    explicit Tensor(Shape shape);

    [[nodiscard]] const Shape& shape() const noexcept { return shape_; }
    [[nodiscard]] std::size_t rank() const noexcept { return shape_.rank(); }
    [[nodiscard]] std::size_t size() const noexcept { return size_; }
    [[nodiscard]] bool is_contiguous() const noexcept { return true; }

    float* data() noexcept { return data_.get(); }
    const float* data() const noexcept { return data_.get(); }
    float& operator[](std::size_t i) noexcept { return data_.get()[i]; }
    const float& operator[](std::size_t i) const noexcept { return data_.get()[i]; }

    [[nodiscard]] Tensor contiguous() const { return *this; }
    [[nodiscard]] Tensor reshape(const Shape& new_shape) const;

    static Tensor zeros(const Shape& shape);
    static Tensor random(const Shape& shape, float low = 0.0f, float high = 1.0f, std::uint32_t seed = 0);

private:
    Shape shape_{};
    std::size_t size_{0};
    std::shared_ptr<float[]> data_{};
};

}  // namespace zyron
