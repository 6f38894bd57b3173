// Host tensor of the standalone drop-in build (see zyron/core/tensor.hpp).
#include "zyron/core/tensor.hpp"

#include <algorithm>
#include <limits>
#include <random>

namespace zyron {

void Shape::validate() const {
    for (auto d : dims_)
        if (d == 0) throw std::invalid_argument("ZYRON Shape: dimensions must be > 0");
}

std::size_t Shape::size() const {
    if (dims_.empty()) return 1;
    std::size_t r = 1;
    for (auto d : dims_) {
        if (r > std::numeric_limits<std::size_t>::max() / d)
            throw std::overflow_error("ZYRON Shape: element count overflow");
        r *= d;
    }
    return r;
}

Tensor::Tensor(Shape shape) : shape_(std::move(shape)), size_(shape_.size()) {
    data_ = std::shared_ptr<float[]>(new float[size_]);
}

Tensor Tensor::reshape(const Shape& new_shape) const {
    if (new_shape.size() != size_) throw std::invalid_argument("ZYRON Tensor: reshape size mismatch");
    Tensor t = *this;
    t.shape_ = new_shape;
    return t;
}

Tensor Tensor::zeros(const Shape& shape) {
    Tensor t(shape);
    std::fill_n(t.data(), t.size(), 0.0f);
    return t;
}

// Same generator and distribution as the reference's Tensor::random, so a
// seed gives the same values with the same C++ standard library.
Tensor Tensor::random(const Shape& shape, float low, float high, std::uint32_t seed) {
    if (low > high) throw std::invalid_argument("ZYRON Tensor: random low must be <= high");
    Tensor t(shape);
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> dist(low, high);
    for (std::size_t i = 0; i < t.size(); ++i) t[i] = dist(rng);
    return t;
}

}  // namespace zyron
