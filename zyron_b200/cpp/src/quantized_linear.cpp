// B200 drop-in of src/quantization/quantized_linear.cpp (ZYRON): same
// constructors, validation and messages; forward() runs the quantized matmul
// with the bias add fused into the kernel epilogue.
#include "zyron/quantization/quantized_linear.hpp"

#include "zq.h"

#include <stdexcept>
#include <utility>

namespace zyron::quantization {

QuantizedLinear::QuantizedLinear(QuantizedMatrix weight, Tensor bias)
    : weight_(std::move(weight)), bias_(std::move(bias)) {
    if (weight_.empty()) throw std::invalid_argument("ZYRON QuantizedLinear: weight cannot be empty");
    if (bias_.size() != 0 && (bias_.rank() != 1 || bias_.size() != weight_.cols()))
        throw std::invalid_argument("ZYRON QuantizedLinear: bias shape mismatch");
}

QuantizedLinear::QuantizedLinear(const Tensor& weight, const Tensor* bias, Type type)
    : weight_(quantize(weight, type)) {
    if (weight.rank() != 2) throw std::invalid_argument("ZYRON QuantizedLinear: weight must be rank-2");
    if (bias) {
        if (bias->rank() != 1 || bias->shape()[0] != weight.shape()[1])
            throw std::invalid_argument("ZYRON QuantizedLinear: bias shape mismatch");
        bias_ = *bias;
    }
}

Tensor QuantizedLinear::forward(const Tensor& input) const {
    if (input.rank() < 2) throw std::invalid_argument("ZYRON QuantizedLinear: input rank must be >= 2");
    if (input.shape()[input.rank() - 1] != in_features())
        throw std::invalid_argument("ZYRON QuantizedLinear: input feature mismatch");
    if (bias_.size() == 0) return matmul(input, weight_);
    const Tensor x = input.is_contiguous() ? input : input.contiguous();
    const std::size_t m = x.size() / in_features();
    auto dims = x.shape().dims();
    dims.back() = out_features();
    Tensor output{Shape(std::move(dims))};
    detail::check(zq_matmul_host(weight_.device_weight(), x.data(), m, bias_.data(), output.data(), nullptr));
    return output;
}

}  // namespace zyron::quantization
