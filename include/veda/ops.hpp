// veda::ops — the reference's tensor-level operations that its tests and callers use directly
// (src/libs/ops/Elementwise.h:19-23, src/libs/ops/Softmax.h:25, 42), on device tensors. Pure
// functions as in the reference: inputs in, a fresh contiguous tensor out; operands broadcast
// numpy-style; any view is accepted. Errors keep the reference's exception types
// (std::invalid_argument for shapes and dimensions).
#pragma once

#include "veda/tensor.hpp"

#include <cstddef>

namespace veda::ops
{

core::Tensor add(const core::Tensor& a, const core::Tensor& b);
core::Tensor mul(const core::Tensor& a, const core::Tensor& b);
core::Tensor add(const core::Tensor& a, float scalar);
core::Tensor mul(const core::Tensor& a, float scalar);

// softmax / log_softmax along `dim` (src/libs/ops/Softmax.cpp:20-151).
core::Tensor softmax(const core::Tensor& tensor, size_t dim);
core::Tensor log_softmax(const core::Tensor& tensor, size_t dim);

} // namespace veda::ops
