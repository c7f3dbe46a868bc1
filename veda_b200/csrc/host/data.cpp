// veda::data::Corpus on the device (include/veda/data.hpp).
#include "veda/data.hpp"

#include "veda_cuda.h"

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace veda::data
{

using core::DType;
using core::Shape;
using core::Tensor;

namespace
{
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

cudaStream_t cs() { return reinterpret_cast<cudaStream_t>(current_stream()); }
} // namespace

Corpus::Corpus(std::vector<int64_t> ids, double validation_fraction, uint64_t seed)
    : ids_(std::move(ids)), state_(seed == 0 ? kGolden : seed)
{
    if (validation_fraction < 0.0 || validation_fraction > 1.0)
    {
        throw std::invalid_argument("Corpus: validation_fraction must lie in [0, 1]");
    }
    // the boundary is rounded once, as the reference does (Corpus.cpp:33-39)
    const double kept = 1.0 - validation_fraction;
    boundary_ = static_cast<size_t>(static_cast<double>(ids_.size()) * kept);
    if (boundary_ > ids_.size())
    {
        boundary_ = ids_.size();
    }
    device_ids_ = Tensor::empty(Shape({2 * (ids_.empty() ? 1 : ids_.size())}), DType::F32);
    if (!ids_.empty() &&
        cudaMemcpyAsync(device_ids_.data_ptr(), ids_.data(), ids_.size() * sizeof(int64_t),
                        cudaMemcpyHostToDevice, cs()) != cudaSuccess)
    {
        throw std::runtime_error("Corpus: upload failed");
    }
}

size_t Corpus::size(Split split) const noexcept
{
    return split == Split::Train ? boundary_ : ids_.size() - boundary_;
}

void Corpus::next_batch_into(size_t batch_size, size_t length, Split split, int64_t* inputs,
                             int64_t* targets)
{
    if (batch_size == 0 || length == 0)
    {
        throw std::invalid_argument("Corpus: batch size and length must be positive");
    }
    const size_t begin = split == Split::Train ? 0 : boundary_;
    const size_t end = split == Split::Train ? boundary_ : ids_.size();
    const size_t available = end - begin;
    const size_t window = length + 1;
    if (available < window)
    {
        throw std::invalid_argument(
            "Corpus: the " + std::string(split == Split::Train ? "training" : "validation") +
            " split holds " + std::to_string(available) + " ids, and a window of length " +
            std::to_string(length) + " needs " + std::to_string(window));
    }
    check(veda_corpus_gather(static_cast<const int64_t*>(device_ids_.data_ptr()),
                             static_cast<int64_t>(begin), static_cast<int64_t>(end), state_,
                             static_cast<int64_t>(batch_size), static_cast<int64_t>(length), inputs,
                             targets, current_stream()),
          "Corpus::next_batch");
    state_ += static_cast<uint64_t>(batch_size) * kGolden;   // batch_size draws, one per row
}

Batch Corpus::next_batch(size_t batch_size, size_t length, Split split)
{
    const size_t n = batch_size * length;
    Batch b{Tensor::empty(Shape({2 * (n ? n : 1)}), DType::F32),
            Tensor::empty(Shape({2 * (n ? n : 1)}), DType::F32), Shape({batch_size, length})};
    next_batch_into(batch_size, length, split, static_cast<int64_t*>(b.inputs.data_ptr()),
                    static_cast<int64_t*>(b.targets.data_ptr()));
    return b;
}

} // namespace veda::data
