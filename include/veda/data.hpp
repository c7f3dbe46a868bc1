// veda::data::Corpus on the device: the reference's batcher (src/libs/data/Corpus.h,
// Corpus.cpp:25-107) with the ids resident in device memory and each batch gathered there.
//
// Same constructor, split rule (cut once by position at size * (1 - validation_fraction)),
// generator (splitmix64, seed 0 meaning 0x9E3779B97F4A7C15) and draw order as the reference, so
// a Corpus built from the same ids and seed yields bit-identical batches in the same sequence.
// next_batch returns device int64 [B*T] inputs and targets, ready for Trainer::step.
#pragma once

#include "veda/tensor.hpp"

#include <cstdint>
#include <vector>

namespace veda::data
{

enum class Split
{
    Train,
    Validation
};

struct Batch
{
    core::Tensor inputs;    // device int64 [B*T] (8-byte elements, held as pairs of fp32 slots)
    core::Tensor targets;   // device int64 [B*T], each the successor of the input beside it
    core::Shape shape;      // [B, T]
};

class Corpus
{
public:
    // std::invalid_argument if validation_fraction lies outside [0, 1] (Corpus.cpp:25-31).
    Corpus(std::vector<int64_t> ids, double validation_fraction, uint64_t seed);

    // B windows of length + 1 ids at random offsets inside the split; std::invalid_argument for an
    // empty batch or a split shorter than one window (Corpus.cpp:64-90).
    Batch next_batch(size_t batch_size, size_t length, Split split);
    // The same into caller-provided device buffers of batch_size * length int64 each.
    void next_batch_into(size_t batch_size, size_t length, Split split, int64_t* inputs,
                         int64_t* targets);

    size_t size(Split split) const noexcept;
    const std::vector<int64_t>& ids() const noexcept { return ids_; }
    size_t boundary() const noexcept { return boundary_; }

private:
    std::vector<int64_t> ids_;
    core::Tensor device_ids_;
    size_t boundary_ = 0;
    uint64_t state_ = 0;
};

} // namespace veda::data
