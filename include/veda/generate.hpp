// Greedy generation on the device from a train::TinyTransformer's weights: the reference's
// generate::Generator (src/libs/generate/Generator.h, Generator.cpp:20-109) with its
// GreedySampler (Sampling.cpp:97-113), the transformer's forward (Model.cpp:154-255) and a KV
// cache (src/libs/model/KVCache.h).
//
// generate() reruns the forward over the whole sequence for every new token; generate_cached()
// prefills the prompt once (keys and values of every layer kept on the device, after QK-norm and
// RoPE) and then feeds one token per step, attending to the cache. A decode step is recorded once
// into a CUDA graph (token, position and every intermediate in fixed device buffers) and replayed
// per token; VEDA_DECODE_GRAPH=0 launches its kernels one by one instead. Both take the last position's
// logits and the first of the largest (ties to the lower id; a NaN logit throws). The reference's
// acceptance rule for the cache is that both give the same tokens.
#pragma once

#include "veda/tensor.hpp"
#include "veda/train.hpp"

#include <cstdint>
#include <vector>

namespace veda::generate
{

struct Options
{
    size_t max_new_tokens = 64;
    std::vector<int32_t> stop_tokens;   // the stop token is never emitted
};

struct Result
{
    std::vector<int32_t> generated;
    bool stopped_on_token = false;
    size_t forward_passes = 0;
};

class Generator
{
public:
    explicit Generator(const train::TinyTransformer& model);

    // std::invalid_argument for an empty prompt, an id outside the vocabulary or a sequence longer
    // than the model's context; std::runtime_error for a NaN logit.
    Result generate(const std::vector<int32_t>& prompt, const Options& options) const;
    Result generate_cached(const std::vector<int32_t>& prompt, const Options& options) const;

    // The logits [V] (fp32 on the host) of the last of `ids` after a full forward: the quantity
    // both loops choose from.
    std::vector<float> last_logits(const std::vector<int32_t>& ids) const;

private:
    struct Cache;
    // Runs the forward over `ids` placed at positions pos0.. (with a cache: its K/V rows for those
    // positions are written and attention reads every cached row up to them) and returns the
    // last position's logits as a device tensor [V].
    core::Tensor forward(const std::vector<int32_t>& ids, size_t pos0, Cache* cache,
                         const core::Tensor& cosines, const core::Tensor& sines) const;
    int32_t pick(const core::Tensor& logits) const;
    struct DecodeStep;
    // Records one decode step (the token and its position read from device buffers, the next
    // token written back, the position advanced) into st's graph.
    void record_step(DecodeStep& st, Cache& cache, const core::Tensor& cosines,
                     const core::Tensor& sines) const;

    const train::TinyTransformer& model_;
};

} // namespace veda::generate
